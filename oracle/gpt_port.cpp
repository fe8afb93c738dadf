// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
//
// Stand-alone CPU restatement of the IndexTTS 2.5 GPT decode path of the
// reference (src/gpt.cpp, src/gpt_sampling.cpp), used as the parity checker
// for the CUDA library and as the "port" CPU baseline.  Kernel math lives in
// cpu_math.hpp.  Differences from the reference, all deliberate:
//   * the layer count is read from the bundle (1..24) so that parity tests can
//     run a shallow model in seconds; the reference insists on 24 (gpt.cpp:8-23);
//   * an optional Philox4x32-10 uniform stream (rng = 1) next to the
//     reference's SplitMix64 (rng = 0, gpt_sampling.cpp:11-26).
// Exceptions are mapped to status codes at the C boundary:
//   0 ok, -1 std::invalid_argument, -2 std::runtime_error, -3 std::logic_error,
//   -9 anything else.
#include <cstring>
#include <limits>
#include <memory>
#include <numeric>
#include <string>

#include "cpu_math.hpp"
#include "mit2_reader.hpp"

namespace orc {

constexpr uint32_t kWidth = 1280, kHeads = 20, kHeadDim = 64, kFfn = 5120, kVocab = 8194,
                   kCapacity = 4096, kMaxLayers = 24;

// Same layout as itts_gen_opts in include/itts_gpt.h.
struct Opts {
    int32_t do_sample;
    uint32_t top_k;
    uint64_t seed;
    float temperature;
    float top_p;
    float repetition_penalty;
    uint32_t num_beams;
    float length_penalty;
    int32_t rng;
};

// gpt_sampling.cpp:11-26
struct SplitMix64 {
    uint64_t state;
    explicit SplitMix64(uint64_t s) : state(s) {}
    uint64_t next_u64() {
        uint64_t z = (state += 0x9E3779B97F4A7C15ULL);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
        return z ^ (z >> 31);
    }
};

// Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC'11): counter = (draw_lo, draw_hi, 0, 0),
// key = (seed_lo, seed_hi); the first two output words form the 64-bit draw.
inline void philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = uint64_t(0xD2511F53u) * c0, p1 = uint64_t(0xCD9E8D57u) * c2;
        const uint32_t n0 = uint32_t(p1 >> 32) ^ c1 ^ k0, n1 = uint32_t(p1);
        const uint32_t n2 = uint32_t(p0 >> 32) ^ c3 ^ k1, n3 = uint32_t(p0);
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

inline uint64_t philox_u64(uint64_t seed, uint64_t draw) {
    const uint32_t ctr[4] = {uint32_t(draw), uint32_t(draw >> 32), 0, 0}, key[2] = {uint32_t(seed), uint32_t(seed >> 32)};
    uint32_t o[4];
    philox4x32_10(ctr, key, o);
    return (uint64_t(o[0]) << 32) | o[1];
}

struct Uniform {
    int mode;
    uint64_t seed, draws = 0;
    SplitMix64 sm;
    Uniform(int m, uint64_t s) : mode(m), seed(s), sm(s) {}
    double next() {
        const uint64_t u = mode == 1 ? philox_u64(seed, draws) : sm.next_u64();
        ++draws;
        return static_cast<double>(u >> 11) * (1.0 / 9007199254740992.0);
    }
};

// gpt_sampling.cpp:28-128
std::vector<float> apply_processors(const std::vector<float>& logits, const std::vector<uint32_t>& history,
                                    const Opts& c) {
    std::vector<float> scores = logits;
    constexpr float neg_inf = -std::numeric_limits<float>::infinity();
    if (c.repetition_penalty != 1.0f) {
        if (c.repetition_penalty <= 0.0f) throw std::runtime_error("GPT repetition penalty must be positive");
        std::vector<uint8_t> seen(scores.size(), 0);
        for (uint32_t tok : history) {
            if (tok >= scores.size() || seen[tok]) continue;
            seen[tok] = 1;
            scores[tok] = scores[tok] < 0.0f ? scores[tok] * c.repetition_penalty : scores[tok] / c.repetition_penalty;
        }
    }
    if (c.temperature <= 0.0f) throw std::runtime_error("GPT sampling temperature must be positive");
    if (c.temperature != 1.0f)
        for (float& s : scores) s /= c.temperature;
    if (c.top_k > 0 && c.top_k < scores.size()) {
        std::vector<float> sorted = scores;
        const size_t kth = size_t(std::max(c.top_k, c.num_beams > 1 ? 2u : 1u) - 1);
        std::nth_element(sorted.begin(), sorted.begin() + kth, sorted.end(), std::greater<float>());
        const float pivot = sorted[kth];
        for (float& s : scores)
            if (s < pivot) s = neg_inf;
    }
    if (c.top_p < 1.0f) {
        if (c.top_p <= 0.0f) throw std::runtime_error("GPT top_p must be in (0, 1]");
        std::vector<size_t> order(scores.size());
        std::iota(order.begin(), order.end(), size_t(0));
        std::sort(order.begin(), order.end(), [&](size_t a, size_t b) {
            return scores[a] == scores[b] ? a < b : scores[a] < scores[b];
        });
        float mx = neg_inf;
        for (float s : scores)
            if (std::isfinite(s)) mx = std::max(mx, s);
        if (!std::isfinite(mx)) throw std::runtime_error("GPT top_p filtering removed all logits");
        double total = 0.0;
        std::vector<double> probs(scores.size(), 0.0);
        for (size_t i = 0; i < scores.size(); ++i)
            if (std::isfinite(scores[i])) {
                probs[i] = std::exp(static_cast<double>(scores[i] - mx));
                total += probs[i];
            }
        if (total <= 0.0) throw std::runtime_error("GPT sampling probability mass is zero");
        double cum = 0.0;
        std::vector<uint8_t> remove(scores.size(), 0);
        const double low = 1.0 - static_cast<double>(c.top_p);
        size_t finite = 0;
        for (size_t idx : order) {
            if (!std::isfinite(scores[idx])) { remove[idx] = 1; continue; }
            ++finite;
            cum += probs[idx] / total;
            if (cum <= low) remove[idx] = 1;
        }
        if (finite > 0)
            for (size_t i = 0; i < std::min(order.size(), c.num_beams > 1 ? size_t(2) : size_t(1)); ++i)
                remove[order[order.size() - 1 - i]] = 0;
        for (size_t i = 0; i < scores.size(); ++i)
            if (remove[i]) scores[i] = neg_inf;
    }
    return scores;
}

// gpt_sampling.cpp:130-165
uint32_t sample_token(const std::vector<float>& s, Uniform& rng) {
    float mx = -std::numeric_limits<float>::infinity();
    for (float v : s)
        if (std::isfinite(v)) mx = std::max(mx, v);
    if (!std::isfinite(mx)) throw std::runtime_error("GPT sampling received no finite logits");
    double total = 0.0;
    std::vector<double> probs(s.size(), 0.0);
    for (size_t i = 0; i < s.size(); ++i)
        if (std::isfinite(s[i])) {
            probs[i] = std::exp(static_cast<double>(s[i] - mx));
            total += probs[i];
        }
    if (total <= 0.0) throw std::runtime_error("GPT sampling probability mass is zero");
    const double target = rng.next() * total;
    double cum = 0.0;
    uint32_t last = 0;
    for (uint32_t i = 0; i < probs.size(); ++i) {
        if (probs[i] <= 0.0) continue;
        last = i;
        cum += probs[i];
        if (target < cum) return i;
    }
    return last;
}

struct Layer {
    const float *ln1g, *ln1b, *ln2g, *ln2b, *bqkv, *bo, *bfc, *bmp;
    std::vector<float> wqkv, wo, wfc, wmp;  // row-major [out, in]
};

struct State {
    uint32_t tokens;
    std::vector<float> kv;  // [layer][K|V][tokens][width]
};

struct Model {
    Bundle b;
    uint32_t layers = 0, mel_pos_rows = 0, text_pos_rows = 0;
    std::vector<Layer> L;
    const float *mel_emb, *mel_pos, *text_emb, *text_pos, *lang_emb, *spk_w, *spk_b;
    const float *lnf_g, *lnf_b, *fn_g, *fn_b, *head_w, *head_b;
    std::unique_ptr<float[]> kv;  // [layer][K|V][capacity][width]
    uint32_t cached = 0;

    explicit Model(const std::string& dir) : b(dir) {
        auto shape = [&](const std::string& n, std::vector<int64_t> want) {
            if (b.info(n).shape != want) throw std::runtime_error("Unsupported 2.5 GPT shape: " + n);
        };
        shape("gpt.spk_emb_proj.weight", {1280, 192});
        shape("gpt.text_embedding.weight", {60510, 1280});
        shape("gpt.lang_embedding.weight", {107, 1280});
        shape("gpt.mel_embedding.weight", {8194, 1280});
        while (layers < kMaxLayers && b.find("gpt.gpt.h." + std::to_string(layers) + ".ln_1.weight")) ++layers;
        if (!layers) throw std::runtime_error("bundle has no GPT layers");
        mel_pos_rows = uint32_t(b.info("gpt.mel_pos_embedding.emb.weight").shape[0]);
        text_pos_rows = uint32_t(b.info("gpt.text_pos_embedding.emb.weight").shape[0]);
        mel_emb = b.f32("gpt.mel_embedding.weight");
        mel_pos = b.f32("gpt.mel_pos_embedding.emb.weight");
        text_emb = b.f32("gpt.text_embedding.weight");
        text_pos = b.f32("gpt.text_pos_embedding.emb.weight");
        lang_emb = b.f32("gpt.lang_embedding.weight");
        spk_w = b.f32("gpt.spk_emb_proj.weight");
        spk_b = b.f32("gpt.spk_emb_proj.bias");
        lnf_g = b.f32("gpt.gpt.ln_f.weight");
        lnf_b = b.f32("gpt.gpt.ln_f.bias");
        fn_g = b.f32("gpt.final_norm.weight");
        fn_b = b.f32("gpt.final_norm.bias");
        head_w = b.f32("gpt.mel_head.weight");
        head_b = b.f32("gpt.mel_head.bias");
        L.resize(layers);
        for (uint32_t i = 0; i < layers; ++i) {
            const std::string p = "gpt.gpt.h." + std::to_string(i);
            shape(p + ".attn.c_attn.weight", {1280, 3840});
            shape(p + ".attn.c_proj.weight", {1280, 1280});
            shape(p + ".mlp.c_fc.weight", {1280, 5120});
            shape(p + ".mlp.c_proj.weight", {5120, 1280});
            Layer& l = L[i];
            l.ln1g = b.f32(p + ".ln_1.weight");
            l.ln1b = b.f32(p + ".ln_1.bias");
            l.ln2g = b.f32(p + ".ln_2.weight");
            l.ln2b = b.f32(p + ".ln_2.bias");
            l.bqkv = b.f32(p + ".attn.c_attn.bias");
            l.bo = b.f32(p + ".attn.c_proj.bias");
            l.bfc = b.f32(p + ".mlp.c_fc.bias");
            l.bmp = b.f32(p + ".mlp.c_proj.bias");
            l.wqkv = transpose(b.f32(p + ".attn.c_attn.weight"), kWidth, 3 * kWidth);
            l.wo = transpose(b.f32(p + ".attn.c_proj.weight"), kWidth, kWidth);
            l.wfc = transpose(b.f32(p + ".mlp.c_fc.weight"), kWidth, kFfn);
            l.wmp = transpose(b.f32(p + ".mlp.c_proj.weight"), kFfn, kWidth);
        }
        kv.reset(new float[size_t(layers) * 2 * kCapacity * kWidth]);
    }
    float* K(uint32_t l) { return kv.get() + (size_t(l) * 2) * kCapacity * kWidth; }
    float* V(uint32_t l) { return kv.get() + (size_t(l) * 2 + 1) * kCapacity * kWidth; }

    // gpt.cpp:42-71
    std::vector<float> prepare(const std::vector<float>& speaker, const std::vector<float>& emotion,
                               const std::vector<uint32_t>& text, uint32_t language) {
        if (speaker.size() != 192 || emotion.size() != kWidth || language >= 107)
            throw std::invalid_argument("Invalid GPT conditioning dimensions");
        std::vector<uint32_t> ids{0};
        for (auto id : text) {
            if (id >= 60510) throw std::invalid_argument("Text token is outside 2.5 vocabulary");
            if (id != 0 && id != 1) ids.push_back(id);
        }
        ids.push_back(1);
        if (ids.size() > 602 || ids.size() > text_pos_rows)
            throw std::invalid_argument("Text segment exceeds GPT position capacity");
        std::vector<float> prefix(3 * kWidth, 0.0f), proj(kWidth);
        linear_rows(spk_w, spk_b, speaker.data(), 1, kWidth, 192, proj.data());
        for (uint32_t i = 0; i < kWidth; ++i) prefix[i] = proj[i] + emotion[i];
        for (size_t r = 0; r < ids.size(); ++r)
            for (uint32_t i = 0; i < kWidth; ++i)
                prefix.push_back((text_emb[size_t(ids[r]) * kWidth + i] + text_pos[r * kWidth + i]) +
                                 lang_emb[size_t(language) * kWidth + i]);
        for (uint32_t i = 0; i < kWidth; ++i)
            prefix.push_back(mel_emb[size_t(8192) * kWidth + i] + mel_pos[i]);
        return prefix;
    }

    // gpt.cpp:88-125
    std::vector<float> run(const float* input, uint32_t t, bool initial, uint32_t code, uint32_t pos) {
        std::vector<float> hidden(size_t(t) * kWidth);
        if (initial) {
            std::memcpy(hidden.data(), input, hidden.size() * 4);
        } else {
            for (uint32_t i = 0; i < kWidth; ++i)
                hidden[i] = mel_emb[size_t(code) * kWidth + i] + mel_pos[size_t(pos) * kWidth + i];
        }
        std::vector<float> x(size_t(t) * kWidth), qkv(size_t(t) * 3 * kWidth), att(size_t(t) * kWidth),
            proj(size_t(t) * kWidth), r(size_t(t) * kWidth), ff(size_t(t) * kFfn);
        for (uint32_t li = 0; li < layers; ++li) {
            const Layer& l = L[li];
            layernorm_rows(hidden.data(), l.ln1g, l.ln1b, t, kWidth, 1e-5f, x.data());
            linear_rows(l.wqkv.data(), l.bqkv, x.data(), t, 3 * kWidth, kWidth, qkv.data());
            if (initial) {
                for (uint32_t tk = 0; tk < t; ++tk) {
                    std::memcpy(K(li) + size_t(tk) * kWidth, qkv.data() + size_t(tk) * 3 * kWidth + kWidth, kWidth * 4);
                    std::memcpy(V(li) + size_t(tk) * kWidth, qkv.data() + size_t(tk) * 3 * kWidth + 2 * kWidth, kWidth * 4);
                }
                causal_attention(qkv.data(), t, kHeads, kHeadDim, att.data());
            } else {
                cached_attention(K(li), V(li), qkv.data(), cached, kHeads, kHeadDim, att.data());
                std::memcpy(K(li) + size_t(cached) * kWidth, qkv.data() + kWidth, kWidth * 4);
                std::memcpy(V(li) + size_t(cached) * kWidth, qkv.data() + 2 * kWidth, kWidth * 4);
            }
            linear_rows(l.wo.data(), l.bo, att.data(), t, kWidth, kWidth, proj.data());
            for (size_t i = 0; i < r.size(); ++i) r[i] = hidden[i] + proj[i];
            layernorm_rows(r.data(), l.ln2g, l.ln2b, t, kWidth, 1e-5f, x.data());
            linear_rows(l.wfc.data(), l.bfc, x.data(), t, kFfn, kWidth, ff.data());
            for (float& v : ff) v = gelu(v);
            linear_rows(l.wmp.data(), l.bmp, ff.data(), t, kWidth, kFfn, proj.data());
            for (size_t i = 0; i < hidden.size(); ++i) hidden[i] = r[i] + proj[i];
        }
        std::vector<float> a(kWidth), c(kWidth), logits(kVocab);
        layernorm_rows(hidden.data() + size_t(t - 1) * kWidth, lnf_g, lnf_b, 1, kWidth, 1e-5f, a.data());
        layernorm_rows(a.data(), fn_g, fn_b, 1, kWidth, 1e-5f, c.data());
        linear_rows(head_w, head_b, c.data(), 1, kVocab, kWidth, logits.data());
        return logits;
    }

    // gpt.cpp:72-78
    std::vector<float> prefill(const std::vector<float>& prefix) {
        if (prefix.empty() || prefix.size() % kWidth || prefix.size() / kWidth > 1024)
            throw std::invalid_argument("Invalid GPT prefill dimensions");
        auto out = run(prefix.data(), uint32_t(prefix.size() / kWidth), true, 0, 0);
        cached = uint32_t(prefix.size() / kWidth);
        return out;
    }
    // gpt.cpp:79-85
    std::vector<float> step(uint32_t code, uint32_t pos) {
        if (!cached || cached >= kCapacity || code >= kVocab || pos >= mel_pos_rows)
            throw std::invalid_argument("GPT step requires valid cache, code and position");
        auto out = run(nullptr, 1, false, code, pos);
        ++cached;
        return out;
    }
    std::shared_ptr<State> checkpoint() {
        if (!cached) throw std::invalid_argument("Invalid KV snapshot");
        auto s = std::make_shared<State>();
        s->tokens = cached;
        s->kv.resize(size_t(layers) * 2 * cached * kWidth);
        for (uint32_t l = 0; l < layers; ++l) {
            std::memcpy(s->kv.data() + (size_t(l) * 2) * cached * kWidth, K(l), size_t(cached) * kWidth * 4);
            std::memcpy(s->kv.data() + (size_t(l) * 2 + 1) * cached * kWidth, V(l), size_t(cached) * kWidth * 4);
        }
        return s;
    }
    void restore(const State& s) {
        for (uint32_t l = 0; l < layers; ++l) {
            std::memcpy(K(l), s.kv.data() + (size_t(l) * 2) * s.tokens * kWidth, size_t(s.tokens) * kWidth * 4);
            std::memcpy(V(l), s.kv.data() + (size_t(l) * 2 + 1) * s.tokens * kWidth, size_t(s.tokens) * kWidth * 4);
        }
        cached = s.tokens;
    }

    // gpt_sampling.cpp:168-189
    std::vector<uint32_t> generate(const std::vector<float>& prefix, const Opts& options, uint32_t maximum,
                                   bool& stopped) {
        if (!maximum || maximum + 1 >= mel_pos_rows || prefix.size() / kWidth + maximum >= kCapacity)
            throw std::invalid_argument("GPT generation capacity exceeded");
        Opts c = options;
        if (!c.do_sample) { c.temperature = 1; c.top_k = 0; c.top_p = 1; }
        if (!std::isfinite(c.temperature) || !std::isfinite(c.top_p) || !std::isfinite(c.repetition_penalty) ||
            c.temperature <= 0 || c.top_p <= 0 || c.top_p > 1 || c.repetition_penalty <= 0)
            throw std::invalid_argument("Invalid GPT generation parameters");
        if (!c.num_beams || c.num_beams > 10 || !std::isfinite(c.length_penalty))
            throw std::invalid_argument("Invalid beam search configuration");
        stopped = false;
        if (c.num_beams > 1) return beams(prefix, c, maximum, stopped);
        Uniform rng(c.rng, c.seed);
        std::vector<uint32_t> codes, history{1, 8192};
        auto logits = prefill(prefix);
        for (uint32_t i = 0; i < maximum; ++i) {
            auto scores = apply_processors(logits, history, c);
            const uint32_t token = c.do_sample ? sample_token(scores, rng)
                                               : uint32_t(std::max_element(scores.begin(), scores.end()) - scores.begin());
            if (token == 8193) { stopped = true; break; }
            if (token >= 8192) throw std::runtime_error("GPT generated invalid semantic code");
            codes.push_back(token);
            history.push_back(token);
            if (i + 1 < maximum) logits = step(token, i + 2);
        }
        return codes;
    }

    // gpt_sampling.cpp:190-245
    std::vector<uint32_t> beams(const std::vector<float>& prefix, const Opts& c, uint32_t maximum, bool& eos_out) {
        struct Beam { std::vector<uint32_t> codes; float score = 0; std::vector<float> logits; std::shared_ptr<State> state; };
        struct Finished { std::vector<uint32_t> codes; double score; bool eos; };
        struct Cand { uint32_t parent, token; float score; };
        Uniform rng(c.rng, c.seed);
        std::vector<Finished> finished;
        Beam init;
        init.logits = prefill(prefix);
        init.state = checkpoint();
        std::vector<Beam> bs(c.num_beams, init);
        for (uint32_t i = 1; i < bs.size(); ++i) bs[i].score = -1e9f;
        auto finish = [&](const Beam& beam, float score, uint32_t length, bool eos) {
            finished.push_back({beam.codes, score / std::pow(static_cast<double>(std::max(length, 1u)), c.length_penalty), eos});
            std::sort(finished.begin(), finished.end(), [](const Finished& a, const Finished& b) { return a.score > b.score; });
            if (finished.size() > c.num_beams) finished.resize(c.num_beams);
        };
        for (uint32_t si = 0; si < maximum; ++si) {
            std::vector<Cand> cands;
            std::vector<float> all;
            for (uint32_t p = 0; p < bs.size(); ++p) {
                auto lp = bs[p].logits;
                float peak = *std::max_element(lp.begin(), lp.end()), sum = 0;
                for (auto v : lp) sum += std::exp(v - peak);
                float log_sum = peak + std::log(sum);
                for (auto& v : lp) v -= log_sum;
                std::vector<uint32_t> history{1, 8192};
                history.insert(history.end(), bs[p].codes.begin(), bs[p].codes.end());
                auto scores = apply_processors(lp, history, c);
                for (auto& v : scores) v += bs[p].score;
                all.insert(all.end(), scores.begin(), scores.end());
            }
            const uint32_t take = 2 * c.num_beams;
            if (c.do_sample) {
                auto avail = all;
                for (uint32_t i = 0; i < take; ++i) {
                    const uint32_t id = sample_token(avail, rng);
                    cands.push_back({id / kVocab, id % kVocab, all[id]});
                    avail[id] = -std::numeric_limits<float>::infinity();
                }
            } else {
                std::vector<uint32_t> order(all.size());
                std::iota(order.begin(), order.end(), 0u);
                std::partial_sort(order.begin(), order.begin() + take, order.end(), [&](uint32_t a, uint32_t b) {
                    return all[a] == all[b] ? a < b : all[a] > all[b];
                });
                for (uint32_t i = 0; i < take; ++i) cands.push_back({order[i] / kVocab, order[i] % kVocab, all[order[i]]});
            }
            std::sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) { return a.score > b.score; });
            std::vector<Beam> next;
            for (uint32_t rank = 0; rank < cands.size(); ++rank) {
                const Cand cand = cands[rank];
                const Beam& parent = bs[cand.parent];
                if (cand.token == 8193) {
                    if (rank < c.num_beams) finish(parent, cand.score, si + 1, true);
                    continue;
                }
                if (cand.token >= 8192) throw std::runtime_error("Beam generated invalid semantic code");
                Beam child;
                child.codes = parent.codes;
                child.codes.push_back(cand.token);
                child.score = cand.score;
                if (si + 1 < maximum) {
                    restore(*parent.state);
                    child.logits = step(cand.token, si + 2);
                    child.state = checkpoint();
                }
                next.push_back(std::move(child));
                if (next.size() == c.num_beams) break;
            }
            if (next.empty()) break;
            bs = std::move(next);
            if (finished.size() == c.num_beams &&
                finished.back().score >= cands[0].score / std::pow(static_cast<double>(si + 1), c.length_penalty)) {
                bs.clear();
                break;
            }
        }
        for (const auto& beam : bs) finish(beam, beam.score, uint32_t(beam.codes.size()), false);
        if (finished.empty()) throw std::runtime_error("Beam search produced no hypotheses");
        eos_out = finished[0].eos;
        return finished[0].codes;
    }
};

thread_local std::string g_error;

template <class F>
int guard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_error = e.what();
        return -1;
    } catch (const std::logic_error& e) {
        g_error = e.what();
        return -3;
    } catch (const std::runtime_error& e) {
        g_error = e.what();
        return -2;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -9;
    }
}

}  // namespace orc

using orc::guard;

extern "C" {

const char* orc_last_error() { return orc::g_error.c_str(); }

int orc_threads() { return orc::pool().size(); }

void* orc_load(const char* dir) {
    orc::Model* m = nullptr;
    if (guard([&] { m = new orc::Model(dir); })) return nullptr;
    return m;
}

void orc_free(void* m) { delete static_cast<orc::Model*>(m); }

uint32_t orc_layers(void* m) { return static_cast<orc::Model*>(m)->layers; }
uint32_t orc_cached_tokens(void* m) { return static_cast<orc::Model*>(m)->cached; }
uint32_t orc_mel_pos_rows(void* m) { return static_cast<orc::Model*>(m)->mel_pos_rows; }

int orc_prepare(void* h, const float* spk, size_t spk_n, const float* emo, size_t emo_n, const uint32_t* ids,
                size_t n, uint32_t lang, float* out, size_t cap_floats, size_t* rows) {
    return guard([&] {
        auto p = static_cast<orc::Model*>(h)->prepare(std::vector<float>(spk, spk + spk_n),
                                                      std::vector<float>(emo, emo + emo_n),
                                                      std::vector<uint32_t>(ids, ids + n), lang);
        if (p.size() > cap_floats) throw std::invalid_argument("output buffer too small");
        std::memcpy(out, p.data(), p.size() * 4);
        *rows = p.size() / orc::kWidth;
    });
}

int orc_prefill(void* h, const float* prefix, size_t n_floats, float* logits) {
    return guard([&] {
        auto l = static_cast<orc::Model*>(h)->prefill(std::vector<float>(prefix, prefix + n_floats));
        std::memcpy(logits, l.data(), l.size() * 4);
    });
}

int orc_step(void* h, uint32_t code, uint32_t pos, float* logits) {
    return guard([&] {
        auto l = static_cast<orc::Model*>(h)->step(code, pos);
        std::memcpy(logits, l.data(), l.size() * 4);
    });
}

int orc_generate(void* h, const float* prefix, size_t n_floats, const orc::Opts* opts, uint32_t maximum,
                 uint32_t* codes, uint32_t* n_codes, int* stopped) {
    return guard([&] {
        bool st = false;
        auto c = static_cast<orc::Model*>(h)->generate(std::vector<float>(prefix, prefix + n_floats), *opts, maximum, st);
        std::memcpy(codes, c.data(), c.size() * 4);
        *n_codes = uint32_t(c.size());
        *stopped = st ? 1 : 0;
    });
}

int orc_apply_processors(const float* logits, size_t n, const uint32_t* hist, size_t hn, const orc::Opts* opts,
                         float* out) {
    return guard([&] {
        auto s = orc::apply_processors(std::vector<float>(logits, logits + n), std::vector<uint32_t>(hist, hist + hn), *opts);
        std::memcpy(out, s.data(), s.size() * 4);
    });
}

// Draws `draw`+1 uniforms from a fresh stream and samples with the last one
// (the CDF rule of gpt_sampling.cpp:130-165).
int orc_sample(const float* scores, size_t n, int rng, uint64_t seed, uint64_t draw, uint32_t* token) {
    return guard([&] {
        orc::Uniform u(rng, seed);
        for (uint64_t i = 0; i < draw; ++i) u.next();
        *token = orc::sample_token(std::vector<float>(scores, scores + n), u);
    });
}

void orc_philox4x32_10(const uint32_t* ctr, const uint32_t* key, uint32_t* out) { orc::philox4x32_10(ctr, key, out); }

uint64_t orc_splitmix64(uint64_t seed, uint64_t draw) {
    orc::SplitMix64 s(seed);
    for (uint64_t i = 0; i < draw; ++i) s.next_u64();
    return s.next_u64();
}

double orc_uniform(int rng, uint64_t seed, uint64_t draw) {
    orc::Uniform u(rng, seed);
    for (uint64_t i = 0; i < draw; ++i) u.next();
    return u.next();
}

void* orc_checkpoint(void* h) {
    std::shared_ptr<orc::State>* out = nullptr;
    if (guard([&] { out = new std::shared_ptr<orc::State>(static_cast<orc::Model*>(h)->checkpoint()); })) return nullptr;
    return out;
}
int orc_restore(void* h, void* s) {
    return guard([&] { static_cast<orc::Model*>(h)->restore(**static_cast<std::shared_ptr<orc::State>*>(s)); });
}
void orc_state_free(void* s) { delete static_cast<std::shared_ptr<orc::State>*>(s); }

}  // extern "C"
