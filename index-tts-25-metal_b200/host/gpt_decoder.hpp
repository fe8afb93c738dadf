// Header-only C++ adapter: the reference's itts25::GptDecoder interface
// (include/itts25/gpt.hpp:7-43) over the B200 C-ABI (include/itts_gpt.h).
//
// Same member names, argument meaning and exception classes as the reference:
// std::invalid_argument for bad shapes/ids/options/capacity, std::logic_error for
// call-order misuse, std::runtime_error otherwise.  Construction takes the bundle
// directory (the reference takes an already-open Weights and a MetalContext).
#pragma once

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "itts_gpt.h"

namespace itts25b200 {

struct GenerationOptions {  // gpt.hpp:7-16 (+ rng)
    bool do_sample = true;
    uint64_t seed = 20261002;
    float temperature = 0.8f;
    uint32_t top_k = 30;
    float top_p = 0.8f;
    float repetition_penalty = 10.0f;
    uint32_t num_beams = 1;
    float length_penalty = 0;
    int rng = ITTS_RNG_SPLITMIX64;
};

struct GenerationResult {  // gpt.hpp:17
    std::vector<uint32_t> codes;
    bool stopped = false;
};

struct GptState {  // gpt.hpp:18
    uint32_t tokens = 0;
    std::shared_ptr<itts_gpt_state> kv;
};

inline void throw_status(int rc, const char* msg) {
    const std::string m = msg ? msg : "";
    switch (rc) {
        case ITTS_OK: return;
        case ITTS_ERR_INVALID_ARGUMENT: throw std::invalid_argument(m);
        case ITTS_ERR_LOGIC: throw std::logic_error(m);
        default: throw std::runtime_error(m);
    }
}

inline itts_gen_opts to_c(const GenerationOptions& o) {
    itts_gen_opts c;
    c.do_sample = o.do_sample ? 1 : 0;
    c.top_k = o.top_k;
    c.seed = o.seed;
    c.temperature = o.temperature;
    c.top_p = o.top_p;
    c.repetition_penalty = o.repetition_penalty;
    c.num_beams = o.num_beams;
    c.length_penalty = o.length_penalty;
    c.rng = o.rng;
    return c;
}

class GptDecoder {
public:
    explicit GptDecoder(const std::string& bundle_dir, int device = 0, int weight_dtype = ITTS_WEIGHTS_F32) {
        const int rc = itts_gpt_create(bundle_dir.c_str(), device, weight_dtype, &ctx_);
        throw_status(rc, itts_gpt_last_error(nullptr));
    }
    ~GptDecoder() { itts_gpt_destroy(ctx_); }
    GptDecoder(const GptDecoder&) = delete;
    GptDecoder& operator=(const GptDecoder&) = delete;

    std::vector<float> prepare(const std::vector<float>& speaker, const std::vector<float>& emotion,
                               const std::vector<uint32_t>& text, uint32_t language) {
        std::vector<float> out((text.size() + 8) * ITTS_GPT_WIDTH);
        size_t rows = 0;
        check(itts_gpt_prepare(ctx_, speaker.data(), speaker.size(), emotion.data(), emotion.size(), text.data(),
                               text.size(), language, out.data(), out.size(), &rows));
        out.resize(rows * ITTS_GPT_WIDTH);
        return out;
    }
    std::vector<float> prefill(const std::vector<float>& prefix) {
        std::vector<float> logits(ITTS_GPT_VOCAB);
        check(itts_gpt_prefill(ctx_, prefix.data(), prefix.size(), logits.data()));
        return logits;
    }
    std::vector<float> step(uint32_t code, uint32_t position) {
        std::vector<float> logits(ITTS_GPT_VOCAB);
        check(itts_gpt_step(ctx_, code, position, logits.data()));
        return logits;
    }
    GenerationResult generate(const std::vector<float>& prefix, const GenerationOptions& options,
                              uint32_t max_tokens = 1500) {
        GenerationResult r;
        r.codes.resize(max_tokens ? max_tokens : 1);
        const itts_gen_opts o = to_c(options);
        uint32_t n = 0;
        int stopped = 0;
        check(itts_gpt_generate(ctx_, prefix.data(), prefix.size(), &o, max_tokens, r.codes.data(), &n, &stopped));
        r.codes.resize(n);
        r.stopped = stopped != 0;
        return r;
    }
    // Independent requests in one call (itts_gpt_generate_batch).
    std::vector<GenerationResult> generate_batch(const std::vector<std::vector<float>>& prefixes,
                                                 const std::vector<GenerationOptions>& options,
                                                 uint32_t max_tokens = 1500) {
        if (prefixes.size() != options.size()) throw std::invalid_argument("one options entry per prefix");
        const size_t b = prefixes.size();
        std::vector<const float*> ptrs(b);
        std::vector<size_t> sizes(b);
        std::vector<itts_gen_opts> o(b);
        for (size_t i = 0; i < b; ++i) {
            ptrs[i] = prefixes[i].data();
            sizes[i] = prefixes[i].size();
            o[i] = to_c(options[i]);
        }
        const size_t stride = max_tokens ? max_tokens : 1;
        std::vector<uint32_t> codes(b * stride), n(b);
        std::vector<int> stopped(b);
        check(itts_gpt_generate_batch(ctx_, b, ptrs.data(), sizes.data(), o.data(), max_tokens, codes.data(), n.data(),
                                      stopped.data()));
        std::vector<GenerationResult> out(b);
        for (size_t i = 0; i < b; ++i) {
            out[i].codes.assign(codes.begin() + i * stride, codes.begin() + i * stride + n[i]);
            out[i].stopped = stopped[i] != 0;
        }
        return out;
    }
    GptState checkpoint() const {
        itts_gpt_state* s = nullptr;
        check(itts_gpt_checkpoint(ctx_, &s));
        return GptState{itts_gpt_cached_tokens(ctx_), std::shared_ptr<itts_gpt_state>(s, itts_gpt_state_free)};
    }
    void restore(const GptState& state) { check(itts_gpt_restore(ctx_, state.kv.get())); }
    uint32_t cached_tokens() const { return itts_gpt_cached_tokens(ctx_); }
    uint64_t launch_count() const { return itts_gpt_launch_count(ctx_); }
    itts_gpt_ctx* handle() const { return ctx_; }

private:
    itts_gpt_ctx* ctx_ = nullptr;
    void check(int rc) const { throw_status(rc, itts_gpt_last_error(ctx_)); }
};

// apply_gpt_sampling_processors (gpt.hpp:19) on the decoder's device.
inline std::vector<float> apply_gpt_sampling_processors(GptDecoder& dec, const std::vector<float>& logits,
                                                        const std::vector<uint32_t>& history,
                                                        const GenerationOptions& options) {
    std::vector<float> out(logits.size());
    const itts_gen_opts o = to_c(options);
    throw_status(itts_gpt_apply_processors(dec.handle(), logits.data(), logits.size(), history.data(), history.size(),
                                           &o, out.data()),
                 itts_gpt_last_error(dec.handle()));
    return out;
}

}  // namespace itts25b200
