// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
//
// CPU implementation of the 24 mit2::MetalContext members that the reference's
// GPT sources call, so that the reference's own, unmodified src/gpt.cpp,
// src/gpt_sampling.cpp, src/weights.cpp and vendor/metal-runtime/bundle.cpp
// compile and run on Linux (Makefile target `_ref/libitts_ref.so`).  The class
// declaration is the reference's header (vendor/metal-runtime/include/mit2/
// metal_context.hpp); only the members below are defined.  Semantics follow
// vendor/metal-runtime/metal_context.mm (pass workspace :4594-4703, KV cache
// :237-249 and :5675-5842, attention :5326-5353 and :6153-6174); kernel math
// comes from cpu_math.hpp.  A C boundary (ref_*) exposes GptDecoder to Python.
#include "mit2/metal_context.hpp"

#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#include "cpu_math.hpp"
#include "itts25/gpt.hpp"
#include "shim_impl.hpp"

namespace mit2 {

namespace {
struct CpuSnapshot final : GpuKvSnapshot {
    std::vector<float> values;
    uint32_t tokens, layers, width;
    CpuSnapshot(std::vector<float> v, uint32_t t, uint32_t l, uint32_t w)
        : values(std::move(v)), tokens(t), layers(l), width(w) {}
};
}  // namespace

MetalContext::MetalContext() : impl_(new Impl()) {}
MetalContext::~MetalContext() { delete impl_; }

std::vector<float> MetalContext::add_f32(const std::vector<float>& a, const std::vector<float>& b) {
    if (a.size() != b.size()) throw std::invalid_argument("add_f32 input size mismatch");
    std::vector<float> out(a.size());
    for (size_t i = 0; i < a.size(); ++i) out[i] = a[i] + b[i];
    ++impl_->submissions;
    return out;
}

std::vector<float> MetalContext::embedding_f32_resident(const std::string&, const std::vector<float>& table,
                                                        const std::vector<uint32_t>& ids, uint32_t width) {
    if (width == 0 || table.size() % width != 0) throw std::invalid_argument("embedding_f32_resident invalid table width");
    std::vector<float> out(ids.size() * size_t(width));
    for (size_t t = 0; t < ids.size(); ++t)
        std::memcpy(out.data() + t * width, table.data() + size_t(ids[t]) * width, size_t(width) * 4);
    ++impl_->submissions;
    return out;
}

std::vector<float> MetalContext::linear_rows_f32_resident(const std::string&, const std::vector<float>& weight,
                                                          const std::string&, const std::vector<float>& bias,
                                                          const std::vector<float>& x, uint32_t tokens, uint32_t rows,
                                                          uint32_t cols) {
    if (!tokens || !rows || !cols || weight.size() != size_t(rows) * cols || bias.size() != rows ||
        x.size() != size_t(tokens) * cols)
        throw std::invalid_argument("linear_rows_f32_resident invalid input sizes");
    std::vector<float> out(size_t(tokens) * rows);
    orc::linear_rows(weight.data(), bias.data(), x.data(), tokens, rows, cols, out.data());
    ++impl_->submissions;
    return out;
}

void MetalContext::beginPass(size_t bytes) {
    if (impl_->pass) throw std::logic_error("beginPass: already in pass mode");
    if (impl_->ws.size() < bytes) impl_->ws.resize(bytes);
    impl_->cursor = impl_->scratch = 0;
    impl_->pass = true;
}
void MetalContext::endPass() {
    if (!impl_->pass) throw std::logic_error("endPass: not in pass mode");
    impl_->pass = false;
    ++impl_->submissions;
}
void MetalContext::passSetScratchBase() {
    impl_->require_pass("passSetScratchBase");
    impl_->scratch = impl_->cursor;
}
void MetalContext::passResetScratch() {
    impl_->require_pass("passResetScratch");
    impl_->cursor = impl_->scratch;
}
PassSlot MetalContext::passAlloc(uint32_t n) {
    impl_->require_pass("passAlloc");
    return impl_->alloc(n);
}
PassSlot MetalContext::passUploadAlloc(const std::vector<float>& data) {
    impl_->require_pass("passUploadAlloc");
    auto s = impl_->alloc(static_cast<uint32_t>(data.size()));
    std::memcpy(impl_->f(s), data.data(), data.size() * 4);
    return s;
}
PassSlot MetalContext::passUploadAllocU32(const std::vector<uint32_t>& data) {
    impl_->require_pass("passUploadAllocU32");
    auto s = impl_->alloc(static_cast<uint32_t>(data.size()));
    std::memcpy(impl_->f(s), data.data(), data.size() * 4);
    return s;
}
std::vector<float> MetalContext::passRead(PassSlot s) const {
    if (impl_->pass) throw std::logic_error("passRead: cannot read while pass is active");
    if (!s.valid() || impl_->ws.empty()) throw std::invalid_argument("passRead: invalid slot or no workspace");
    const float* p = impl_->f(s);
    return std::vector<float>(p, p + s.element_count);
}

PassSlot MetalContext::add_f32_pass(PassSlot a, PassSlot b) {
    impl_->require_pass("add_f32_pass");
    auto out = impl_->alloc(a.element_count);
    float *x = impl_->f(a), *y = impl_->f(b), *o = impl_->f(out);
    for (uint32_t i = 0; i < a.element_count; ++i) o[i] = x[i] + y[i];
    return out;
}
void MetalContext::add_f32_pass_into(PassSlot a, PassSlot b, PassSlot out) {
    impl_->require_pass("add_f32_pass_into");
    float *x = impl_->f(a), *y = impl_->f(b), *o = impl_->f(out);
    for (uint32_t i = 0; i < a.element_count; ++i) o[i] = x[i] + y[i];
}
PassSlot MetalContext::linear_rows_f32_pass(const std::string&, const std::vector<float>& w, const std::string&,
                                            const std::vector<float>& b, PassSlot x, uint32_t tokens, uint32_t rows,
                                            uint32_t cols) {
    impl_->require_pass("linear_rows_f32_pass");
    if (w.size() != size_t(rows) * cols || b.size() != rows) throw std::invalid_argument("linear_rows_f32_pass sizes");
    auto out = impl_->alloc(tokens * rows);
    orc::linear_rows(w.data(), b.data(), impl_->f(x), tokens, rows, cols, impl_->f(out));
    return out;
}
PassSlot MetalContext::layernorm_rows_f32_pass(const std::string&, const std::vector<float>& g, const std::string&,
                                               const std::vector<float>& be, PassSlot x, uint32_t tokens,
                                               uint32_t width, float eps) {
    impl_->require_pass("layernorm_rows_f32_pass");
    auto out = impl_->alloc(tokens * width);
    orc::layernorm_rows(impl_->f(x), g.data(), be.data(), tokens, width, eps, impl_->f(out));
    return out;
}
PassSlot MetalContext::gelu_f32_pass(PassSlot x, uint32_t count) {
    impl_->require_pass("gelu_f32_pass");
    auto out = impl_->alloc(count);
    float *i = impl_->f(x), *o = impl_->f(out);
    for (uint32_t k = 0; k < count; ++k) o[k] = orc::gelu(i[k]);
    return out;
}
PassSlot MetalContext::gpt_build_current_pass(PassSlot token_slot, const std::string&, const std::vector<float>& mel,
                                              const std::string&, const std::vector<float>& pos, uint32_t width,
                                              uint32_t position) {
    impl_->require_pass("gpt_build_current_pass");
    auto out = impl_->alloc(width);
    uint32_t token;
    std::memcpy(&token, impl_->f(token_slot), 4);
    float* o = impl_->f(out);
    for (uint32_t i = 0; i < width; ++i) o[i] = mel[size_t(token) * width + i] + pos[size_t(position) * width + i];
    return out;
}

// metal_context.mm:5675-5700: capacity floor 2048, grow-only layout.
void MetalContext::gptKvCacheCreate(uint32_t layers, uint32_t max_tokens, uint32_t width) {
    if (!layers || !max_tokens || !width) throw std::invalid_argument("gptKvCacheCreate invalid dims");
    uint32_t cap = std::max<uint32_t>(max_tokens, 2048);
    if (!impl_->kv.empty() && impl_->kv_layers == layers && impl_->kv_width == width && impl_->kv_cap >= cap) return;
    cap = std::max(cap, impl_->kv_cap);
    impl_->kv.assign(size_t(layers) * 2 * cap * width, 0.0f);
    impl_->kv_layers = layers;
    impl_->kv_cap = cap;
    impl_->kv_width = width;
}
void MetalContext::gptKvStoreFromQkv_pass(uint32_t layer, PassSlot qkv, uint32_t tokens) {
    impl_->require_pass("gptKvStoreFromQkv_pass");
    if (impl_->kv.empty() || layer >= impl_->kv_layers || tokens > impl_->kv_cap)
        throw std::invalid_argument("gptKvStoreFromQkv_pass invalid args");
    const uint32_t w = impl_->kv_width;
    const float* q = impl_->f(qkv);
    for (uint32_t t = 0; t < tokens; ++t) {
        std::memcpy(impl_->K(layer) + size_t(t) * w, q + size_t(t) * 3 * w + w, size_t(w) * 4);
        std::memcpy(impl_->V(layer) + size_t(t) * w, q + size_t(t) * 3 * w + 2 * w, size_t(w) * 4);
    }
}
PassSlot MetalContext::gpt_causal_attention_f32_pass(PassSlot qkv, uint32_t tokens, uint32_t heads, uint32_t head_dim) {
    impl_->require_pass("gpt_causal_attention_f32_pass");
    if (tokens == 0 || tokens > 4096 || (1024 % head_dim) != 0)
        throw std::invalid_argument("gpt_causal_attention_f32_pass invalid args");
    auto out = impl_->alloc(tokens * heads * head_dim);
    orc::causal_attention(impl_->f(qkv), tokens, heads, head_dim, impl_->f(out));
    return out;
}
PassSlot MetalContext::gpt_cached_attention_resident_pass(uint32_t layer, PassSlot qkv, uint32_t cache_tokens,
                                                          uint32_t heads, uint32_t head_dim) {
    impl_->require_pass("gpt_cached_attention_resident_pass");
    if (impl_->kv.empty() || layer >= impl_->kv_layers || cache_tokens + 1 > impl_->kv_cap || cache_tokens + 1 > 4096 ||
        heads * head_dim != impl_->kv_width)
        throw std::invalid_argument("gpt_cached_attention_resident_pass invalid args");
    const uint32_t w = impl_->kv_width;
    auto out = impl_->alloc(w);
    const float* q = impl_->f(qkv);
    orc::cached_attention(impl_->K(layer), impl_->V(layer), q, cache_tokens, heads, head_dim, impl_->f(out));
    std::memcpy(impl_->K(layer) + size_t(cache_tokens) * w, q + w, size_t(w) * 4);
    std::memcpy(impl_->V(layer) + size_t(cache_tokens) * w, q + 2 * w, size_t(w) * 4);
    return out;
}
// metal_context.mm:5702-5731 (CPU copy form): values [layer][K|V][tokens][width].
std::shared_ptr<GpuKvSnapshot> MetalContext::gptKvSnapshot(uint32_t tokens) {
    if (impl_->pass || impl_->kv.empty() || !tokens || tokens > impl_->kv_cap)
        throw std::invalid_argument("Invalid KV snapshot");
    const size_t n = size_t(tokens) * impl_->kv_width;
    std::vector<float> v(n * 2 * impl_->kv_layers);
    for (uint32_t l = 0; l < impl_->kv_layers; ++l) {
        std::memcpy(v.data() + 2 * l * n, impl_->K(l), n * 4);
        std::memcpy(v.data() + (2 * l + 1) * n, impl_->V(l), n * 4);
    }
    return std::make_shared<CpuSnapshot>(std::move(v), tokens, impl_->kv_layers, impl_->kv_width);
}
void MetalContext::gptKvRestore(const std::shared_ptr<GpuKvSnapshot>& snapshot, uint32_t tokens) {
    auto s = std::dynamic_pointer_cast<CpuSnapshot>(snapshot);
    if (impl_->pass || !s || s->tokens != tokens || s->layers != impl_->kv_layers || s->width != impl_->kv_width ||
        tokens > impl_->kv_cap)
        throw std::invalid_argument("Invalid KV restore");
    const size_t n = size_t(tokens) * impl_->kv_width;
    for (uint32_t l = 0; l < impl_->kv_layers; ++l) {
        std::memcpy(impl_->K(l), s->values.data() + 2 * l * n, n * 4);
        std::memcpy(impl_->V(l), s->values.data() + (2 * l + 1) * n, n * 4);
    }
}
void MetalContext::gptKvSnapshotsClear() {}

}  // namespace mit2

// ------------------------------------------------------------- C boundary
namespace {
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
struct Handle {
    itts25::Weights w;
    mit2::MetalContext m;
    itts25::GptDecoder g;
    explicit Handle(const std::string& dir) : w(dir), m(), g(w, m) {}
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
itts25::GenerationOptions to_options(const Opts& o, bool sampling = true) {
    if (sampling && o.rng != 0) throw std::invalid_argument("the reference samples with SplitMix64 only");
    itts25::GenerationOptions g;
    g.do_sample = o.do_sample != 0;
    g.seed = o.seed;
    g.temperature = o.temperature;
    g.top_k = o.top_k;
    g.top_p = o.top_p;
    g.repetition_penalty = o.repetition_penalty;
    g.num_beams = o.num_beams;
    g.length_penalty = o.length_penalty;
    return g;
}
}  // namespace

extern "C" {
const char* ref_last_error() { return g_error.c_str(); }
int ref_threads() { return orc::pool().size(); }
void* ref_load(const char* dir) {
    Handle* h = nullptr;
    if (guard([&] { h = new Handle(dir); })) return nullptr;
    return h;
}
void ref_free(void* h) { delete static_cast<Handle*>(h); }
uint32_t ref_cached_tokens(void* h) { return static_cast<Handle*>(h)->g.cached_tokens(); }
int ref_prepare(void* h, const float* spk, size_t spk_n, const float* emo, size_t emo_n, const uint32_t* ids, size_t n,
                uint32_t lang, float* out, size_t cap_floats, size_t* rows) {
    return guard([&] {
        auto p = static_cast<Handle*>(h)->g.prepare(std::vector<float>(spk, spk + spk_n), std::vector<float>(emo, emo + emo_n),
                                                    std::vector<uint32_t>(ids, ids + n), lang);
        if (p.size() > cap_floats) throw std::invalid_argument("output buffer too small");
        std::memcpy(out, p.data(), p.size() * 4);
        *rows = p.size() / 1280;
    });
}
int ref_prefill(void* h, const float* prefix, size_t n_floats, float* logits) {
    return guard([&] {
        auto l = static_cast<Handle*>(h)->g.prefill(std::vector<float>(prefix, prefix + n_floats));
        std::memcpy(logits, l.data(), l.size() * 4);
    });
}
int ref_step(void* h, uint32_t code, uint32_t pos, float* logits) {
    return guard([&] {
        auto l = static_cast<Handle*>(h)->g.step(code, pos);
        std::memcpy(logits, l.data(), l.size() * 4);
    });
}
int ref_generate(void* h, const float* prefix, size_t n_floats, const Opts* o, uint32_t maximum, uint32_t* codes,
                 uint32_t* n_codes, int* stopped) {
    return guard([&] {
        auto r = static_cast<Handle*>(h)->g.generate(std::vector<float>(prefix, prefix + n_floats), to_options(*o), maximum);
        std::memcpy(codes, r.codes.data(), r.codes.size() * 4);
        *n_codes = uint32_t(r.codes.size());
        *stopped = r.stopped ? 1 : 0;
    });
}
int ref_apply_processors(const float* logits, size_t n, const uint32_t* hist, size_t hn, const Opts* o, float* out) {
    return guard([&] {
        auto s = itts25::apply_gpt_sampling_processors(std::vector<float>(logits, logits + n),
                                                       std::vector<uint32_t>(hist, hist + hn), to_options(*o, false));
        std::memcpy(out, s.data(), s.size() * 4);
    });
}
void* ref_checkpoint(void* h) {
    itts25::GptState* s = nullptr;
    if (guard([&] { s = new itts25::GptState(static_cast<Handle*>(h)->g.checkpoint()); })) return nullptr;
    return s;
}
int ref_restore(void* h, void* s) {
    return guard([&] { static_cast<Handle*>(h)->g.restore(*static_cast<itts25::GptState*>(s)); });
}
void ref_state_free(void* s) { delete static_cast<itts25::GptState*>(s); }
}
