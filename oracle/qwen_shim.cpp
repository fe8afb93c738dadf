// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
//
// CPU definitions of the mit2::MetalContext members that the reference's
// Qwen3-0.6B decoder (src/qwen.cpp) calls beyond those of the GPT
// (ref_shim.cpp), so the reference's own, unmodified qwen.cpp compiles and runs
// on Linux, and a C boundary (ref_qwen_*) exposing QwenDecoder to Python.
// Kernel math follows vendor/metal-runtime/metal/kernels.metal:
//   embedding gather          mit2_embedding_f32          (:281-294)
//   RMSNorm rows with eps     mit2_rmsnorm_f32_rows_eps   (:995-1030)
//   SiLU(a) * b               mit2_silu_mul_f32           (:363-374)
//   argmax, first index       mit2_gpt_argmax_f32         (:1269-1305)
//   half-rotation RoPE        itts25_qwen_rope            (:3111-3115)
//   K/V store + GQA attention itts25_qwen_store, itts25_qwen_attention (:3116-3131)
// and the pass plumbing of metal_context.mm (:4886-4930, :6111-6125).  Sums
// are carried in double and rounded once per output, as in cpu_math.hpp.  The
// RoPE inverse frequencies 1e6^(-j/64) are the correctly rounded floats of the
// exact values (the reference evaluates pow() in float on the GPU); the angle
// is their float product with the position, as in the kernel.
#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "itts25/qwen.hpp"
#include "itts25/weights.hpp"
#include "mit2/metal_context.hpp"
#include "shim_impl.hpp"

namespace {

constexpr uint32_t kQwenHeadDim = 128;

float rope_inv_freq(uint32_t j) { return float(std::pow(1000000.0, -double(j) / 64.0)); }

}  // namespace

namespace mit2 {

PassSlot MetalContext::embedding_f32_pass(const std::string&, const std::vector<float>& table, PassSlot ids,
                                          uint32_t tokens, uint32_t width) {
    if (!tokens || !width || ids.element_count != tokens || table.size() % width)
        throw std::invalid_argument("Embedding dimensions");
    auto out = (impl_->require_pass("embedding_f32_pass"), impl_->alloc(tokens * width));
    const uint32_t* id = reinterpret_cast<const uint32_t*>(impl_->f(ids));
    for (uint32_t t = 0; t < tokens; ++t) {
        if (size_t(id[t]) * width >= table.size()) throw std::invalid_argument("embedding id out of range");
        std::memcpy(impl_->f(out) + size_t(t) * width, table.data() + size_t(id[t]) * width, size_t(width) * 4);
    }
    return out;
}

PassSlot MetalContext::rmsnorm_rows_eps_f32_pass(const std::string&, const std::vector<float>& g, PassSlot x,
                                                 uint32_t tokens, uint32_t width, float eps) {
    if (g.size() != width || x.element_count != tokens * width) throw std::invalid_argument("rmsnorm sizes");
    auto out = (impl_->require_pass("rmsnorm_rows_eps_f32_pass"), impl_->alloc(tokens * width));
    const float* in = impl_->f(x);
    float* o = impl_->f(out);
    for (uint32_t t = 0; t < tokens; ++t) {
        const float* r = in + size_t(t) * width;
        double ss = 0;
        for (uint32_t i = 0; i < width; ++i) ss += double(r[i]) * double(r[i]);
        const double inv = 1.0 / std::sqrt(ss / width + double(eps));
        for (uint32_t i = 0; i < width; ++i) o[size_t(t) * width + i] = float(double(r[i]) * inv * double(g[i]));
    }
    return out;
}

PassSlot MetalContext::silu_mul_f32_pass(PassSlot a, PassSlot b) {
    if (a.element_count != b.element_count) throw std::invalid_argument("silu_mul sizes");
    auto out = (impl_->require_pass("silu_mul_f32_pass"), impl_->alloc(a.element_count));
    const float *x = impl_->f(a), *y = impl_->f(b);
    float* o = impl_->f(out);
    for (uint32_t i = 0; i < a.element_count; ++i) {
        const double v = x[i];
        o[i] = float(v / (1.0 + std::exp(-v)) * double(y[i]));
    }
    return out;
}

PassSlot MetalContext::gpt_argmax_pass(PassSlot logits, uint32_t vocab) {
    auto out = (impl_->require_pass("gpt_argmax_pass"), impl_->alloc(1));
    const float* l = impl_->f(logits);
    uint32_t best = 0;
    for (uint32_t i = 1; i < vocab; ++i)
        if (l[i] > l[best]) best = i;
    *reinterpret_cast<uint32_t*>(impl_->f(out)) = best;
    return out;
}

std::vector<uint32_t> MetalContext::passReadU32(PassSlot s) const {
    if (impl_->pass) throw std::logic_error("passReadU32: cannot read while pass is active");
    const uint32_t* p = reinterpret_cast<const uint32_t*>(impl_->ws.data() + s.byte_offset);
    return std::vector<uint32_t>(p, p + s.element_count);
}

PassSlot MetalContext::qwen_rope_f32_pass(PassSlot x, uint32_t tokens, uint32_t heads, uint32_t offset) {
    if (x.element_count != tokens * heads * kQwenHeadDim) throw std::invalid_argument("rope sizes");
    auto out = (impl_->require_pass("qwen_rope_f32_pass"), impl_->alloc(x.element_count));
    const float* in = impl_->f(x);
    float* o = impl_->f(out);
    for (uint32_t id = 0; id < x.element_count; ++id) {
        const uint32_t d = id % kQwenHeadDim, base = id - d, t = id / (heads * kQwenHeadDim);
        const float angle = float(offset + t) * rope_inv_freq(d % 64);
        const double rotated = d < 64 ? -double(in[base + d + 64]) : double(in[base + d - 64]);
        o[id] = float(double(in[id]) * std::cos(double(angle)) + rotated * std::sin(double(angle)));
    }
    return out;
}

PassSlot MetalContext::qwen_attention_f32_pass(uint32_t layer, PassSlot q, PassSlot k, PassSlot v, uint32_t tokens,
                                               uint32_t offset) {
    impl_->require_pass("qwen_attention_f32_pass");
    if (impl_->kv.empty() || layer >= impl_->kv_layers || impl_->kv_width != 1024 || offset + tokens > impl_->kv_cap)
        throw std::invalid_argument("Invalid Qwen attention cache");
    float* K = impl_->K(layer);
    float* V = impl_->V(layer);
    std::memcpy(K + size_t(offset) * 1024, impl_->f(k), size_t(tokens) * 1024 * 4);
    std::memcpy(V + size_t(offset) * 1024, impl_->f(v), size_t(tokens) * 1024 * 4);
    auto out = impl_->alloc(tokens * 2048);
    const float* Q = impl_->f(q);
    float* o = impl_->f(out);
    std::vector<double> p;
    for (uint32_t t = 0; t < tokens; ++t)
        for (uint32_t h = 0; h < 16; ++h) {
            const float* qv = Q + size_t(t) * 2048 + h * kQwenHeadDim;
            const uint32_t count = offset + t + 1, kv = h / 2;
            p.assign(count, 0.0);
            double peak = -INFINITY;
            for (uint32_t key = 0; key < count; ++key) {
                double dot = 0;
                for (uint32_t d = 0; d < kQwenHeadDim; ++d)
                    dot += double(qv[d]) * double(K[size_t(key) * 1024 + kv * kQwenHeadDim + d]);
                p[key] = dot * 0.08838834764831844;
                peak = std::max(peak, p[key]);
            }
            double sum = 0;
            for (uint32_t key = 0; key < count; ++key) sum += (p[key] = std::exp(p[key] - peak));
            for (uint32_t d = 0; d < kQwenHeadDim; ++d) {
                double acc = 0;
                for (uint32_t key = 0; key < count; ++key)
                    acc += p[key] / sum * double(V[size_t(key) * 1024 + kv * kQwenHeadDim + d]);
                o[size_t(t) * 2048 + h * kQwenHeadDim + d] = float(acc);
            }
        }
    return out;
}

}  // namespace mit2

namespace {
thread_local std::string g_qwen_error;
struct QwenHandle {
    itts25::Weights w;
    itts25::QwenDecoder d;
    explicit QwenHandle(const char* dir) : w(dir), d(w) {}
};
template <class F>
int qguard(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_qwen_error = e.what();
        return -1;
    } catch (const std::exception& e) {
        g_qwen_error = e.what();
        return -2;
    }
}
}  // namespace

extern "C" {
const char* ref_qwen_last_error() { return g_qwen_error.c_str(); }
void* ref_qwen_load(const char* dir) {
    try {
        return new QwenHandle(dir);
    } catch (const std::exception& e) {
        g_qwen_error = e.what();
        return nullptr;
    }
}
void ref_qwen_free(void* h) { delete static_cast<QwenHandle*>(h); }
// QwenDecoder::prefill (qwen.cpp:19-22): logits [151936] of the last prompt token.
int ref_qwen_prefill(void* h, const uint32_t* ids, size_t n, float* logits) {
    return qguard([&] {
        auto v = static_cast<QwenHandle*>(h)->d.prefill(std::vector<uint32_t>(ids, ids + n));
        std::memcpy(logits, v.data(), v.size() * 4);
    });
}
// QwenDecoder::step (qwen.cpp:23).
int ref_qwen_step(void* h, uint32_t id, float* logits) {
    return qguard([&] {
        auto v = static_cast<QwenHandle*>(h)->d.step(id);
        std::memcpy(logits, v.data(), v.size() * 4);
    });
}
// QwenDecoder::generate (qwen.cpp:44-50): greedy ids up to and including EOS.
int ref_qwen_generate(void* h, const uint32_t* ids, size_t n, uint32_t maximum, uint32_t* out, uint32_t* out_n) {
    return qguard([&] {
        auto v = static_cast<QwenHandle*>(h)->d.generate(std::vector<uint32_t>(ids, ids + n), maximum);
        std::memcpy(out, v.data(), v.size() * 4);
        *out_n = uint32_t(v.size());
    });
}
}
