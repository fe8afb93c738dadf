// ORACLE / TEST INFRASTRUCTURE — never linked into the product library.
//
// CPU definitions of the mit2::MetalContext members that the reference's
// semantic codec (src/codec.cpp) calls beyond those of the GPT (ref_shim.cpp),
// so the reference's own, unmodified codec.cpp compiles and runs on Linux, and
// a C boundary (ref_codec_*) exposing EnhancedCodec::decode to Python.
// Kernel math follows vendor/metal-runtime/metal/kernels.metal:
//   conv1d same padding     mit2_conv1d_same_f32          (:1397-1425)
//   depthwise conv1d same   mit2_depthwise_conv1d_same_f32 (:1516-1540)
//   nearest interpolation   mit2_nearest_interpolate_f32  (:1376-1395)
//   exact-form GELU         itts25_codec_gelu             (:3132-3137)
//   channel scale           itts25_codec_scale            (:3138-3140)
// and the pass plumbing of metal_context.mm (:5030-5060, :5862-5870,
// :6205-6236).  Sums are carried in double and rounded once per output, as in
// cpu_math.hpp.  CodecOps (src/codec_ops.mm, Metal) serves only the codec's
// encode path; its members here refuse to run.
#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "cpu_math.hpp"
#include "itts25/codec.hpp"
#include "itts25/weights.hpp"
#include "mit2/metal_context.hpp"
#include "shim_impl.hpp"

namespace {

// out[t][o] = b[o] + sum_{c, k} x[t + k - kernel/2][c] * w[o][c][k] (zero padding).
void conv1d_same(const float* x, const float* w, const float* b, uint32_t tokens, uint32_t in_ch, uint32_t out_ch,
                 uint32_t kernel, float* out) {
    const int pad = int(kernel / 2);
    orc::pool().run(out_ch, [&](size_t o0, size_t o1) {
        for (size_t o = o0; o < o1; ++o)
            for (uint32_t t = 0; t < tokens; ++t) {
                double acc = b[o];
                for (uint32_t c = 0; c < in_ch; ++c)
                    for (uint32_t k = 0; k < kernel; ++k) {
                        const int s = int(t) + int(k) - pad;
                        if (s >= 0 && s < int(tokens))
                            acc += double(x[size_t(s) * in_ch + c]) * double(w[(o * in_ch + c) * kernel + k]);
                    }
                out[size_t(t) * out_ch + o] = float(acc);
            }
    });
}

void depthwise_same(const float* x, const float* w, const float* b, uint32_t tokens, uint32_t ch, uint32_t kernel,
                    float* out) {
    const int pad = int(kernel / 2);
    for (uint32_t t = 0; t < tokens; ++t)
        for (uint32_t c = 0; c < ch; ++c) {
            double acc = b[c];
            for (uint32_t k = 0; k < kernel; ++k) {
                const int s = int(t) + int(k) - pad;
                if (s >= 0 && s < int(tokens)) acc += double(x[size_t(s) * ch + c]) * double(w[size_t(c) * kernel + k]);
            }
            out[size_t(t) * ch + c] = float(acc);
        }
}

// GELU 0.5 x (1 + erf(x / sqrt 2)) with erf from the Abramowitz-Stegun 7.1.26
// rational approximation, in the float operations of itts25_codec_gelu.
float codec_gelu(float x) {
    const float v = x * 0.7071067811865475f, a = std::fabs(v), t = 1.0f / (1.0f + 0.3275911f * a);
    const float p = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    float erf = 1.0f - p * std::exp(-a * a);
    if (v < 0) erf = -erf;
    return 0.5f * x * (1.0f + erf);
}

}  // namespace

namespace mit2 {

PassSlot MetalContext::conv1d_same_f32_pass(const std::string&, const std::vector<float>& w, const std::string&,
                                            const std::vector<float>& b, PassSlot x, uint32_t tokens, uint32_t in_ch,
                                            uint32_t out_ch, uint32_t kernel) {
    if (w.size() != size_t(out_ch) * in_ch * kernel || b.size() != out_ch || x.element_count != tokens * in_ch)
        throw std::invalid_argument("conv1d_same_f32_pass sizes");
    auto out = (impl_->require_pass("conv1d_same_f32_pass"), impl_->alloc(tokens * out_ch));
    conv1d_same(impl_->f(x), w.data(), b.data(), tokens, in_ch, out_ch, kernel, impl_->f(out));
    return out;
}
PassSlot MetalContext::depthwise_conv1d_same_pass(const std::string&, const std::vector<float>& w, const std::string&,
                                                  const std::vector<float>& b, PassSlot x, uint32_t tokens,
                                                  uint32_t channels, uint32_t kernel) {
    if (w.size() != size_t(channels) * kernel || b.size() != channels || x.element_count != tokens * channels)
        throw std::invalid_argument("depthwise_conv1d_same_pass sizes");
    auto out = (impl_->require_pass("depthwise_conv1d_same_pass"), impl_->alloc(tokens * channels));
    depthwise_same(impl_->f(x), w.data(), b.data(), tokens, channels, kernel, impl_->f(out));
    return out;
}
PassSlot MetalContext::codec_gelu_pass(PassSlot x) {
    auto out = (impl_->require_pass("codec_gelu_pass"), impl_->alloc(x.element_count));
    const float* i = impl_->f(x);
    float* o = impl_->f(out);
    for (uint32_t k = 0; k < x.element_count; ++k) o[k] = codec_gelu(i[k]);
    return out;
}
PassSlot MetalContext::codec_scale_pass(PassSlot x, const std::string&, const std::vector<float>& gamma) {
    if (gamma.empty() || x.element_count % gamma.size()) throw std::invalid_argument("Codec scale dimensions");
    auto out = (impl_->require_pass("codec_scale_pass"), impl_->alloc(x.element_count));
    const float* i = impl_->f(x);
    float* o = impl_->f(out);
    for (uint32_t k = 0; k < x.element_count; ++k) o[k] = i[k] * gamma[k % gamma.size()];
    return out;
}
PassSlot MetalContext::nearest_interpolate_pass(PassSlot x, uint32_t in_tokens, uint32_t out_tokens, uint32_t width) {
    if (!in_tokens || !out_tokens || x.element_count != in_tokens * width)
        throw std::invalid_argument("Interpolation dimensions");
    auto out = (impl_->require_pass("nearest_interpolate_pass"), impl_->alloc(out_tokens * width));
    const float scale = float(in_tokens) / out_tokens;
    const float* i = impl_->f(x);
    float* o = impl_->f(out);
    for (uint32_t t = 0; t < out_tokens; ++t) {
        uint32_t s = uint32_t(std::floor(float(t) * scale));
        if (s >= in_tokens) s = in_tokens - 1;
        std::memcpy(o + size_t(t) * width, i + size_t(s) * width, size_t(width) * 4);
    }
    return out;
}
void MetalContext::copy_f32_pass_into(PassSlot src, PassSlot dst, uint32_t count) {
    impl_->require_pass("copy_f32_pass_into");
    std::memcpy(impl_->f(dst), impl_->f(src), size_t(count) * 4);
}

// Members the codec's encode-only helpers reference (codec.cpp norm/conv).
std::vector<float> MetalContext::layernorm_rows_f32_resident(const std::string&, const std::vector<float>& g,
                                                             const std::string&, const std::vector<float>& be,
                                                             const std::vector<float>& x, uint32_t tokens,
                                                             uint32_t width, float eps) {
    if (g.size() != width || be.size() != width || x.size() != size_t(tokens) * width)
        throw std::invalid_argument("layernorm_rows_f32_resident invalid input sizes");
    std::vector<float> out(x.size());
    orc::layernorm_rows(x.data(), g.data(), be.data(), tokens, width, eps, out.data());
    return out;
}
std::vector<float> MetalContext::conv1d_same_f32_resident(const std::string&, const std::vector<float>& w,
                                                          const std::string&, const std::vector<float>& b,
                                                          const std::vector<float>& x, uint32_t tokens,
                                                          uint32_t in_ch, uint32_t out_ch, uint32_t kernel) {
    std::vector<float> out(size_t(tokens) * out_ch);
    conv1d_same(x.data(), w.data(), b.data(), tokens, in_ch, out_ch, kernel, out.data());
    return out;
}
std::vector<float> MetalContext::depthwise_conv1d_same_f32_resident(const std::string&, const std::vector<float>& w,
                                                                    const std::string&, const std::vector<float>& b,
                                                                    const std::vector<float>& x, uint32_t tokens,
                                                                    uint32_t channels, uint32_t kernel) {
    std::vector<float> out(size_t(tokens) * channels);
    depthwise_same(x.data(), w.data(), b.data(), tokens, channels, kernel, out.data());
    return out;
}

}  // namespace mit2

namespace itts25 {
struct CodecOps::Impl {};
CodecOps::CodecOps() : impl_(new Impl()) {}
CodecOps::~CodecOps() = default;
uint64_t CodecOps::submissions() const { return 0; }
std::vector<float> CodecOps::gelu(const std::vector<float>&) { throw std::logic_error("codec encode is not in the shim"); }
std::vector<float> CodecOps::scale(const std::vector<float>&, const std::vector<float>&) {
    throw std::logic_error("codec encode is not in the shim");
}
std::vector<float> CodecOps::downsample(const std::vector<float>&, const std::vector<float>&, const std::vector<float>&,
                                        uint32_t) {
    throw std::logic_error("codec encode is not in the shim");
}
std::vector<uint32_t> CodecOps::quantize(const std::vector<float>&, const std::vector<float>&) {
    throw std::logic_error("codec encode is not in the shim");
}
}  // namespace itts25

namespace {
thread_local std::string g_codec_error;
struct CodecHandle {
    itts25::Weights w;
    mit2::MetalContext m;
    itts25::EnhancedCodec c;
    explicit CodecHandle(const char* dir) : w(dir), c(w, m) {}
};
}  // namespace

extern "C" {
const char* ref_codec_last_error() { return g_codec_error.c_str(); }
void* ref_codec_load(const char* dir) {
    try {
        return new CodecHandle(dir);
    } catch (const std::exception& e) {
        g_codec_error = e.what();
        return nullptr;
    }
}
void ref_codec_free(void* h) { delete static_cast<CodecHandle*>(h); }
// EnhancedCodec::decode (codec.cpp:59-69): n codes -> [2n, 1024] floats.
int ref_codec_decode(void* h, const uint32_t* codes, size_t n, float* out, size_t out_floats) {
    try {
        auto v = static_cast<CodecHandle*>(h)->c.decode(std::vector<uint32_t>(codes, codes + n));
        if (v.size() > out_floats) throw std::invalid_argument("output buffer too small");
        std::memcpy(out, v.data(), v.size() * 4);
        return 0;
    } catch (const std::invalid_argument& e) {
        g_codec_error = e.what();
        return -1;
    } catch (const std::exception& e) {
        g_codec_error = e.what();
        return -2;
    }
}
}
