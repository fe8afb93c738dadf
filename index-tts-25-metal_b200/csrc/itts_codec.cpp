// Host runtime of the B200 semantic-codec decoder: implements
// include/itts_codec.h.  Mirrors the reference's EnhancedCodec
// (src/codec.cpp): the same shape checks at construction (:6-22), the same
// code-id checks at decode (:51-52); the tensor math runs on the device
// (codec.cu).
#include "itts_codec.h"

#include <cuda_runtime.h>

#include <memory>
#include <new>
#include <string>
#include <vector>

#include "codec.hpp"
#include "mit2_bundle.hpp"

namespace {

thread_local std::string g_codec_create_error;

struct CodecFailure {
    int code;
    std::string msg;
};

[[noreturn]] void cfail(int code, const std::string& msg) { throw CodecFailure{code, msg}; }

void cck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        cfail(e == cudaErrorMemoryAllocation ? ITTS_ERR_OUT_OF_MEMORY : ITTS_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
    }
}

}  // namespace

struct itts_codec_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    char* d_weights = nullptr;
    itts::CodecWeights w{};
    itts::CodecScratch sc{};
    float* d_scratch = nullptr;
    size_t scratch_tokens = 0;
    uint32_t* d_codes = nullptr;
    float* d_out = nullptr;
    size_t out_tokens = 0;
    cudaEvent_t ev[2] = {nullptr, nullptr};  // around the kernels of a decode
    itts_codec_timing timing{};
    itts::CodecTc tc;  // tensor-core GEMM state
    int gemm_mode = 0; // 0: tensor-core GEMMs, 1: CUDA-core GEMMs

    ~itts_codec_ctx() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : {(void*)d_weights, (void*)d_scratch, (void*)d_codes, (void*)d_out})
            if (p) cudaFree(p);
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        itts::codec_tc_free(&tc);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

template <class F>
int cguard(itts_codec_ctx* ctx, F&& f) {
    try {
        f();
        return ITTS_OK;
    } catch (const CodecFailure& e) {
        if (ctx) ctx->err = e.msg;
        return e.code;
    } catch (const std::bad_alloc&) {
        if (ctx) ctx->err = "host allocation failed";
        return ITTS_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        if (ctx) ctx->err = e.what();
        return ITTS_ERR_RUNTIME;
    }
}

// codec.cpp:6-22
void validate(const itts::Mit2Bundle& b) {
    if (b.target() != "index-tts2.5") cfail(ITTS_ERR_RUNTIME, "Expected an IndexTTS 2.5 model bundle");
    b.check_sizes();
    auto shape = [&](const std::string& name, std::vector<int64_t> want) {
        const auto* t = b.find(name);
        if (!t || t->shape != want) cfail(ITTS_ERR_RUNTIME, "Unsupported 2.5 codec shape: " + name);
    };
    shape("codec.down.weight", {1024, 1024, 3});
    shape("codec.up.weight", {1024, 1024, 3});
    shape("codec.quantizer.quantizers.0.codebook.weight", {8192, 8});
    for (const char* block : {"encoder", "decoder"}) {
        const std::string p = std::string("codec.") + block + ".0";
        shape(p + ".embed.weight", {384, 1024, 7});
        for (int i = 0; i < 12; ++i) {
            const std::string l = p + ".convnext." + std::to_string(i);
            shape(l + ".dwconv.weight", {384, 1, 7});
            shape(l + ".pwconv1.weight", {2048, 384});
            shape(l + ".pwconv2.weight", {384, 2048});
        }
    }
}

// The decoder's tensors (and only those), uploaded into one allocation.
void upload(itts_codec_ctx* c, const itts::Mit2Bundle& b) {
    std::vector<std::pair<std::string, std::vector<int64_t>>> names;
    auto want = [&](const std::string& n, std::vector<int64_t> shape) { names.emplace_back(n, std::move(shape)); };
    const std::string q = "codec.quantizer.quantizers.0", d = "codec.decoder.0";
    want(q + ".codebook.weight", {8192, 8});
    want(q + ".out_project.weight", {1024, 8});
    want(q + ".out_project.bias", {1024});
    want(d + ".embed.weight", {384, 1024, 7});
    want(d + ".embed.bias", {384});
    want(d + ".norm.weight", {384});
    want(d + ".norm.bias", {384});
    for (int i = 0; i < 12; ++i) {
        const std::string l = d + ".convnext." + std::to_string(i);
        want(l + ".dwconv.weight", {384, 1, 7});
        want(l + ".dwconv.bias", {384});
        want(l + ".norm.weight", {384});
        want(l + ".norm.bias", {384});
        want(l + ".pwconv1.weight", {2048, 384});
        want(l + ".pwconv1.bias", {2048});
        want(l + ".pwconv2.weight", {384, 2048});
        want(l + ".pwconv2.bias", {384});
        want(l + ".gamma", {384});
    }
    want(d + ".final_layer_norm.weight", {384});
    want(d + ".final_layer_norm.bias", {384});
    want("codec.decoder.1.weight", {1024, 384});
    want("codec.decoder.1.bias", {1024});
    want("codec.up.weight", {1024, 1024, 3});
    want("codec.up.bias", {1024});
    size_t total = 0;
    std::vector<size_t> off;
    for (const auto& n : names) {
        const auto* t = b.find(n.first);
        if (!t || t->shape != n.second) cfail(ITTS_ERR_RUNTIME, "Unsupported 2.5 codec shape: " + n.first);
        off.push_back(total);
        total += (t->nbytes + 255) & ~size_t(255);
    }
    void* p = nullptr;
    cck(cudaMalloc(&p, total), "codec weight allocation");
    c->d_weights = static_cast<char*>(p);
    for (size_t i = 0; i < names.size(); ++i) {
        const auto& t = b.info(names[i].first);
        cck(cudaMemcpy(c->d_weights + off[i], b.data(t), t.nbytes, cudaMemcpyHostToDevice), "codec weight upload");
    }
    size_t k = 0;
    auto next = [&]() { return reinterpret_cast<const float*>(c->d_weights + off[k++]); };
    itts::CodecWeights& w = c->w;
    w.codebook = next();
    w.out_w = next();
    w.out_b = next();
    w.embed_w = next();
    w.embed_b = next();
    w.norm_g = next();
    w.norm_b = next();
    for (auto& bw : w.block) {
        bw.dw_w = next();
        bw.dw_b = next();
        bw.ln_g = next();
        bw.ln_b = next();
        bw.pw1_w = next();
        bw.pw1_b = next();
        bw.pw2_w = next();
        bw.pw2_b = next();
        bw.gamma = next();
    }
    w.final_g = next();
    w.final_b = next();
    w.head_w = next();
    w.head_b = next();
    w.up_w = next();
    w.up_b = next();
}

void ensure_scratch(itts_codec_ctx* c, size_t T) {
    if (c->scratch_tokens >= T) return;
    if (c->d_scratch) cudaFree(c->d_scratch);
    if (c->d_codes) cudaFree(c->d_codes);
    if (c->d_out) cudaFree(c->d_out);
    c->d_scratch = nullptr;
    c->d_codes = nullptr;
    c->d_out = nullptr;
    c->scratch_tokens = 0;
    void* p = nullptr;
    cck(cudaMalloc(&p, T * (1024 + 384 + 384 + 2048) * sizeof(float)), "codec scratch allocation");
    c->d_scratch = static_cast<float*>(p);
    c->sc.hidden = c->d_scratch;
    c->sc.h = c->sc.hidden + T * 1024;
    c->sc.x = c->sc.h + T * 384;
    c->sc.u = c->sc.x + T * 384;
    cck(cudaMalloc(&p, T * sizeof(uint32_t)), "codec code buffer");
    c->d_codes = static_cast<uint32_t*>(p);
    cck(cudaMalloc(&p, 2 * T * 1024 * sizeof(float)), "codec output buffer");
    c->d_out = static_cast<float*>(p);
    c->scratch_tokens = T;
}

}  // namespace

extern "C" {

const char* itts_codec_last_error(const itts_codec_ctx* ctx) {
    return ctx ? ctx->err.c_str() : g_codec_create_error.c_str();
}

int itts_codec_create(const char* bundle_dir, int device, itts_codec_ctx** out) {
    g_codec_create_error.clear();
    if (!out) {
        g_codec_create_error = "out is null";
        return ITTS_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    std::unique_ptr<itts_codec_ctx> c(new (std::nothrow) itts_codec_ctx());
    if (!c) return ITTS_ERR_OUT_OF_MEMORY;
    c->device = device;
    const int rc = cguard(c.get(), [&] {
        if (!bundle_dir) cfail(ITTS_ERR_INVALID_ARGUMENT, "bundle_dir is null");
        itts::Mit2Bundle bundle(bundle_dir);
        validate(bundle);
        int n = 0;
        cck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) cfail(ITTS_ERR_INVALID_ARGUMENT, "device index out of range");
        cck(cudaSetDevice(device), "cudaSetDevice");
        cck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream creation");
        upload(c.get(), bundle);
        cck(itts::codec_tc_init(&c->tc, c->w, c->stream), "tensor-core GEMM setup");
    });
    if (rc != ITTS_OK) {
        g_codec_create_error = c->err;
        return rc;
    }
    *out = c.release();
    return ITTS_OK;
}

void itts_codec_destroy(itts_codec_ctx* ctx) { delete ctx; }

int itts_codec_decode(itts_codec_ctx* ctx, const uint32_t* codes, size_t n, float* out, size_t out_floats) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return cguard(ctx, [&] {
        cck(cudaSetDevice(ctx->device), "cudaSetDevice");
        // codec.cpp:51-52
        bool bad = !codes || n == 0 || n > ITTS_CODEC_MAX_CODES;
        for (size_t i = 0; !bad && i < n; ++i) bad = codes[i] >= 8192;
        if (bad) cfail(ITTS_ERR_INVALID_ARGUMENT, "Codec expects 1..5000 code IDs in [0,8192)");
        if (!out || out_floats < 2 * n * 1024) cfail(ITTS_ERR_INVALID_ARGUMENT, "output buffer too small");
        ensure_scratch(ctx, n);
        if (!ctx->ev[0]) {
            cck(cudaEventCreate(&ctx->ev[0]), "event creation");
            cck(cudaEventCreate(&ctx->ev[1]), "event creation");
        }
        cck(cudaMemcpyAsync(ctx->d_codes, codes, n * 4, cudaMemcpyHostToDevice, ctx->stream), "code upload");
        cck(cudaEventRecord(ctx->ev[0], ctx->stream), "event record");
        const bool tc = ctx->gemm_mode == 0;
        cck(itts::codec_decode_device(ctx->w, ctx->sc, tc ? &ctx->tc : nullptr, ctx->d_codes, int(n), ctx->d_out,
                                      ctx->stream),
            "codec decode launch");
        cck(cudaEventRecord(ctx->ev[1], ctx->stream), "event record");
        cck(cudaMemcpyAsync(out, ctx->d_out, 2 * n * 1024 * 4, cudaMemcpyDeviceToHost, ctx->stream), "features read");
        int status = 0;
        if (tc) cck(cudaMemcpyAsync(&status, ctx->tc.status, sizeof status, cudaMemcpyDeviceToHost, ctx->stream),
                    "status read");
        cck(cudaStreamSynchronize(ctx->stream), "codec decode");
        if (status) {  // a GEMM wait gave up: the features are not valid
            cck(cudaMemsetAsync(ctx->tc.status, 0, sizeof status, ctx->stream), "status clear");
            cck(cudaStreamSynchronize(ctx->stream), "status clear");
            cfail(ITTS_ERR_DEVICE_TIMEOUT, "codec GEMM device wait timed out (status " + std::to_string(status) + ")");
        }
        float ms = 0.f;
        cck(cudaEventElapsedTime(&ms, ctx->ev[0], ctx->ev[1]), "event time");
        ctx->timing =
            itts_codec_timing{ms, uint32_t(n), uint32_t(tc ? itts::kCodecLaunchesTc : itts::kCodecLaunches)};
    });
}

int itts_codec_set_gemm_mode(itts_codec_ctx* ctx, int mode) {
    if (!ctx || mode < 0 || mode > 1) return ITTS_ERR_INVALID_ARGUMENT;
    ctx->gemm_mode = mode;
    return ITTS_OK;
}

int itts_codec_last_timing(const itts_codec_ctx* ctx, itts_codec_timing* out) {
    if (!ctx || !out) return ITTS_ERR_INVALID_ARGUMENT;
    *out = ctx->timing;
    return ITTS_OK;
}

}  // extern "C"
