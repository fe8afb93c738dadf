// Host runtime of the B200 Qwen3-0.6B decoder: implements include/itts_qwen.h.
// Mirrors the reference's QwenDecoder (src/qwen.cpp): the same shape checks
// at construction (:5-14), the same argument checks and messages (:19-23,
// :44-50), greedy selection by first index of the maximum.  The prompt pass
// runs per layer as RMSNorm / tensor-core GEMM / attention launches
// (qwen.cu, gemm_tma.cu); a decode step is one CUDA graph (captured once per
// context) replayed per token, its kernels reading the token and position from
// the device State that the step's argmax advances.
#include "itts_qwen.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "mit2_bundle.hpp"
#include "qwen.hpp"

namespace q = itts::qwen;

namespace {

thread_local std::string g_qwen_create_error;

struct QwenFailure {
    int code;
    std::string msg;
};
[[noreturn]] void qfail(int code, const std::string& msg) { throw QwenFailure{code, msg}; }
[[noreturn]] void invalid(const std::string& msg) { qfail(ITTS_ERR_INVALID_ARGUMENT, msg); }

void qck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        qfail(e == cudaErrorMemoryAllocation ? ITTS_ERR_OUT_OF_MEMORY : ITTS_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
    }
}

template <class T>
T* dalloc(size_t n, const char* what) {
    void* p = nullptr;
    qck(cudaMalloc(&p, n * sizeof(T)), what);
    return static_cast<T*>(p);
}

constexpr int kCounters = 2048;  // >= output tiles of the largest prompt GEMM (gate|up at 3072 rows: 1152)

// The four prompt GEMM matrices of a layer: fp32 (decode), TF32 hi / lo (prompt).
enum Mat : int { kMatQkv = 0, kMatO = 1, kMatGu = 2, kMatDown = 3 };
constexpr int kMatRows[4] = {q::kQkv, q::kDim, 2 * q::kFfn, q::kDim};
constexpr int kMatCols[4] = {q::kDim, q::kQDim, q::kDim, q::kFfn};

}  // namespace

struct itts_qwen_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    std::vector<void*> allocs;
    q::Weights w{};
    q::Buffers b{};
    float* wsplit = nullptr;          // per layer and matrix: hi [rows][cols], then lo
    std::vector<itts::TmaMap> wmaps;  // [layer][matrix][hi, lo]
    itts::TmaMap amap[6];             // x, att, gu (hi, lo) for amap_rows rows
    int amap_rows = -1;
    float* ws = nullptr;
    int* counters = nullptr;
    q::State* h_state = nullptr;      // pinned
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    cudaEvent_t ev[3] = {nullptr, nullptr, nullptr};
    uint32_t cached = 0;
    itts_qwen_timing timing{};

    ~itts_qwen_ctx() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
        for (void* p : allocs) cudaFree(p);
        if (h_state) cudaFreeHost(h_state);
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        if (stream) cudaStreamDestroy(stream);
    }
    template <class T>
    T* alloc(size_t n, const char* what) {
        T* p = dalloc<T>(n, what);
        allocs.push_back(p);
        return p;
    }
};

namespace {

template <class F>
int qguard(itts_qwen_ctx* ctx, F&& f) {
    try {
        f();
        return ITTS_OK;
    } catch (const QwenFailure& e) {
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

// qwen.cpp:5-14, plus the norm weights run() reads.
void validate(const itts::Mit2Bundle& b) {
    if (b.target() != "index-tts2.5") qfail(ITTS_ERR_RUNTIME, "Expected an IndexTTS 2.5 model bundle");
    b.check_sizes();
    auto shape = [&](const std::string& name, std::vector<int64_t> want) {
        const auto* t = b.find(name);
        if (!t || t->shape != want) invalid("Unsupported Qwen shape: " + name);
    };
    shape("qwen.model.embed_tokens.weight", {q::kVocab, q::kDim});
    for (int i = 0; i < q::kLayers; ++i) {
        const std::string p = "qwen.model.layers." + std::to_string(i);
        shape(p + ".self_attn.q_proj.weight", {2048, 1024});
        shape(p + ".self_attn.k_proj.weight", {1024, 1024});
        shape(p + ".self_attn.v_proj.weight", {1024, 1024});
        shape(p + ".self_attn.o_proj.weight", {1024, 2048});
        shape(p + ".self_attn.q_norm.weight", {128});
        shape(p + ".self_attn.k_norm.weight", {128});
        shape(p + ".mlp.gate_proj.weight", {3072, 1024});
        shape(p + ".mlp.up_proj.weight", {3072, 1024});
        shape(p + ".mlp.down_proj.weight", {1024, 3072});
        shape(p + ".input_layernorm.weight", {1024});
        shape(p + ".post_attention_layernorm.weight", {1024});
    }
    shape("qwen.model.norm.weight", {1024});
}

const float* host_f32(const itts::Mit2Bundle& b, const std::string& name) {
    return reinterpret_cast<const float*>(b.data(b.info(name)));
}

float* upload(itts_qwen_ctx* c, const float* src, size_t n, const char* what) {
    float* d = c->alloc<float>(n, what);
    qck(cudaMemcpy(d, src, n * 4, cudaMemcpyHostToDevice), what);
    return d;
}

void load(itts_qwen_ctx* c, const itts::Mit2Bundle& b) {
    c->w.embed = upload(c, host_f32(b, "qwen.model.embed_tokens.weight"), size_t(q::kVocab) * q::kDim, "embedding");
    c->w.norm = upload(c, host_f32(b, "qwen.model.norm.weight"), q::kDim, "norm");
    size_t per_layer = 0;
    for (int m = 0; m < 4; ++m) per_layer += 2 * size_t(kMatRows[m]) * kMatCols[m];
    c->wsplit = c->alloc<float>(per_layer * q::kLayers, "split weights");
    c->wmaps.resize(size_t(q::kLayers) * 8);
    float* tmp = c->alloc<float>(size_t(2) * q::kFfn * q::kDim, "gate / up staging");
    std::vector<float> qkv(size_t(q::kQkv) * q::kDim);
    for (int l = 0; l < q::kLayers; ++l) {
        const std::string p = "qwen.model.layers." + std::to_string(l);
        q::LayerW& L = c->w.layer[l];
        L.ln1 = upload(c, host_f32(b, p + ".input_layernorm.weight"), q::kDim, "norm");
        L.ln2 = upload(c, host_f32(b, p + ".post_attention_layernorm.weight"), q::kDim, "norm");
        L.qn = upload(c, host_f32(b, p + ".self_attn.q_norm.weight"), q::kHeadDim, "norm");
        L.kn = upload(c, host_f32(b, p + ".self_attn.k_norm.weight"), q::kHeadDim, "norm");
        std::memcpy(qkv.data(), host_f32(b, p + ".self_attn.q_proj.weight"), size_t(q::kQDim) * q::kDim * 4);
        std::memcpy(qkv.data() + size_t(q::kQDim) * q::kDim, host_f32(b, p + ".self_attn.k_proj.weight"),
                    size_t(q::kKvDim) * q::kDim * 4);
        std::memcpy(qkv.data() + size_t(q::kQDim + q::kKvDim) * q::kDim, host_f32(b, p + ".self_attn.v_proj.weight"),
                    size_t(q::kKvDim) * q::kDim * 4);
        L.w_qkv = upload(c, qkv.data(), qkv.size(), "q|k|v weights");
        L.w_o = upload(c, host_f32(b, p + ".self_attn.o_proj.weight"), size_t(q::kDim) * q::kQDim, "o weights");
        qck(cudaMemcpy(tmp, host_f32(b, p + ".mlp.gate_proj.weight"), size_t(q::kFfn) * q::kDim * 4,
                       cudaMemcpyHostToDevice),
            "gate weights");
        qck(cudaMemcpy(tmp + size_t(q::kFfn) * q::kDim, host_f32(b, p + ".mlp.up_proj.weight"),
                       size_t(q::kFfn) * q::kDim * 4, cudaMemcpyHostToDevice),
            "up weights");
        float* gu = c->alloc<float>(size_t(2) * q::kFfn * q::kDim, "gate|up weights");
        qck(q::launch_interleave_rows(tmp, tmp + size_t(q::kFfn) * q::kDim, gu, q::kFfn, q::kDim, c->stream),
            "gate|up interleave");
        qck(cudaStreamSynchronize(c->stream), "gate|up interleave");
        L.w_gu = gu;
        L.w_down = upload(c, host_f32(b, p + ".mlp.down_proj.weight"), size_t(q::kDim) * q::kFfn, "down weights");
        const float* src[4] = {L.w_qkv, L.w_o, L.w_gu, L.w_down};
        float* dst = c->wsplit + per_layer * l;
        for (int m = 0; m < 4; ++m) {
            const size_t n = size_t(kMatRows[m]) * kMatCols[m];
            qck(itts::tma_split(src[m], dst, dst + n, n, c->stream), "weight split");
            qck(itts::tma_make_map(&c->wmaps[(l * 4 + m) * 2], dst, kMatRows[m], kMatCols[m]), "tensor map");
            qck(itts::tma_make_map(&c->wmaps[(l * 4 + m) * 2 + 1], dst + n, kMatRows[m], kMatCols[m]), "tensor map");
            dst += 2 * n;
        }
    }
}

void alloc_buffers(itts_qwen_ctx* c) {
    const size_t T = q::kMaxPrompt;
    q::Buffers& b = c->b;
    b.hidden = c->alloc<float>(T * q::kDim, "hidden");
    b.qkv = c->alloc<float>(T * q::kQkv, "qkv");
    b.x_hi = c->alloc<float>(T * q::kDim, "x");
    b.x_lo = c->alloc<float>(T * q::kDim, "x");
    b.att_hi = c->alloc<float>(T * q::kQDim, "attention");
    b.att_lo = c->alloc<float>(T * q::kQDim, "attention");
    b.gu_hi = c->alloc<float>(T * q::kFfn, "swiglu");
    b.gu_lo = c->alloc<float>(T * q::kFfn, "swiglu");
    b.part = c->alloc<float>(size_t(q::kQHeads) * q::kMaxChunks * q::kPartStride, "attention partials");
    b.logits = c->alloc<float>(q::kVocab, "logits");
    b.best = c->alloc<float>(size_t(2) * q::kHeadCtas, "argmax partials");
    b.kv = c->alloc<float>(size_t(q::kLayers) * 2 * q::kCap * q::kKvDim, "KV cache");
    b.ids = c->alloc<uint32_t>(T, "prompt ids");
    b.out = c->alloc<uint32_t>(q::kMaxGenerate + 1, "selected ids");
    b.st = c->alloc<q::State>(1, "decode state");
    b.cnt = c->alloc<int>(16, "arrival counters");
    qck(cudaMemset(b.cnt, 0, 16 * 4), "arrival counters");
    b.status = c->alloc<int>(4, "status");
    qck(cudaMemset(b.status, 0, 16), "status");
    c->ws = c->alloc<float>(itts::tma_workspace_floats(), "GEMM workspace");
    c->counters = c->alloc<int>(kCounters, "GEMM counters");
    qck(cudaMemset(c->counters, 0, kCounters * 4), "GEMM counters");
    void* h = nullptr;
    qck(cudaMallocHost(&h, sizeof(q::State)), "pinned state");
    c->h_state = static_cast<q::State*>(h);
}

void put_state(itts_qwen_ctx* c, uint32_t token, uint32_t pos, uint32_t max_out) {
    *c->h_state = q::State{token, pos, 0u, 0u, max_out, {0u, 0u, 0u}};
    qck(cudaMemcpyAsync(c->b.st, c->h_state, sizeof(q::State), cudaMemcpyHostToDevice, c->stream), "state upload");
}

void get_state(itts_qwen_ctx* c) {
    qck(cudaMemcpyAsync(c->h_state, c->b.st, sizeof(q::State), cudaMemcpyDeviceToHost, c->stream), "state read");
    qck(cudaStreamSynchronize(c->stream), "qwen");
}

void gemm(itts_qwen_ctx* c, int layer, int m, const itts::TmaMap* a, int epi, const float* R, float* C, float* C_lo,
          int T) {
    itts::TmaGemm g{a,      &c->wmaps[(layer * 4 + m) * 2], nullptr,          R,  C, C_lo, T, kMatRows[m],
                    kMatCols[m], epi, c->ws, c->counters, kCounters, c->b.status};
    qck(itts::tma_gemm(g, c->stream), "prompt GEMM");
}

// The prompt pass (qwen.cpp:24-43 with t = n, offset 0): logits of the last
// position and the argmax into the State (out[0]).
void run_prompt(itts_qwen_ctx* c, const uint32_t* ids, size_t n, uint32_t max_out) {
    for (size_t i = 0; i < n; ++i)
        if (ids[i] >= uint32_t(q::kVocab)) invalid("Invalid Qwen token");
    const int T = int(n);
    q::Buffers& b = c->b;
    if (c->amap_rows != T) {
        const float* base[6] = {b.x_hi, b.x_lo, b.att_hi, b.att_lo, b.gu_hi, b.gu_lo};
        const int cols[6] = {q::kDim, q::kDim, q::kQDim, q::kQDim, q::kFfn, q::kFfn};
        for (int i = 0; i < 6; ++i) qck(itts::tma_make_map(&c->amap[i], base[i], T, cols[i]), "tensor map");
        c->amap_rows = T;
    }
    qck(cudaEventRecord(c->ev[0], c->stream), "event");
    qck(cudaMemcpyAsync(b.ids, ids, n * 4, cudaMemcpyHostToDevice, c->stream), "prompt upload");
    put_state(c, 0, uint32_t(n), max_out);
    qck(cudaMemsetAsync(c->counters, 0, kCounters * 4, c->stream), "GEMM counters");
    qck(q::launch_embed(c->w, b, T, c->stream), "embedding");
    for (int l = 0; l < q::kLayers; ++l) {
        const q::LayerW& L = c->w.layer[l];
        qck(q::launch_rmsnorm_split(b.hidden, L.ln1, b.x_hi, b.x_lo, T, c->stream), "rmsnorm");
        gemm(c, l, kMatQkv, &c->amap[0], itts::TmaEpiBias, nullptr, b.qkv, nullptr, T);
        qck(q::launch_qk_norm_rope(L, b, l, T, false, c->stream), "q/k norm + rope");
        qck(q::launch_attn_prefill(b, l, T, c->stream), "attention");
        gemm(c, l, kMatO, &c->amap[2], itts::TmaEpiResid, b.hidden, b.hidden, nullptr, T);
        qck(q::launch_rmsnorm_split(b.hidden, L.ln2, b.x_hi, b.x_lo, T, c->stream), "rmsnorm");
        gemm(c, l, kMatGu, &c->amap[0], itts::TmaEpiSwiGLU, nullptr, b.gu_hi, b.gu_lo, T);
        gemm(c, l, kMatDown, &c->amap[4], itts::TmaEpiResid, b.hidden, b.hidden, nullptr, T);
    }
    qck(q::launch_head(c->w, b, b.hidden + size_t(T - 1) * q::kDim, false, c->stream), "head");
    qck(cudaEventRecord(c->ev[1], c->stream), "event");
}

void ensure_graph(itts_qwen_ctx* c) {
    if (c->exec) return;
    qck(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "graph capture");
    cudaError_t e = q::launch_decode_embed(c->w, c->b, c->stream);
    for (int l = 0; l < q::kLayers && e == cudaSuccess; ++l) e = q::launch_decode_layer(c->w.layer[l], c->b, l, c->stream);
    if (e == cudaSuccess) e = q::launch_head(c->w, c->b, c->b.hidden, true, c->stream);
    cudaGraph_t g = nullptr;
    const cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        qck(e, "decode step capture");
    }
    qck(e2, "graph capture");
    c->graph = g;
    qck(cudaGraphInstantiate(&c->exec, g, 0), "graph instantiate");
}

void check_status(itts_qwen_ctx* c) {
    int st[4] = {0, 0, 0, 0};
    qck(cudaMemcpy(st, c->b.status, sizeof st, cudaMemcpyDeviceToHost), "status read");
    if (st[0]) {
        qck(cudaMemset(c->b.status, 0, sizeof st), "status reset");
        qfail(ITTS_ERR_DEVICE_TIMEOUT, "device wait timed out (status " + std::to_string(st[0]) + ")");
    }
}

float elapsed(cudaEvent_t a, cudaEvent_t b) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, a, b);
    return ms;
}

}  // namespace

extern "C" {

const char* itts_qwen_last_error(const itts_qwen_ctx* ctx) {
    return ctx ? ctx->err.c_str() : g_qwen_create_error.c_str();
}

int itts_qwen_create(const char* bundle_dir, int device, itts_qwen_ctx** out) {
    g_qwen_create_error.clear();
    if (!out) {
        g_qwen_create_error = "out is null";
        return ITTS_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    std::unique_ptr<itts_qwen_ctx> c(new (std::nothrow) itts_qwen_ctx());
    if (!c) return ITTS_ERR_OUT_OF_MEMORY;
    c->device = device;
    const int rc = qguard(c.get(), [&] {
        if (!bundle_dir) invalid("bundle_dir is null");
        itts::Mit2Bundle bundle(bundle_dir);
        validate(bundle);
        int n = 0;
        qck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) invalid("device index out of range");
        qck(cudaSetDevice(device), "cudaSetDevice");
        cudaDeviceProp prop{};
        qck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major < 10) qfail(ITTS_ERR_RUNTIME, "this library is built for sm_100a (B200) devices only");
        qck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream creation");
        for (cudaEvent_t& e : c->ev) qck(cudaEventCreate(&e), "event creation");
        qck(q::init_tables(), "RoPE table");
        qck(q::prepare_kernels(), "kernel configuration");
        alloc_buffers(c.get());
        load(c.get(), bundle);
        qck(cudaDeviceSynchronize(), "load");
    });
    if (rc != ITTS_OK) {
        g_qwen_create_error = c->err;
        return rc;
    }
    *out = c.release();
    return ITTS_OK;
}

void itts_qwen_destroy(itts_qwen_ctx* ctx) { delete ctx; }

uint32_t itts_qwen_cached_tokens(const itts_qwen_ctx* ctx) { return ctx ? ctx->cached : 0; }

int itts_qwen_last_timing(const itts_qwen_ctx* ctx, itts_qwen_timing* out) {
    if (!ctx || !out) return ITTS_ERR_INVALID_ARGUMENT;
    *out = ctx->timing;
    return ITTS_OK;
}

int itts_qwen_prefill(itts_qwen_ctx* ctx, const uint32_t* ids, size_t n, float* logits) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return qguard(ctx, [&] {
        qck(cudaSetDevice(ctx->device), "cudaSetDevice");
        if (!ids || n == 0 || n > size_t(q::kMaxPrompt)) invalid("Qwen prompt capacity is 3072 tokens");
        ctx->cached = 0;
        run_prompt(ctx, ids, n, q::kMaxGenerate + 1);
        if (logits)
            qck(cudaMemcpyAsync(logits, ctx->b.logits, size_t(q::kVocab) * 4, cudaMemcpyDeviceToHost, ctx->stream),
                "logits read");
        get_state(ctx);
        check_status(ctx);
        ctx->cached = uint32_t(n);
        ctx->timing = itts_qwen_timing{elapsed(ctx->ev[0], ctx->ev[1]), 0.f, 0u, uint32_t(n)};
    });
}

int itts_qwen_step(itts_qwen_ctx* ctx, uint32_t id, float* logits) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return qguard(ctx, [&] {
        qck(cudaSetDevice(ctx->device), "cudaSetDevice");
        if (!ctx->cached || ctx->cached >= uint32_t(q::kCap)) invalid("Qwen cache capacity exceeded");
        if (id >= uint32_t(q::kVocab)) invalid("Invalid Qwen token");
        ensure_graph(ctx);
        put_state(ctx, id, ctx->cached, 1);
        qck(cudaEventRecord(ctx->ev[1], ctx->stream), "event");
        qck(cudaGraphLaunch(ctx->exec, ctx->stream), "decode step");
        qck(cudaEventRecord(ctx->ev[2], ctx->stream), "event");
        if (logits)
            qck(cudaMemcpyAsync(logits, ctx->b.logits, size_t(q::kVocab) * 4, cudaMemcpyDeviceToHost, ctx->stream),
                "logits read");
        get_state(ctx);
        check_status(ctx);
        ++ctx->cached;
        ctx->timing = itts_qwen_timing{0.f, elapsed(ctx->ev[1], ctx->ev[2]), 1u, 0u};
    });
}

int itts_qwen_generate(itts_qwen_ctx* ctx, const uint32_t* ids, size_t n, uint32_t maximum, uint32_t* out,
                       size_t out_cap, uint32_t* n_out) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return qguard(ctx, [&] {
        qck(cudaSetDevice(ctx->device), "cudaSetDevice");
        // qwen.cpp:45-46, in that order
        if (!maximum || maximum > uint32_t(q::kMaxGenerate) || n + maximum > size_t(q::kCap))
            invalid("Qwen generation capacity exceeded");
        if (!ids || n == 0 || n > size_t(q::kMaxPrompt)) invalid("Qwen prompt capacity is 3072 tokens");
        if (!out || !n_out || out_cap < maximum) invalid("output buffer too small");
        ensure_graph(ctx);
        ctx->cached = 0;
        run_prompt(ctx, ids, n, maximum);
        // Steps in groups; the State's done flag (EOS or `maximum` ids) makes
        // every kernel of later steps return at once.
        uint32_t steps = 0;
        get_state(ctx);
        while (!ctx->h_state->done && steps + 1 < maximum) {
            const uint32_t k = std::min<uint32_t>(8, maximum - 1 - steps);
            for (uint32_t i = 0; i < k; ++i) qck(cudaGraphLaunch(ctx->exec, ctx->stream), "decode step");
            steps += k;
            get_state(ctx);
        }
        qck(cudaEventRecord(ctx->ev[2], ctx->stream), "event");
        check_status(ctx);
        const q::State st = *ctx->h_state;
        std::vector<uint32_t> sel(st.n_out);
        if (st.n_out)
            qck(cudaMemcpy(sel.data(), ctx->b.out, size_t(st.n_out) * 4, cudaMemcpyDeviceToHost), "ids read");
        ctx->cached = uint32_t(n) + (st.n_out ? st.n_out - 1 : 0);
        qck(cudaEventSynchronize(ctx->ev[2]), "qwen");
        ctx->timing = itts_qwen_timing{elapsed(ctx->ev[0], ctx->ev[1]), elapsed(ctx->ev[1], ctx->ev[2]),
                                       st.n_out ? st.n_out - 1 : 0, uint32_t(n)};
        std::memcpy(out, sel.data(), sel.size() * 4);
        *n_out = st.n_out;
        if (sel.empty() || sel.back() != q::kEos)
            qfail(ITTS_ERR_RUNTIME, "Qwen did not reach EOS within 1024 generated tokens");
    });
}

}  // extern "C"
