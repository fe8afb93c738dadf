// Host runtime of the B200 GPT decoder: implements include/itts_gpt.h.
//
// Mirrors the reference's GptDecoder (src/gpt.cpp, src/gpt_sampling.cpp):
// the same argument checks and error classes, the same generation loop
// semantics (history seeded with {1, 8192}, first generated code at mel
// position 2, stop code 8193, codes >= 8192 rejected), the same beam-search
// bookkeeping.  All tensor math runs on the device (decode.cu, prefill.cu,
// misc.cu); the host owns validation, memory and launch order.
#include "itts_gpt.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <memory>
#include <new>
#include <numeric>
#include <string>
#include <vector>

#include "mit2_bundle.hpp"
#include "model.hpp"

namespace {

thread_local std::string g_create_error;

struct Failure {
    int code;
    std::string msg;
};

[[noreturn]] void fail(int code, const std::string& msg) { throw Failure{code, msg}; }
[[noreturn]] void invalid(const std::string& msg) { fail(ITTS_ERR_INVALID_ARGUMENT, msg); }

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(e == cudaErrorMemoryAllocation ? ITTS_ERR_OUT_OF_MEMORY : ITTS_ERR_CUDA,
             std::string(what) + ": " + cudaGetErrorString(e));
    }
}

constexpr uint32_t kW = 1280, kVocab = 8194, kCap = 4096, kH = 20, kHd = 64;

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

template <class T>
T* dev_alloc(size_t count, const char* what) {
    void* p = nullptr;
    ck(cudaMalloc(&p, count * sizeof(T)), what);
    return static_cast<T*>(p);
}

}  // namespace

struct itts_gpt_state {
    int device = 0;
    uint32_t tokens = 0, layers = 0;
    float* d = nullptr;  // [layer][K|V][head][tokens][64]
    ~itts_gpt_state() {
        if (d) {
            int cur = 0;
            cudaGetDevice(&cur);
            cudaSetDevice(device);
            cudaFree(d);
            cudaSetDevice(cur);
        }
    }
};

struct itts_gpt_ctx {
    int device = 0, dtype = 0, sm_count = 0, mode = 0;
    int prefill_mode = 0;           // 0: tensor-core GEMMs, 1: CUDA-core fp32 tiles
    itts::TmaPrefill tma{};         // TF32-split weights and activations of the tensor-core prefill
    cudaStream_t stream = nullptr;
    std::string err;
    uint32_t layers = 0, mel_pos_rows = 0, text_pos_rows = 0;
    char* d_weights = nullptr;
    size_t weight_bytes = 0;
    uint64_t stream_bytes = 0;
    itts::ModelW hw{};
    itts::ModelW* d_model = nullptr;
    const float *spk_w = nullptr, *spk_b = nullptr, *text_emb = nullptr, *text_pos = nullptr, *lang_emb = nullptr;
    float* d_kv = nullptr;
    float *d_hidden = nullptr, *d_x = nullptr, *d_qkv = nullptr, *d_att = nullptr, *d_r = nullptr, *d_ff = nullptr;
    float* d_att_part = nullptr;  // prefill attention chunk partials (inside the d_hidden block)
    int* d_att_cnt = nullptr;     // their arrival counters (inside the d_hidden block)
    float* d_act = nullptr;
    itts::DecodeBuffers db{};
    uint32_t* d_history = nullptr;  // {1, 8192}
    uint32_t* d_codes = nullptr;    // [kCap]
    uint32_t* d_info = nullptr;     // [4]
    float* d_misc = nullptr;        // prepare inputs / processor buffers
    size_t tagged_bytes = 0;        // bytes of the tagged hand-off region (db.qkv ...)
    uint32_t* d_hist = nullptr;     // processor history (grown on demand)
    size_t d_hist_cap = 0;
    void* d_sampler_big = nullptr;  // per-CTA sampler workspace
    float* h_stage = nullptr;       // pinned [1024 * 1280]
    float* h_logits = nullptr;      // pinned [8194 * 10]
    uint32_t* h_codes = nullptr;    // pinned [kCap]
    itts::DecodeCtl* h_ctl = nullptr;
    uint32_t cached = 0, prefix_rows = 0;
    bool have_prefill = false;
    uint64_t launches = 0;
    unsigned long long wait_ns = 0;  // device wait limit of decode launches (0: the kernels' default)
    // batched decode (allocated on first use): KV arenas, activations, state
    float* d_bkv = nullptr;          // b_arenas KV arenas of arena_floats each
    uint32_t b_arenas = 0;
    size_t arena_floats = 0;
    char* d_bact = nullptr;          // activations, partials, counters, state, sets, codes, beam buffers
    void* d_bbig = nullptr;          // kMaxBatch sampler workspaces
    itts::BatchArgs bargs{};         // pointers into d_bact (M, options and flags are set per call)
    float* d_bscores = nullptr;      // beam search: [kMaxBatch][8194] scores
    float* d_btmp = nullptr;         // beam search: [kMaxBatch][8448] log-softmax scratch
    uint32_t* d_bhist = nullptr;     // beam search: [kMaxBatch][kCap + 2] histories
    itts::BatchState* h_bstate = nullptr;  // pinned
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};  // generate timing: start, prefill done, decode done; serve start
    itts_gpt_timing timing{};        // accumulated over the last generate / generate_batch call
    bool pending = false;           // an async decode has not been synced yet
    uint32_t* pending_info = nullptr;

    ~itts_gpt_ctx() {
        cudaSetDevice(device);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : {(void*)d_weights, (void*)d_model, (void*)d_kv, (void*)d_hidden, (void*)d_act,
                        (void*)d_history, (void*)d_codes, (void*)d_info, (void*)d_misc, (void*)d_hist,
                        d_sampler_big, (void*)d_bkv, (void*)d_bact, d_bbig})
            if (p) cudaFree(p);
        for (void* p : {(void*)h_stage, (void*)h_logits, (void*)h_codes, (void*)h_ctl, (void*)h_bstate})
            if (p) cudaFreeHost(p);
        for (cudaEvent_t e : ev)
            if (e) cudaEventDestroy(e);
        itts::tma_prefill_free(&tma);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

template <class F>
int guard(itts_gpt_ctx* ctx, F&& f, bool set_device = true) {
    try {
        if (ctx && set_device) ck(cudaSetDevice(ctx->device), "cudaSetDevice");
        f();
        return ITTS_OK;
    } catch (const Failure& e) {
        if (ctx) ctx->err = e.msg;
        return e.code;
    } catch (const std::bad_alloc&) {
        if (ctx) ctx->err = "host allocation failed";
        return ITTS_ERR_OUT_OF_MEMORY;
    } catch (const std::invalid_argument& e) {
        if (ctx) ctx->err = e.what();
        return ITTS_ERR_INVALID_ARGUMENT;
    } catch (const std::exception& e) {
        if (ctx) ctx->err = e.what();
        return ITTS_ERR_RUNTIME;
    }
}

// ---------------------------------------------------------------- loading
// src/weights.cpp:11-27 and src/gpt.cpp:8-23: container, target and shape
// checks.  Host only, so malformed bundles are rejected before any CUDA call.
void validate_bundle(itts_gpt_ctx* c, const itts::Mit2Bundle& b) {
    if (b.target() != "index-tts2.5") fail(ITTS_ERR_RUNTIME, "Expected an IndexTTS 2.5 model bundle");
    b.check_sizes();
    auto shape = [&](const std::string& n, std::vector<int64_t> want) {
        if (b.info(n).shape != want) fail(ITTS_ERR_RUNTIME, "Unsupported 2.5 GPT shape: " + n);
    };
    // gpt.cpp:8-23
    shape("gpt.spk_emb_proj.weight", {1280, 192});
    shape("gpt.text_embedding.weight", {60510, 1280});
    shape("gpt.lang_embedding.weight", {107, 1280});
    shape("gpt.mel_embedding.weight", {8194, 1280});
    uint32_t layers = 0;
    while (layers < 24 && b.find("gpt.gpt.h." + std::to_string(layers) + ".ln_1.weight")) ++layers;
    if (!layers) fail(ITTS_ERR_RUNTIME, "bundle has no GPT layers");
    const char* conv[4] = {"attn.c_attn", "attn.c_proj", "mlp.c_fc", "mlp.c_proj"};
    const std::vector<int64_t> conv_shape[4] = {{1280, 3840}, {1280, 1280}, {1280, 5120}, {5120, 1280}};
    for (uint32_t i = 0; i < layers; ++i)
        for (int k = 0; k < 4; ++k) shape("gpt.gpt.h." + std::to_string(i) + "." + conv[k] + ".weight", conv_shape[k]);
    auto vec = [&](const std::string& n, int64_t len) { shape(n, {len}); };
    for (uint32_t i = 0; i < layers; ++i) {
        const std::string p = "gpt.gpt.h." + std::to_string(i);
        vec(p + ".ln_1.weight", 1280);
        vec(p + ".ln_1.bias", 1280);
        vec(p + ".ln_2.weight", 1280);
        vec(p + ".ln_2.bias", 1280);
        vec(p + ".attn.c_attn.bias", 3840);
        vec(p + ".attn.c_proj.bias", 1280);
        vec(p + ".mlp.c_fc.bias", 5120);
        vec(p + ".mlp.c_proj.bias", 1280);
    }
    for (const char* n : {"gpt.gpt.ln_f.weight", "gpt.gpt.ln_f.bias", "gpt.final_norm.weight", "gpt.final_norm.bias"})
        vec(n, 1280);
    vec("gpt.spk_emb_proj.bias", 1280);
    shape("gpt.mel_head.weight", {8194, 1280});
    vec("gpt.mel_head.bias", 8194);
    const auto& mp = b.info("gpt.mel_pos_embedding.emb.weight");
    const auto& tp = b.info("gpt.text_pos_embedding.emb.weight");
    if (mp.shape.size() != 2 || mp.shape[1] != 1280 || mp.shape[0] < 3)
        fail(ITTS_ERR_RUNTIME, "Unsupported 2.5 GPT shape: gpt.mel_pos_embedding.emb.weight");
    if (tp.shape.size() != 2 || tp.shape[1] != 1280)
        fail(ITTS_ERR_RUNTIME, "Unsupported 2.5 GPT shape: gpt.text_pos_embedding.emb.weight");
    c->layers = layers;
    c->mel_pos_rows = uint32_t(mp.shape[0]);
    c->text_pos_rows = uint32_t(tp.shape[0]);
}

void upload_weights(itts_gpt_ctx* c, const itts::Mit2Bundle& b) {
    const uint32_t layers = c->layers;
    // device layout: every tensor 256-byte aligned in one allocation
    std::vector<std::pair<const itts::TensorInfo*, size_t>> plan;
    size_t total = 0;
    // the streamed matrices (Conv1D blocks and mel_head) are bf16 in a bf16 context
    const bool wb = c->dtype == ITTS_WEIGHTS_BF16;
    auto is_conv = [](const itts::TensorInfo& t) { return t.name.rfind("gpt.gpt.h.", 0) == 0 && t.shape.size() == 2; };
    auto is_matrix = [&](const itts::TensorInfo& t) { return is_conv(t) || t.name == "gpt.mel_head.weight"; };
    auto dev_bytes = [&](const itts::TensorInfo& t) { return wb && is_matrix(t) ? t.nbytes / 2 : t.nbytes; };
    auto add = [&](const std::string& n) {
        const auto* t = &b.info(n);
        plan.emplace_back(t, total);
        total += align256(dev_bytes(*t));
        return plan.size() - 1;
    };
    std::vector<size_t> idx;
    for (const char* n : {"gpt.spk_emb_proj.weight", "gpt.spk_emb_proj.bias", "gpt.text_embedding.weight",
                          "gpt.text_pos_embedding.emb.weight", "gpt.lang_embedding.weight",
                          "gpt.mel_embedding.weight", "gpt.mel_pos_embedding.emb.weight", "gpt.gpt.ln_f.weight",
                          "gpt.gpt.ln_f.bias", "gpt.final_norm.weight", "gpt.final_norm.bias",
                          "gpt.mel_head.weight", "gpt.mel_head.bias"})
        idx.push_back(add(n));
    const char* per_layer[12] = {"ln_1.weight", "ln_1.bias", "attn.c_attn.weight", "attn.c_attn.bias",
                                 "attn.c_proj.weight", "attn.c_proj.bias", "ln_2.weight", "ln_2.bias",
                                 "mlp.c_fc.weight", "mlp.c_fc.bias", "mlp.c_proj.weight", "mlp.c_proj.bias"};
    for (uint32_t i = 0; i < layers; ++i)
        for (const char* n : per_layer) idx.push_back(add("gpt.gpt.h." + std::to_string(i) + "." + n));
    c->d_weights = dev_alloc<char>(total, "weight allocation");
    c->weight_bytes = total;

    // upload; Conv1D matrices go through a staging buffer and a transpose,
    // bf16 matrices are rounded to nearest even on the device
    float* stage = dev_alloc<float>(size_t(wb ? 8194 : 5120) * 1280, "transpose staging");
    try {
        for (const auto& pe : plan) {
            const itts::TensorInfo& t = *pe.first;
            char* dst = c->d_weights + pe.second;
            if (is_conv(t)) {
                ck(cudaMemcpy(stage, b.data(t), t.nbytes, cudaMemcpyHostToDevice), "weight upload");
                ck(wb ? itts::launch_transpose_bf16(stage, dst, int(t.shape[0]), int(t.shape[1]), nullptr)
                      : itts::launch_transpose(stage, reinterpret_cast<float*>(dst), int(t.shape[0]),
                                               int(t.shape[1]), nullptr),
                   "transpose launch");
                ck(cudaDeviceSynchronize(), "transpose");
            } else if (wb && is_matrix(t)) {
                ck(cudaMemcpy(stage, b.data(t), t.nbytes, cudaMemcpyHostToDevice), "weight upload");
                ck(itts::launch_to_bf16(stage, dst, t.nbytes / 4, nullptr), "bf16 conversion launch");
                ck(cudaDeviceSynchronize(), "bf16 conversion");
            } else {
                ck(cudaMemcpy(dst, b.data(t), t.nbytes, cudaMemcpyHostToDevice), "weight upload");
            }
        }
    } catch (...) {
        cudaFree(stage);
        throw;
    }
    cudaFree(stage);
    auto ptr = [&](size_t i) { return reinterpret_cast<const float*>(c->d_weights + plan[idx[i]].second); };
    c->spk_w = ptr(0);
    c->spk_b = ptr(1);
    c->text_emb = ptr(2);
    c->text_pos = ptr(3);
    c->lang_emb = ptr(4);
    c->hw.mel_emb = ptr(5);
    c->hw.mel_pos = ptr(6);
    c->hw.lnf_g = ptr(7);
    c->hw.lnf_b = ptr(8);
    c->hw.fn_g = ptr(9);
    c->hw.fn_b = ptr(10);
    c->hw.w_head = ptr(11);
    c->hw.b_head = ptr(12);
    c->hw.layers = int(layers);
    for (uint32_t i = 0; i < layers; ++i) {
        const size_t o = 13 + size_t(i) * 12;
        itts::LayerW& L = c->hw.layer[i];
        L.ln1_g = ptr(o + 0);
        L.ln1_b = ptr(o + 1);
        L.w_qkv = ptr(o + 2);
        L.b_qkv = ptr(o + 3);
        L.w_o = ptr(o + 4);
        L.b_o = ptr(o + 5);
        L.ln2_g = ptr(o + 6);
        L.ln2_b = ptr(o + 7);
        L.w_fc = ptr(o + 8);
        L.b_fc = ptr(o + 9);
        L.w_mp = ptr(o + 10);
        L.b_mp = ptr(o + 11);
    }
    // algorithmic bytes streamed per decode step: matrices, biases, LayerNorms,
    // mel_head and its bias, the final LayerNorms, two embedding rows
    const uint64_t mat_elems = 19660800ull * layers + 10488320ull;
    const uint64_t vec_floats = (11520ull + 5120ull) * layers + 8194ull + 5120ull + 2560ull;
    c->stream_bytes = (wb ? 2ull : 4ull) * mat_elems + 4ull * vec_floats;
}

void alloc_buffers(itts_gpt_ctx* c) {
    const size_t kv_floats = size_t(c->layers) * 2 * kH * kCap * kHd;
    c->d_kv = dev_alloc<float>(kv_floats, "KV cache allocation");
    const size_t T = 1024;
    // hidden, x, att, r + qkv + ff + attention partials + their counters
    const size_t pre = T * kW * 4 + T * 3840 + T * 5120 + itts::kAttPartFloats + itts::kAttCounters;
    c->d_hidden = dev_alloc<float>(pre, "prefill scratch");
    c->d_x = c->d_hidden + T * kW;
    c->d_att = c->d_x + T * kW;
    c->d_r = c->d_att + T * kW;
    c->d_qkv = c->d_r + T * kW;
    c->d_ff = c->d_qkv + T * 3840;
    c->d_att_part = c->d_ff + T * 5120;
    c->d_att_cnt = reinterpret_cast<int*>(c->d_att_part + itts::kAttPartFloats);
    ck(cudaMemset(c->d_att_cnt, 0, itts::kAttCounters * sizeof(int)), "prefill scratch");
    // decode activations (each region 256-byte aligned): the tagged hand-off
    // words (qkv, h, hm, attn, f), logits, attention partials, control block
    const size_t sizes[8] = {3840 * 8, kW * 8, kW * 8, kW * 8, 5120 * 8, 8448 * 4, size_t(kH) * 256 * 68 * 4,
                             sizeof(itts::DecodeCtl)};
    size_t total = 0;
    for (size_t s : sizes) total += align256(s);
    c->d_act = reinterpret_cast<float*>(dev_alloc<char>(total, "decode buffers"));
    char* p = reinterpret_cast<char*>(c->d_act);
    char* regions[8];
    for (int i = 0; i < 8; ++i) {
        regions[i] = p;
        p += align256(sizes[i]);
    }
    c->tagged_bytes = size_t(regions[5] - regions[0]);
    c->db.kv = c->d_kv;
    c->db.qkv = reinterpret_cast<unsigned long long*>(regions[0]);
    c->db.h = reinterpret_cast<unsigned long long*>(regions[1]);
    c->db.hm = reinterpret_cast<unsigned long long*>(regions[2]);
    c->db.attn = reinterpret_cast<unsigned long long*>(regions[3]);
    c->db.f = reinterpret_cast<float*>(regions[4]);
    c->db.logits = reinterpret_cast<float*>(regions[5]);
    c->db.part = reinterpret_cast<float*>(regions[6]);
    c->db.ctl = reinterpret_cast<itts::DecodeCtl*>(regions[7]);
    c->db.sampler_big = reinterpret_cast<itts::SamplerBig*>(
        dev_alloc<char>(size_t(c->sm_count) * itts::sampler_big_bytes(), "sampler workspace"));
    c->d_sampler_big = c->db.sampler_big;
    ck(cudaMemset(c->d_act, 0, total), "decode buffer init");
    c->d_history = dev_alloc<uint32_t>(2, "history");
    const uint32_t hist[2] = {1, 8192};
    ck(cudaMemcpy(c->d_history, hist, sizeof hist, cudaMemcpyHostToDevice), "history upload");
    c->d_codes = dev_alloc<uint32_t>(kCap, "codes");
    c->d_info = dev_alloc<uint32_t>(4, "info");
    c->d_misc = dev_alloc<float>(192 + 1280 + 1024 + 2 * 8448, "misc buffers");
    ck(cudaMallocHost(&c->h_stage, T * kW * 4), "pinned staging");
    ck(cudaMallocHost(&c->h_logits, size_t(kVocab) * 10 * 4), "pinned logits");
    ck(cudaMallocHost(&c->h_codes, kCap * 4), "pinned codes");
    ck(cudaMallocHost(&c->h_ctl, sizeof(itts::DecodeCtl)), "pinned control");
    c->d_model = dev_alloc<itts::ModelW>(1, "model table");
    ck(cudaMemcpy(c->d_model, &c->hw, sizeof(itts::ModelW), cudaMemcpyHostToDevice), "model table upload");
}

// ------------------------------------------------------------- execution
void check_status(itts_gpt_ctx* c) {
    ck(cudaMemcpyAsync(c->h_ctl, c->db.ctl, sizeof(itts::DecodeCtl), cudaMemcpyDeviceToHost, c->stream), "status read");
    ck(cudaStreamSynchronize(c->stream), "stream sync");
    const int code = c->h_ctl->status[0];
    if (!code) return;
    const std::string where = " (site " + std::to_string(c->h_ctl->status[1]) + ", cta " +
                              std::to_string(c->h_ctl->status[2]) + ", detail " + std::to_string(c->h_ctl->status[3]) + ")";
    switch (code) {
        case itts::kStatusInvalidCode: fail(ITTS_ERR_RUNTIME, "GPT generated invalid semantic code");
        case itts::kStatusNoFiniteLogits: fail(ITTS_ERR_RUNTIME, "GPT sampling received no finite logits");
        case itts::kStatusZeroMass: fail(ITTS_ERR_RUNTIME, "GPT sampling probability mass is zero");
        case itts::kStatusBarrierTimeout: fail(ITTS_ERR_DEVICE_TIMEOUT, "device grid barrier timed out" + where);
        default: fail(ITTS_ERR_RUNTIME, "device error " + std::to_string(code) + where);
    }
}

void finish_pending(itts_gpt_ctx* c) {
    if (!c->pending) return;
    c->pending = false;
    uint32_t info[4] = {0, 0, 0, 0};
    ck(cudaMemcpyAsync(info, c->pending_info, sizeof info, cudaMemcpyDeviceToHost, c->stream), "info read");
    check_status(c);
    c->cached += info[3];
}

void reset_ctl(itts_gpt_ctx* c) {
    ck(cudaMemsetAsync(c->db.ctl, 0, sizeof(itts::DecodeCtl), c->stream), "control reset");
}

itts::DecodeArgs decode_args(itts_gpt_ctx* c) {
    itts::DecodeArgs a{};
    a.w = c->d_model;
    a.b = c->db;
    a.history = c->d_history;
    a.history_n = 2;
    a.codes = c->d_codes;
    a.wait_ns = c->wait_ns;
    return a;
}

void launch_decode(itts_gpt_ctx* c, const itts::DecodeArgs& a) {
    reset_ctl(c);
    // epochs restart at 1 in every launch: clear the tagged hand-off words
    ck(cudaMemsetAsync(c->db.qkv, 0, c->tagged_bytes, c->stream), "hand-off reset");
    if (c->mode == 0) {
        ck(c->dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::launch_decode_persistent(a, c->sm_count, c->stream)
                                         : itts::wf32::launch_decode_persistent(a, c->sm_count, c->stream),
           "persistent decode launch");
        ++c->launches;
    } else {
        ck(c->dtype == ITTS_WEIGHTS_BF16
               ? itts::wbf16::launch_decode_layered(a, int(c->layers), c->sm_count, c->stream, &c->launches)
               : itts::wf32::launch_decode_layered(a, int(c->layers), c->sm_count, c->stream, &c->launches),
           "layered decode launch");
    }
}

// The tensor-core prefill state in prefill mode 0, else null.
itts::TmaPrefill* tma_of(itts_gpt_ctx* c) { return c->prefill_mode == 0 && c->tma.wsplit ? &c->tma : nullptr; }

// prefix already in d_hidden
void run_prefill(itts_gpt_ctx* c, uint32_t rows) {
    itts::PrefillArgs p{&c->hw,   c->d_hidden, c->d_x,    c->d_qkv,  c->d_att,
                        c->d_r,   c->d_ff,     c->d_kv,   int(rows), c->dtype == ITTS_WEIGHTS_BF16,
                        c->db.ctl->status,     tma_of(c), c->d_att_part, c->d_att_cnt};
    ck(itts::launch_prefill_layers(p, c->stream, &c->launches), "prefill launch");
    reset_ctl(c);
    itts::DecodeArgs a = decode_args(c);
    a.head_src = c->d_hidden + size_t(rows - 1) * kW;
    ck(c->dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::launch_head(a, c->sm_count, c->stream)
                                     : itts::wf32::launch_head(a, c->sm_count, c->stream),
       "head launch");
    ++c->launches;
}

void validate_prefix(size_t n_floats) {
    if (n_floats == 0 || n_floats % kW || n_floats / kW > 1024) invalid("Invalid GPT prefill dimensions");
}

void host_prefill(itts_gpt_ctx* c, const float* prefix, size_t n_floats) {
    validate_prefix(n_floats);
    if (!prefix) invalid("prefix is null");
    const uint32_t rows = uint32_t(n_floats / kW);
    std::memcpy(c->h_stage, prefix, n_floats * 4);
    ck(cudaMemcpyAsync(c->d_hidden, c->h_stage, n_floats * 4, cudaMemcpyHostToDevice, c->stream), "prefix upload");
    run_prefill(c, rows);
    c->cached = rows;
    c->prefix_rows = rows;
    c->have_prefill = true;
}

// gpt_sampling.cpp:170-173
itts::SampleOpts configure(const itts_gen_opts& in, float* length_penalty) {
    itts_gen_opts o = in;
    if (!o.do_sample) {
        o.temperature = 1;
        o.top_k = 0;
        o.top_p = 1;
    }
    if (!std::isfinite(o.temperature) || !std::isfinite(o.top_p) || !std::isfinite(o.repetition_penalty) ||
        o.temperature <= 0 || o.top_p <= 0 || o.top_p > 1 || o.repetition_penalty <= 0)
        invalid("Invalid GPT generation parameters");
    if (!o.num_beams || o.num_beams > 10 || !std::isfinite(o.length_penalty))
        invalid("Invalid beam search configuration");
    if (o.rng != ITTS_RNG_SPLITMIX64 && o.rng != ITTS_RNG_PHILOX) invalid("Invalid random stream selector");
    if (length_penalty) *length_penalty = o.length_penalty;
    return itts::SampleOpts{o.do_sample, o.top_k, o.seed, o.temperature, o.top_p, o.repetition_penalty, o.num_beams,
                            o.rng};
}

void validate_capacity(itts_gpt_ctx* c, size_t prefix_rows, uint32_t maximum) {
    if (!maximum || maximum + 1 >= c->mel_pos_rows || prefix_rows + maximum >= kCap)
        invalid("GPT generation capacity exceeded");
}

// one cached decode step with `code` at `pos`; logits stay in db.logits
void device_step(itts_gpt_ctx* c, uint32_t code, uint32_t pos) {
    if (!c->cached || c->cached >= kCap || code >= kVocab || pos >= c->mel_pos_rows)
        invalid("GPT step requires valid cache, code and position");
    itts::DecodeArgs a = decode_args(c);
    a.mode = itts::kModeStep;
    a.n_iter = 1;
    a.s0 = c->cached;
    a.pos0 = pos;
    a.first_code = code;
    launch_decode(c, a);
    ++c->cached;
}

// ------------------------------------------------------------ KV states
itts_gpt_state* make_checkpoint(itts_gpt_ctx* c) {
    if (!c->cached) invalid("Invalid KV snapshot");
    auto s = std::make_unique<itts_gpt_state>();
    s->device = c->device;
    s->tokens = c->cached;
    s->layers = c->layers;
    s->d = dev_alloc<float>(size_t(c->layers) * 2 * kH * c->cached * kHd, "KV snapshot");
    const size_t width = size_t(c->cached) * kHd * 4;
    for (uint32_t l = 0; l < c->layers * 2; ++l)
        ck(cudaMemcpy2DAsync(s->d + size_t(l) * kH * c->cached * kHd, width,
                             c->d_kv + size_t(l) * kH * kCap * kHd, size_t(kCap) * kHd * 4, width, kH,
                             cudaMemcpyDeviceToDevice, c->stream),
           "KV snapshot copy");
    return s.release();
}

void apply_restore(itts_gpt_ctx* c, const itts_gpt_state* s) {
    if (!s || s->layers != c->layers || s->device != c->device || !s->tokens || s->tokens > kCap)
        invalid("Invalid KV restore");
    const size_t width = size_t(s->tokens) * kHd * 4;
    for (uint32_t l = 0; l < c->layers * 2; ++l)
        ck(cudaMemcpy2DAsync(c->d_kv + size_t(l) * kH * kCap * kHd, size_t(kCap) * kHd * 4,
                             s->d + size_t(l) * kH * s->tokens * kHd, width, width, kH, cudaMemcpyDeviceToDevice,
                             c->stream),
           "KV restore copy");
    c->cached = s->tokens;
}

// ------------------------------------------------------------ batched decode
// Buffers of the batched path, allocated on first use; `arenas` KV arenas.
void ensure_batch(itts_gpt_ctx* c, uint32_t arenas) {
    using namespace itts;
    if (!c->d_bact) {
        const size_t B = kMaxBatch;
        const size_t sizes[] = {B * kW * 4,                  // x
                                B * 3840 * 4,                // qkv
                                B * kW * 4,                  // attn
                                B * kW * 4,                  // hm
                                B * 5120 * 4,                // f
                                B * kBatchLogitsStride * 4,  // logits
                                B * kH * 8 * 68 * 4,         // attention partials
                                size_t(24) * B * kH * 4,     // attention arrival counters
                                sizeof(BatchState),          // step state
                                B * kSeenWords * 4,          // repetition-penalty sets
                                B * kCap * 4,                // codes
                                B * kVocab * 4,              // beam scores
                                B * 8448 * 4,                // beam log-softmax scratch
                                B * (kCap + 2) * 4};         // beam histories
        constexpr int n = int(sizeof(sizes) / sizeof(sizes[0]));
        size_t total = 0;
        for (size_t z : sizes) total += align256(z);
        c->d_bact = dev_alloc<char>(total, "batched decode buffers");
        ck(cudaMemset(c->d_bact, 0, total), "batched buffer init");
        char* r[n];
        char* p = c->d_bact;
        for (int i = 0; i < n; ++i) {
            r[i] = p;
            p += align256(sizes[i]);
        }
        BatchArgs& a = c->bargs;
        a.x = reinterpret_cast<float*>(r[0]);
        a.qkv = reinterpret_cast<float*>(r[1]);
        a.attn = reinterpret_cast<float*>(r[2]);
        a.hm = reinterpret_cast<float*>(r[3]);
        a.f = reinterpret_cast<float*>(r[4]);
        a.logits = reinterpret_cast<float*>(r[5]);
        a.part = reinterpret_cast<float*>(r[6]);
        a.head_cnt = reinterpret_cast<unsigned*>(r[7]);
        a.st = reinterpret_cast<BatchState*>(r[8]);
        a.seen = reinterpret_cast<uint32_t*>(r[9]);
        a.codes = reinterpret_cast<uint32_t*>(r[10]);
        c->d_bscores = reinterpret_cast<float*>(r[11]);
        c->d_btmp = reinterpret_cast<float*>(r[12]);
        c->d_bhist = reinterpret_cast<uint32_t*>(r[13]);
        c->d_bbig = dev_alloc<char>(B * sampler_big_bytes(), "batched sampler workspace");
        a.big = reinterpret_cast<SamplerBig*>(c->d_bbig);
        ck(cudaMallocHost(&c->h_bstate, sizeof(BatchState)), "pinned batch state");
        c->arena_floats = size_t(c->layers) * 2 * kH * kCap * kHd;
    }
    if (c->b_arenas < arenas) {
        if (c->d_bkv) cudaFree(c->d_bkv);
        c->d_bkv = nullptr;
        c->b_arenas = 0;
        c->d_bkv = dev_alloc<float>(size_t(arenas) * c->arena_floats, "batched KV arenas");
        c->b_arenas = arenas;
    }
    c->bargs.kv = c->d_bkv;
    c->bargs.arena_floats = c->arena_floats;
}

// Batch arguments for M rows (options per row; scaled_head in the generate loop).
itts::BatchArgs batch_args(itts_gpt_ctx* c, uint32_t M, const itts::SampleOpts* o, bool scaled_head) {
    itts::BatchArgs a = c->bargs;
    a.d = decode_args(c);
    a.M = M;
    for (uint32_t m = 0; m < M; ++m) a.opts[m] = o[m];
    a.scaled_head = scaled_head ? 1 : 0;
    return a;
}

// Prefill of one row into KV arena `arena`; its last-row logits go to row m
// of the batched logits.
void batch_prefill(itts_gpt_ctx* c, const float* prefix, size_t n_floats, uint32_t arena, uint32_t m) {
    validate_prefix(n_floats);
    if (!prefix) invalid("prefix is null");
    const uint32_t rows = uint32_t(n_floats / kW);
    ck(cudaMemcpyAsync(c->d_hidden, prefix, n_floats * 4, cudaMemcpyHostToDevice, c->stream), "prefix upload");
    itts::PrefillArgs p{&c->hw,
                        c->d_hidden,
                        c->d_x,
                        c->d_qkv,
                        c->d_att,
                        c->d_r,
                        c->d_ff,
                        c->d_bkv + size_t(arena) * c->arena_floats,
                        int(rows),
                        c->dtype == ITTS_WEIGHTS_BF16,
                        c->db.ctl->status,
                        tma_of(c),
                        c->d_att_part,
                        c->d_att_cnt};
    ck(itts::launch_prefill_layers(p, c->stream, &c->launches), "prefill launch");
    itts::DecodeArgs a = decode_args(c);
    a.head_src = c->d_hidden + size_t(rows - 1) * kW;
    a.b.logits = c->bargs.logits + size_t(m) * itts::kBatchLogitsStride;
    ck(c->dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::launch_head(a, c->sm_count, c->stream)
                                     : itts::wf32::launch_head(a, c->sm_count, c->stream),
       "head launch");
    ++c->launches;
}

// One forward step of the rows in the state (codes drawn at global step
// st.step - 1): the persistent kernel, or in layered mode one launch per phase.
void batch_forward(itts_gpt_ctx* c, const itts::BatchArgs& a) {
    if (c->mode == 0) {
        reset_ctl(c);  // grid-barrier counter
        ck(c->dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::launch_batch_persistent(a, 1, 0, c->sm_count, c->stream)
                                         : itts::wf32::launch_batch_persistent(a, 1, 0, c->sm_count, c->stream),
           "batched decode launch");
        ++c->launches;
        return;
    }
    ck(c->dtype == ITTS_WEIGHTS_BF16
           ? itts::wbf16::launch_batch_forward(a, int(c->layers), c->sm_count, c->stream, &c->launches)
           : itts::wf32::launch_batch_forward(a, int(c->layers), c->sm_count, c->stream, &c->launches),
       "batched forward launch");
}

// `iters` iterations of: a draw of every active row, then a forward step of
// the rows still active (persistent kernel; layered mode: one sampler launch
// and one forward launch sequence, whose kernels return at once when no row
// is active).
void batch_generate(itts_gpt_ctx* c, const itts::BatchArgs& a, uint32_t iters) {
    if (c->mode == 0) {
        reset_ctl(c);
        ck(c->dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::launch_batch_persistent(a, iters, 1, c->sm_count, c->stream)
                                         : itts::wf32::launch_batch_persistent(a, iters, 1, c->sm_count, c->stream),
           "batched decode launch");
        ++c->launches;
        return;
    }
    for (uint32_t i = 0; i < iters; ++i) {
        ck(itts::launch_batch_sample(a, c->stream), "batched sampler launch");
        ++c->launches;
        batch_forward(c, a);
    }
}

// Device-time marks of a generate call (events on the context's stream):
// 0 before the prefill(s), 1 before the token loop, 2 after it.
void mark(itts_gpt_ctx* c, int k) { ck(cudaEventRecord(c->ev[k], c->stream), "event record"); }

// After the call's final synchronisation: adds the marked intervals.
void add_timing(itts_gpt_ctx* c, uint32_t forward_steps, uint32_t rows) {
    float a = 0.f, b = 0.f;
    ck(cudaEventElapsedTime(&a, c->ev[0], c->ev[1]), "event time");
    ck(cudaEventElapsedTime(&b, c->ev[1], c->ev[2]), "event time");
    c->timing.prefill_ms += a;
    c->timing.decode_ms += b;
    c->timing.forward_steps += forward_steps;
    c->timing.rows = std::max(c->timing.rows, rows);
}

void put_state(itts_gpt_ctx* c) {
    ck(cudaMemcpyAsync(c->bargs.st, c->h_bstate, sizeof(itts::BatchState), cudaMemcpyHostToDevice, c->stream),
       "batch state upload");
}

// generate (gpt_sampling.cpp:168-189) for up to kMaxBatch greedy/sampled
// requests in lockstep: each request is prefilled into its own KV arena, then
// every step runs the sampler of every row and one batched forward step; a
// row that stops is left out of later draws.
void generate_rows(itts_gpt_ctx* c, size_t M, const float* const* prefixes, const size_t* n_floats,
                   const itts::SampleOpts* o, uint32_t max_tokens, uint32_t* codes, uint32_t* n_codes, int* stopped) {
    using namespace itts;
    ensure_batch(c, uint32_t(M));
    reset_ctl(c);
    ck(cudaMemsetAsync(c->bargs.head_cnt, 0, size_t(24) * kMaxBatch * kH * 4, c->stream), "counter reset");
    mark(c, 0);
    for (size_t m = 0; m < M; ++m) batch_prefill(c, prefixes[m], n_floats[m], uint32_t(m), uint32_t(m));
    BatchState& st = *c->h_bstate;
    std::memset(&st, 0, sizeof st);
    std::vector<uint32_t> seen(size_t(M) * kSeenWords, 0u);
    for (size_t m = 0; m < M; ++m) {
        st.s0[m] = uint32_t(n_floats[m] / kW);
        st.arena[m] = uint32_t(m);
        st.maxc[m] = max_tokens;
        for (uint32_t t : {1u, 8192u}) seen[m * kSeenWords + (t >> 5)] |= 1u << (t & 31);
    }
    st.active = (1u << M) - 1;
    put_state(c);
    ck(cudaMemcpyAsync(c->bargs.seen, seen.data(), seen.size() * 4, cudaMemcpyHostToDevice, c->stream), "seen upload");
    BatchArgs a = batch_args(c, uint32_t(M), o, true);
    a.codes_stride = max_tokens;
    mark(c, 1);
    batch_generate(c, a, max_tokens);
    mark(c, 2);
    std::vector<uint32_t> out(size_t(M) * max_tokens);
    ck(cudaMemcpyAsync(out.data(), c->bargs.codes, out.size() * 4, cudaMemcpyDeviceToHost, c->stream), "codes read");
    ck(cudaMemcpyAsync(c->h_bstate, c->bargs.st, sizeof(BatchState), cudaMemcpyDeviceToHost, c->stream),
       "batch state read");
    check_status(c);
    add_timing(c, max_tokens - 1, uint32_t(M));
    for (size_t m = 0; m < M; ++m) {
        n_codes[m] = st.n_codes[m];
        stopped[m] = int(st.stopped[m]);
        std::memcpy(codes + m * size_t(max_tokens), out.data() + m * size_t(max_tokens), size_t(st.n_codes[m]) * 4);
    }
    c->cached = 0;  // the context's own cache no longer follows a prefill
    c->have_prefill = false;
}

// Continuous batching: requests (gpt_sampling.cpp:168-189 each) decoded with
// up to R rows in flight.  The host meets the device at sync points: finished
// rows hand their codes back and the next requests are prefilled into the
// free rows (each row its own KV arena, start step and code limit); then the
// batched kernel runs until the first row reaches its limit (at most
// kServeChunk steps, so a row that ends on the stop code waits at most that
// long for a successor).
constexpr uint32_t kServeChunk = 64;

void serve_rows(itts_gpt_ctx* c, size_t n, const float* const* prefixes, const size_t* n_floats,
                const itts::SampleOpts* o, const uint32_t* max_tokens, uint32_t max_rows, uint32_t* const* codes,
                uint32_t* n_codes, int* stopped) {
    using namespace itts;
    const uint32_t R = uint32_t(std::min<size_t>({size_t(max_rows), n, size_t(kMaxBatch)}));
    ensure_batch(c, R);
    reset_ctl(c);
    ck(cudaMemsetAsync(c->bargs.head_cnt, 0, size_t(24) * kMaxBatch * kH * 4, c->stream), "counter reset");
    BatchState& st = *c->h_bstate;
    ck(cudaStreamSynchronize(c->stream), "serve start");
    std::memset(&st, 0, sizeof st);
    std::vector<long> row_req(R, -1);
    std::vector<SampleOpts> ro(kMaxBatch, o[0]);
    size_t next = 0;
    uint32_t forwards = 0;
    mark(c, 3);
    float prefill_ms = 0.f;
    cudaEvent_t e0 = c->ev[0], e1 = c->ev[1];
    for (;;) {
        // admit requests into free rows
        bool admitted = false;
        for (uint32_t m = 0; m < R && next < n; ++m) {
            if (row_req[m] >= 0) continue;
            if (!admitted) ck(cudaEventRecord(e0, c->stream), "event record");
            admitted = true;
            const size_t q = next++;
            batch_prefill(c, prefixes[q], n_floats[q], m, m);
            st.s0[m] = uint32_t(n_floats[q] / kW);
            st.arena[m] = m;
            st.base[m] = st.step;
            st.maxc[m] = max_tokens[q];
            st.n_codes[m] = 0;
            st.stopped[m] = 0;
            st.active |= 1u << m;
            ro[m] = o[q];
            uint32_t seen[kSeenWords] = {};
            for (uint32_t t : {1u, 8192u}) seen[t >> 5] |= 1u << (t & 31);
            ck(cudaMemcpyAsync(c->bargs.seen + size_t(m) * kSeenWords, seen, sizeof seen, cudaMemcpyHostToDevice,
                               c->stream),
               "seen upload");
            row_req[m] = long(q);
        }
        if (admitted) {
            ck(cudaEventRecord(e1, c->stream), "event record");
            ck(cudaEventSynchronize(e1), "prefill");
            float ms = 0.f;
            ck(cudaEventElapsedTime(&ms, e0, e1), "event time");
            prefill_ms += ms;
        }
        if (!st.active) break;
        uint32_t iters = kServeChunk;
        for (uint32_t m = 0; m < R; ++m)
            if ((st.active >> m) & 1u) iters = std::min(iters, st.maxc[m] - (st.step - st.base[m]));
        put_state(c);
        BatchArgs a = batch_args(c, R, ro.data(), true);
        a.codes_stride = kCap;
        batch_generate(c, a, iters);
        forwards += iters;
        ck(cudaMemcpyAsync(c->h_bstate, c->bargs.st, sizeof(BatchState), cudaMemcpyDeviceToHost, c->stream),
           "batch state read");
        check_status(c);
        // hand finished rows back
        for (uint32_t m = 0; m < R; ++m) {
            if (row_req[m] < 0 || ((st.active >> m) & 1u)) continue;
            const size_t q = size_t(row_req[m]);
            n_codes[q] = st.n_codes[m];
            stopped[q] = int(st.stopped[m]);
            if (st.n_codes[m])
                ck(cudaMemcpy(codes[q], c->bargs.codes + size_t(m) * kCap, size_t(st.n_codes[m]) * 4,
                              cudaMemcpyDeviceToHost),
                   "codes read");
            row_req[m] = -1;
        }
    }
    mark(c, 2);
    ck(cudaStreamSynchronize(c->stream), "serve end");
    float total = 0.f;
    ck(cudaEventElapsedTime(&total, c->ev[3], c->ev[2]), "event time");
    c->timing.prefill_ms += prefill_ms;
    c->timing.decode_ms += total - prefill_ms;
    c->timing.forward_steps += forwards;
    c->timing.rows = std::max(c->timing.rows, R);
    c->cached = 0;  // the context's own cache no longer follows a prefill
    c->have_prefill = false;
}

// ------------------------------------------------------------ beam search
// gpt_sampling.cpp:190-245 with the hypotheses decoded as the rows of one
// batched step.  Each hypothesis owns a KV arena; a child keeps its parent's
// arena when it is the parent's first surviving child, otherwise it takes an
// arena no child claimed and the parent's cached rows are copied there on
// the device.  Per step: the beam scores of every parent (float log-softmax,
// processors with num_beams > 1 semantics, + the cumulative score) on the
// device, the candidate choice and hypothesis bookkeeping of the reference on
// the host, then one batched forward step of the children.
uint64_t splitmix_draw(uint64_t seed, uint64_t n) {
    uint64_t z = seed + (n + 1) * 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}
uint64_t philox_draw(uint64_t seed, uint64_t draw) {
    uint32_t c0 = uint32_t(draw), c1 = uint32_t(draw >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = uint64_t(0xD2511F53u) * c0, p1 = uint64_t(0xCD9E8D57u) * c2;
        const uint32_t n0 = uint32_t(p1 >> 32) ^ c1 ^ k0, n1 = uint32_t(p1), n2 = uint32_t(p0 >> 32) ^ c3 ^ k1,
                       n3 = uint32_t(p0);
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return (uint64_t(c0) << 32) | c1;
}

// sample_gpt_token_from_logits (gpt_sampling.cpp:130-165) over n*8194 scores.
uint32_t sample_flat(const std::vector<float>& s, int rng, uint64_t seed, uint64_t draw) {
    float mx = -std::numeric_limits<float>::infinity();
    for (float v : s)
        if (std::isfinite(v)) mx = std::max(mx, v);
    if (!std::isfinite(mx)) fail(ITTS_ERR_RUNTIME, "GPT sampling received no finite logits");
    double total = 0.0;
    std::vector<double> probs(s.size(), 0.0);
    for (size_t i = 0; i < s.size(); ++i)
        if (std::isfinite(s[i])) {
            probs[i] = std::exp(static_cast<double>(s[i] - mx));
            total += probs[i];
        }
    if (total <= 0.0) fail(ITTS_ERR_RUNTIME, "GPT sampling probability mass is zero");
    const uint64_t u = rng == 1 ? philox_draw(seed, draw) : splitmix_draw(seed, draw);
    const double target = static_cast<double>(u >> 11) * (1.0 / 9007199254740992.0) * total;
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

std::vector<uint32_t> beam_search(itts_gpt_ctx* c, const float* prefix, size_t n_floats, const itts::SampleOpts& o,
                                  float length_penalty, uint32_t maximum, bool& eos_out) {
    using namespace itts;
    const uint32_t nb = o.num_beams;
    ensure_batch(c, nb);
    reset_ctl(c);
    ck(cudaMemsetAsync(c->bargs.head_cnt, 0, size_t(24) * kMaxBatch * kH * 4, c->stream), "counter reset");
    struct Beam {
        std::vector<uint32_t> codes;
        float score = 0;
        uint32_t arena = 0;
    };
    struct Finished {
        std::vector<uint32_t> codes;
        double score;
        bool eos;
    };
    struct Cand {
        uint32_t parent, token;
        float score;
    };
    const uint32_t rows = uint32_t(n_floats / kW);
    mark(c, 0);
    batch_prefill(c, prefix, n_floats, 0, 0);
    // every initial hypothesis starts from the prefill's logits and arena 0 (gpt_sampling.cpp:196-198)
    for (uint32_t p = 1; p < nb; ++p)
        ck(cudaMemcpyAsync(c->bargs.logits + size_t(p) * kBatchLogitsStride, c->bargs.logits, kVocab * 4,
                           cudaMemcpyDeviceToDevice, c->stream),
           "beam logits");
    std::vector<Beam> beams(nb);
    for (uint32_t i = 1; i < nb; ++i) beams[i].score = -1e9f;
    uint64_t draws = 0;
    std::vector<Finished> finished;
    auto finish = [&](const Beam& beam, float score, uint32_t length, bool eos) {
        finished.push_back({beam.codes, score / std::pow(static_cast<double>(std::max(length, 1u)), length_penalty), eos});
        std::sort(finished.begin(), finished.end(), [](const Finished& a, const Finished& b) { return a.score > b.score; });
        if (finished.size() > nb) finished.resize(nb);
    };
    const size_t hstride = kCap + 2;
    std::vector<uint32_t> hist(hstride * nb);
    std::vector<float> all;
    std::vector<SampleOpts> ro(nb, o);
    uint32_t forwards = 0;
    mark(c, 1);
    for (uint32_t si = 0; si < maximum; ++si) {
        const uint32_t np = uint32_t(beams.size());
        for (uint32_t p = 0; p < np; ++p) {
            uint32_t* h = hist.data() + p * hstride;
            h[0] = 1;
            h[1] = 8192;
            std::copy(beams[p].codes.begin(), beams[p].codes.end(), h + 2);
        }
        ck(cudaMemcpyAsync(c->d_bhist, hist.data(), size_t(np) * hstride * 4, cudaMemcpyHostToDevice, c->stream),
           "history upload");
        for (uint32_t p = 0; p < np; ++p) {
            ck(launch_beam_scores(c->bargs.logits + size_t(p) * kBatchLogitsStride, o, c->d_bhist + p * hstride,
                                  uint32_t(beams[p].codes.size() + 2), beams[p].score, c->d_btmp + size_t(p) * 8448,
                                  c->d_bscores + size_t(p) * kVocab, c->db.ctl->status, c->stream),
               "beam score launch");
            ++c->launches;
        }
        all.resize(size_t(np) * kVocab);
        ck(cudaMemcpyAsync(all.data(), c->d_bscores, all.size() * 4, cudaMemcpyDeviceToHost, c->stream),
           "beam scores read");
        check_status(c);  // synchronises: the host buffers above are free again
        std::vector<Cand> cands;
        const uint32_t take = 2 * nb;
        if (o.do_sample) {
            auto avail = all;
            for (uint32_t i = 0; i < take; ++i) {
                const uint32_t id = sample_flat(avail, o.rng, o.seed, draws++);
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
        std::vector<uint32_t> parent_of;
        for (uint32_t rank = 0; rank < cands.size(); ++rank) {
            const Cand cand = cands[rank];
            const Beam& parent = beams[cand.parent];
            if (cand.token == 8193) {
                if (rank < nb) finish(parent, cand.score, si + 1, true);
                continue;
            }
            if (cand.token >= 8192) fail(ITTS_ERR_RUNTIME, "Beam generated invalid semantic code");
            Beam child;
            child.codes = parent.codes;
            child.codes.push_back(cand.token);
            child.score = cand.score;
            next.push_back(std::move(child));
            parent_of.push_back(cand.parent);
            if (next.size() == nb) break;
        }
        if (next.empty()) break;
        if (si + 1 < maximum) {
            // a parent's first child keeps its arena; later children get a copy
            std::vector<char> claimed(nb, 0);
            std::vector<int> src(next.size(), -1);
            for (size_t i = 0; i < next.size(); ++i) {
                const uint32_t pa = beams[parent_of[i]].arena;
                if (!claimed[pa]) {
                    claimed[pa] = 1;
                    next[i].arena = pa;
                } else {
                    src[i] = int(pa);
                }
            }
            const size_t width = size_t(rows + si) * kHd * 4;  // the parent's cached rows
            for (size_t i = 0; i < next.size(); ++i) {
                if (src[i] < 0) continue;
                uint32_t dst = 0;
                while (claimed[dst]) ++dst;
                claimed[dst] = 1;
                next[i].arena = dst;
                const float* from = c->d_bkv + size_t(src[i]) * c->arena_floats;
                float* to = c->d_bkv + size_t(dst) * c->arena_floats;
                ck(cudaMemcpy2DAsync(to, size_t(kCap) * kHd * 4, from, size_t(kCap) * kHd * 4, width,
                                     size_t(c->layers) * 2 * kH, cudaMemcpyDeviceToDevice, c->stream),
                   "beam KV copy");
            }
            BatchState& st = *c->h_bstate;
            std::memset(&st, 0, sizeof st);
            for (size_t i = 0; i < next.size(); ++i) {
                st.token[i] = next[i].codes.back();
                st.s0[i] = rows;
                st.arena[i] = next[i].arena;
            }
            st.active = (1u << next.size()) - 1;
            st.step = si + 1;  // forward step si: mel position si + 2 over rows + si cached tokens
            put_state(c);
            batch_forward(c, batch_args(c, uint32_t(next.size()), ro.data(), false));
            ++forwards;
        }
        beams = std::move(next);
        if (finished.size() == nb &&
            finished.back().score >= cands[0].score / std::pow(static_cast<double>(si + 1), length_penalty)) {
            beams.clear();
            break;
        }
    }
    mark(c, 2);
    check_status(c);
    add_timing(c, forwards, nb);
    for (const auto& beam : beams) finish(beam, beam.score, uint32_t(beam.codes.size()), false);
    if (finished.empty()) fail(ITTS_ERR_RUNTIME, "Beam search produced no hypotheses");
    eos_out = finished[0].eos;
    c->cached = 0;  // the context's own cache no longer follows a prefill
    c->have_prefill = false;
    return finished[0].codes;
}

}  // namespace

namespace itts {
void set_thread_error(const std::string& msg) { g_create_error = msg; }
}  // namespace itts

// ================================================================ C-ABI
extern "C" {

void itts_gen_opts_default(itts_gen_opts* o) {
    if (!o) return;
    o->do_sample = 1;
    o->top_k = 30;
    o->seed = 20261002ull;
    o->temperature = 0.8f;
    o->top_p = 0.8f;
    o->repetition_penalty = 10.0f;
    o->num_beams = 1;
    o->length_penalty = 0.0f;
    o->rng = ITTS_RNG_SPLITMIX64;
}

const char* itts_gpt_last_error(const itts_gpt_ctx* ctx) { return ctx ? ctx->err.c_str() : g_create_error.c_str(); }

int itts_gpt_create(const char* bundle_dir, int device, int weight_dtype, itts_gpt_ctx** out) {
    g_create_error.clear();
    if (!out) {
        g_create_error = "out is null";
        return ITTS_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    std::unique_ptr<itts_gpt_ctx> c(new (std::nothrow) itts_gpt_ctx());
    if (!c) return ITTS_ERR_OUT_OF_MEMORY;
    c->device = device;
    c->dtype = weight_dtype;
    const int rc = guard(c.get(), [&] {
        if (!bundle_dir) invalid("bundle_dir is null");
        if (weight_dtype != ITTS_WEIGHTS_F32 && weight_dtype != ITTS_WEIGHTS_BF16)
            invalid("weight_dtype must be ITTS_WEIGHTS_F32 or ITTS_WEIGHTS_BF16");
        itts::Mit2Bundle bundle(bundle_dir);
        validate_bundle(c.get(), bundle);
        int n = 0;
        ck(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) invalid("device index out of range");
        ck(cudaSetDevice(device), "cudaSetDevice");
        cudaDeviceProp prop{};
        ck(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major < 10) fail(ITTS_ERR_RUNTIME, "this library is built for sm_100a (B200) devices only");
        c->sm_count = prop.multiProcessorCount;
        // the decode kernel gives each SM at most 64 rows of any matrix (mel_head: 8194)
        if ((8194 + c->sm_count - 1) / c->sm_count > 64) fail(ITTS_ERR_RUNTIME, "device has too few SMs");
        if (!prop.cooperativeLaunch) fail(ITTS_ERR_RUNTIME, "device lacks cooperative launch");
        int per_sm = 0;
        ck(itts::sampler_configure(), "sampler kernel configuration");
        ck(weight_dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::decode_configure(&per_sm)
                                             : itts::wf32::decode_configure(&per_sm),
           "decode kernel configuration");
        ck(weight_dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::batch_configure() : itts::wf32::batch_configure(),
           "batched kernel configuration");
        if (per_sm < 1) fail(ITTS_ERR_RUNTIME, "persistent decode kernel does not fit on an SM");
        ck(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream creation");
        for (cudaEvent_t& e : c->ev) ck(cudaEventCreate(&e), "event creation");
        upload_weights(c.get(), bundle);
        alloc_buffers(c.get());
        ck(itts::tma_prefill_init(&c->tma, c->hw, weight_dtype == ITTS_WEIGHTS_BF16, c->stream),
           "tensor-core prefill setup");
        ck(cudaDeviceSynchronize(), "load");
    }, /*set_device=*/false);
    if (rc != ITTS_OK) {
        g_create_error = c->err;
        return rc;
    }
    *out = c.release();
    return ITTS_OK;
}

void itts_gpt_destroy(itts_gpt_ctx* ctx) { delete ctx; }

int itts_gpt_get_info(const itts_gpt_ctx* ctx, itts_gpt_info* info) {
    if (!ctx || !info) return ITTS_ERR_INVALID_ARGUMENT;
    info->layers = ctx->layers;
    info->mel_pos_rows = ctx->mel_pos_rows;
    info->text_pos_rows = ctx->text_pos_rows;
    info->sm_count = uint32_t(ctx->sm_count);
    info->weight_bytes = ctx->weight_bytes;
    info->stream_bytes = ctx->stream_bytes;
    info->weight_dtype = ctx->dtype;
    info->device = ctx->device;
    return ITTS_OK;
}

int itts_gpt_prepare(itts_gpt_ctx* ctx, const float* speaker, size_t speaker_n, const float* emotion, size_t emotion_n,
                     const uint32_t* text, size_t text_n, uint32_t language, float* out, size_t out_floats,
                     size_t* rows) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        if (speaker_n != 192 || emotion_n != kW || language >= 107 || !speaker || !emotion)
            invalid("Invalid GPT conditioning dimensions");
        std::vector<uint32_t> ids{0};
        for (size_t i = 0; i < text_n; ++i) {
            const uint32_t id = text[i];
            if (id >= 60510) invalid("Text token is outside 2.5 vocabulary");
            if (id != 0 && id != 1) ids.push_back(id);
        }
        ids.push_back(1);
        if (ids.size() > 602 || ids.size() > ctx->text_pos_rows) invalid("Text segment exceeds GPT position capacity");
        const size_t nrows = 3 + ids.size() + 1;
        if (!out || !rows || out_floats < nrows * kW) invalid("output buffer too small");
        float* d_spk = ctx->d_misc;
        float* d_emo = d_spk + 192;
        uint32_t* d_ids = reinterpret_cast<uint32_t*>(d_emo + 1280);
        ck(cudaMemcpyAsync(d_spk, speaker, 192 * 4, cudaMemcpyHostToDevice, ctx->stream), "speaker upload");
        ck(cudaMemcpyAsync(d_emo, emotion, kW * 4, cudaMemcpyHostToDevice, ctx->stream), "emotion upload");
        ck(cudaMemcpyAsync(d_ids, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, ctx->stream), "ids upload");
        itts::PrepareArgs a{ctx->spk_w, ctx->spk_b, ctx->text_emb, ctx->text_pos, ctx->lang_emb, ctx->hw.mel_emb,
                            ctx->hw.mel_pos, d_spk, d_emo, d_ids, uint32_t(ids.size()), language, ctx->d_x};
        ck(itts::launch_prepare(a, ctx->stream), "prepare launch");
        ++ctx->launches;
        ck(cudaMemcpyAsync(ctx->h_stage, ctx->d_x, nrows * kW * 4, cudaMemcpyDeviceToHost, ctx->stream), "prefix read");
        ck(cudaStreamSynchronize(ctx->stream), "prepare");
        std::memcpy(out, ctx->h_stage, nrows * kW * 4);
        *rows = nrows;
    });
}

int itts_gpt_prefill(itts_gpt_ctx* ctx, const float* prefix, size_t n_floats, float* logits) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        host_prefill(ctx, prefix, n_floats);
        if (logits) ck(cudaMemcpyAsync(ctx->h_logits, ctx->db.logits, kVocab * 4, cudaMemcpyDeviceToHost, ctx->stream),
                       "logits read");
        check_status(ctx);
        if (logits) std::memcpy(logits, ctx->h_logits, kVocab * 4);
    });
}

int itts_gpt_step(itts_gpt_ctx* ctx, uint32_t code, uint32_t position, float* logits) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        device_step(ctx, code, position);
        if (logits) ck(cudaMemcpyAsync(ctx->h_logits, ctx->db.logits, kVocab * 4, cudaMemcpyDeviceToHost, ctx->stream),
                       "logits read");
        check_status(ctx);
        if (logits) std::memcpy(logits, ctx->h_logits, kVocab * 4);
    });
}

// One request of generate / generate_batch (gpt_sampling.cpp:168-189; beams
// :190-245); options already validated into `o`.
void generate_one(itts_gpt_ctx* ctx, const float* prefix, size_t n_floats, const itts::SampleOpts& o, float lp,
                  uint32_t max_tokens, uint32_t* codes, uint32_t* n_codes, int* stopped) {
    if (o.num_beams > 1) {
        bool eos = false;
        auto r = beam_search(ctx, prefix, n_floats, o, lp, max_tokens, eos);
        std::memcpy(codes, r.data(), r.size() * 4);
        *n_codes = uint32_t(r.size());
        *stopped = eos ? 1 : 0;
        return;
    }
    mark(ctx, 0);
    host_prefill(ctx, prefix, n_floats);
    itts::DecodeArgs a = decode_args(ctx);
    a.mode = itts::kModeGenerate;
    a.n_iter = max_tokens;
    a.s0 = ctx->cached;
    a.pos0 = 2;  // first generated code sits at mel position 2 (gpt_sampling.cpp:184-186)
    a.opts = o;
    mark(ctx, 1);
    launch_decode(ctx, a);
    mark(ctx, 2);
    ck(cudaMemcpyAsync(ctx->h_codes, ctx->d_codes, size_t(max_tokens) * 4, cudaMemcpyDeviceToHost, ctx->stream),
       "codes read");
    check_status(ctx);
    const itts::DecodeCtl& ctl = *ctx->h_ctl;
    add_timing(ctx, ctl.info[3], 1);
    ctx->cached += ctl.info[3];
    *n_codes = ctl.info[0];
    *stopped = int(ctl.info[1]);
    std::memcpy(codes, ctx->h_codes, size_t(ctl.info[0]) * 4);
}

int itts_gpt_generate(itts_gpt_ctx* ctx, const float* prefix, size_t n_floats, const itts_gen_opts* opts,
                      uint32_t max_tokens, uint32_t* codes, uint32_t* n_codes, int* stopped) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        if (!opts || !codes || !n_codes || !stopped) invalid("null output or options");
        validate_capacity(ctx, n_floats / kW, max_tokens);
        float lp = 0;
        const itts::SampleOpts o = configure(*opts, &lp);
        ctx->timing = itts_gpt_timing{};
        generate_one(ctx, prefix, n_floats, o, lp, max_tokens, codes, n_codes, stopped);
    });
}

int itts_gpt_generate_batch(itts_gpt_ctx* ctx, size_t batch, const float* const* prefixes, const size_t* n_floats,
                            const itts_gen_opts* opts, uint32_t max_tokens, uint32_t* codes, uint32_t* n_codes,
                            int* stopped) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        if (batch == 0) return;
        if (!prefixes || !n_floats || !opts || !codes || !n_codes || !stopped) invalid("null batch argument");
        std::vector<itts::SampleOpts> o(batch);
        std::vector<float> lp(batch, 0.f);
        for (size_t i = 0; i < batch; ++i) {  // every request is checked before any runs
            if (!prefixes[i]) invalid("null prefix in batch");
            validate_capacity(ctx, n_floats[i] / kW, max_tokens);
            o[i] = configure(opts[i], &lp[i]);
        }
        ctx->timing = itts_gpt_timing{};
        // beam requests run one at a time; the others decode in lockstep,
        // up to kMaxBatch rows per batched launch sequence
        std::vector<size_t> rows;
        for (size_t i = 0; i < batch; ++i) {
            if (o[i].num_beams > 1)
                generate_one(ctx, prefixes[i], n_floats[i], o[i], lp[i], max_tokens, codes + i * size_t(max_tokens),
                             n_codes + i, stopped + i);
            else
                rows.push_back(i);
        }
        if (rows.size() == 1) {
            const size_t i = rows[0];
            generate_one(ctx, prefixes[i], n_floats[i], o[i], lp[i], max_tokens, codes + i * size_t(max_tokens),
                         n_codes + i, stopped + i);
            return;
        }
        for (size_t b0 = 0; b0 < rows.size(); b0 += itts::kMaxBatch) {
            const size_t M = std::min<size_t>(itts::kMaxBatch, rows.size() - b0);
            std::vector<const float*> pp(M);
            std::vector<size_t> nf(M);
            std::vector<itts::SampleOpts> oo(M);
            std::vector<uint32_t> cc(M * size_t(max_tokens)), nc(M);
            std::vector<int> sp(M);
            for (size_t k = 0; k < M; ++k) {
                pp[k] = prefixes[rows[b0 + k]];
                nf[k] = n_floats[rows[b0 + k]];
                oo[k] = o[rows[b0 + k]];
            }
            generate_rows(ctx, M, pp.data(), nf.data(), oo.data(), max_tokens, cc.data(), nc.data(), sp.data());
            for (size_t k = 0; k < M; ++k) {
                const size_t i = rows[b0 + k];
                n_codes[i] = nc[k];
                stopped[i] = sp[k];
                std::memcpy(codes + i * size_t(max_tokens), cc.data() + k * size_t(max_tokens), size_t(nc[k]) * 4);
            }
        }
    });
}

int itts_gpt_serve(itts_gpt_ctx* ctx, size_t n, const float* const* prefixes, const size_t* n_floats,
                   const itts_gen_opts* opts, const uint32_t* max_tokens, uint32_t max_rows, uint32_t* const* codes,
                   uint32_t* n_codes, int* stopped) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        if (n == 0) return;
        if (!prefixes || !n_floats || !opts || !max_tokens || !codes || !n_codes || !stopped)
            invalid("null serve argument");
        if (max_rows == 0) invalid("max_rows must be at least 1");
        std::vector<itts::SampleOpts> o(n);
        for (size_t i = 0; i < n; ++i) {  // every request is checked before any runs
            if (!prefixes[i] || !codes[i]) invalid("null prefix or code buffer in serve");
            validate_prefix(n_floats[i]);
            validate_capacity(ctx, n_floats[i] / kW, max_tokens[i]);
            o[i] = configure(opts[i], nullptr);
            if (o[i].num_beams > 1) invalid("serve decodes requests without beams");
        }
        ctx->timing = itts_gpt_timing{};
        serve_rows(ctx, n, prefixes, n_floats, o.data(), max_tokens, max_rows, codes, n_codes, stopped);
    });
}

int itts_gpt_checkpoint(itts_gpt_ctx* ctx, itts_gpt_state** out) {
    if (!ctx || !out) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        *out = make_checkpoint(ctx);
        ck(cudaStreamSynchronize(ctx->stream), "snapshot");
    });
}

int itts_gpt_restore(itts_gpt_ctx* ctx, const itts_gpt_state* state) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        apply_restore(ctx, state);
        ck(cudaStreamSynchronize(ctx->stream), "restore");
    });
}

void itts_gpt_state_free(itts_gpt_state* state) { delete state; }

uint32_t itts_gpt_cached_tokens(const itts_gpt_ctx* ctx) { return ctx ? ctx->cached : 0; }

int itts_gpt_apply_processors(itts_gpt_ctx* ctx, const float* logits, size_t n, const uint32_t* history,
                              size_t history_n, const itts_gen_opts* opts, float* out) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        if (!logits || !out || !opts || (history_n && !history)) invalid("null argument");
        if (n != kVocab) invalid("logits must have 8194 entries");
        // gpt_sampling.cpp:33-71 error checks
        if (opts->repetition_penalty != 1.0f && opts->repetition_penalty <= 0.0f)
            fail(ITTS_ERR_RUNTIME, "GPT repetition penalty must be positive");
        if (opts->temperature <= 0.0f) fail(ITTS_ERR_RUNTIME, "GPT sampling temperature must be positive");
        if (opts->top_p < 1.0f && opts->top_p <= 0.0f) fail(ITTS_ERR_RUNTIME, "GPT top_p must be in (0, 1]");
        if (ctx->d_hist_cap < std::max<size_t>(history_n, 1)) {
            if (ctx->d_hist) cudaFree(ctx->d_hist);
            ctx->d_hist = nullptr;
            ctx->d_hist_cap = std::max<size_t>(history_n, 4096);
            ctx->d_hist = dev_alloc<uint32_t>(ctx->d_hist_cap * 11, "history buffer");
        }
        float* d_in = ctx->d_misc + 192 + 1280 + 1024;
        float* d_out = d_in + 8448;
        std::memcpy(ctx->h_logits, logits, kVocab * 4);
        ck(cudaMemcpyAsync(d_in, ctx->h_logits, kVocab * 4, cudaMemcpyHostToDevice, ctx->stream), "logits upload");
        if (history_n)
            ck(cudaMemcpyAsync(ctx->d_hist, history, history_n * 4, cudaMemcpyHostToDevice, ctx->stream),
               "history upload");
        const itts::SampleOpts o{opts->do_sample, opts->top_k, opts->seed, opts->temperature, opts->top_p,
                                 opts->repetition_penalty, opts->num_beams, opts->rng};
        reset_ctl(ctx);
        ck(itts::launch_processors(d_in, o, ctx->d_hist, uint32_t(history_n), d_out, ctx->db.ctl->status, ctx->stream),
           "processors launch");
        ++ctx->launches;
        ck(cudaMemcpyAsync(ctx->h_logits + 8448, d_out, kVocab * 4, cudaMemcpyDeviceToHost, ctx->stream), "scores read");
        check_status(ctx);
        std::memcpy(out, ctx->h_logits + 8448, kVocab * 4);
    });
}

int itts_gpt_stream(itts_gpt_ctx* ctx, void** cuda_stream) {
    if (!ctx || !cuda_stream) return ITTS_ERR_INVALID_ARGUMENT;
    *cuda_stream = ctx->stream;
    return ITTS_OK;
}

int itts_gpt_prefill_async(itts_gpt_ctx* ctx, const float* d_prefix, uint32_t rows, float* d_logits) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        validate_prefix(size_t(rows) * kW);
        if (!d_prefix) invalid("prefix is null");
        ck(cudaMemcpyAsync(ctx->d_hidden, d_prefix, size_t(rows) * kW * 4, cudaMemcpyDeviceToDevice, ctx->stream),
           "prefix copy");
        run_prefill(ctx, rows);
        if (d_logits)
            ck(cudaMemcpyAsync(d_logits, ctx->db.logits, kVocab * 4, cudaMemcpyDeviceToDevice, ctx->stream),
               "logits copy");
        ctx->cached = rows;
        ctx->prefix_rows = rows;
        ctx->have_prefill = true;
    });
}

int itts_gpt_decode_async(itts_gpt_ctx* ctx, const itts_gen_opts* opts, uint32_t max_tokens, uint32_t* d_codes,
                          uint32_t* d_info) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        if (!opts || !d_codes || !d_info) invalid("null output or options");
        if (!ctx->have_prefill || ctx->cached != ctx->prefix_rows)
            fail(ITTS_ERR_LOGIC, "decode_async must directly follow a prefill");
        validate_capacity(ctx, ctx->prefix_rows, max_tokens);
        const itts::SampleOpts o = configure(*opts, nullptr);
        if (o.num_beams > 1) invalid("decode_async supports num_beams == 1");
        itts::DecodeArgs a = decode_args(ctx);
        a.mode = itts::kModeGenerate;
        a.n_iter = max_tokens;
        a.s0 = ctx->cached;
        a.pos0 = 2;
        a.opts = o;
        a.codes = d_codes;
        a.info_out = d_info;
        launch_decode(ctx, a);
        ctx->have_prefill = false;
        ctx->pending = true;
        ctx->pending_info = d_info;
    });
}

int itts_gpt_sync(itts_gpt_ctx* ctx) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        if (ctx->pending)
            finish_pending(ctx);
        else
            check_status(ctx);
    });
}

int itts_gpt_set_decode_mode(itts_gpt_ctx* ctx, int mode) {
    if (!ctx || (mode != 0 && mode != 1)) return ITTS_ERR_INVALID_ARGUMENT;
    ctx->mode = mode;
    return ITTS_OK;
}

int itts_gpt_set_prefill_mode(itts_gpt_ctx* ctx, int mode) {
    if (!ctx || (mode != 0 && mode != 1)) return ITTS_ERR_INVALID_ARGUMENT;
    ctx->prefill_mode = mode;
    return ITTS_OK;
}

uint64_t itts_gpt_launch_count(const itts_gpt_ctx* ctx) { return ctx ? ctx->launches : 0; }

int itts_gpt_last_timing(const itts_gpt_ctx* ctx, itts_gpt_timing* out) {
    if (!ctx || !out) return ITTS_ERR_INVALID_ARGUMENT;
    *out = ctx->timing;
    return ITTS_OK;
}

int itts_gpt_set_wait_limit(itts_gpt_ctx* ctx, uint64_t ns) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    ctx->wait_ns = ns;
    return ITTS_OK;
}

int itts_gpt_wait_probe(itts_gpt_ctx* ctx) {
    if (!ctx) return ITTS_ERR_INVALID_ARGUMENT;
    return guard(ctx, [&] {
        finish_pending(ctx);
        reset_ctl(ctx);
        ck(cudaMemsetAsync(ctx->db.qkv, 0, ctx->tagged_bytes, ctx->stream), "hand-off reset");
        const itts::DecodeArgs a = decode_args(ctx);
        ck(ctx->dtype == ITTS_WEIGHTS_BF16 ? itts::wbf16::launch_wait_probe(a, ctx->sm_count, ctx->stream)
                                           : itts::wf32::launch_wait_probe(a, ctx->sm_count, ctx->stream),
           "wait probe launch");
        ++ctx->launches;
        check_status(ctx);
    });
}

}  // extern "C"
