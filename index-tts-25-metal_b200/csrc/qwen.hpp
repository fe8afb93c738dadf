// Qwen3-0.6B decoder on B200 (src/qwen.cpp): device-side weights, state and
// launchers shared by the kernels (qwen.cu) and the host runtime
// (itts_qwen.cpp).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "model.hpp"

namespace itts {
namespace qwen {

constexpr int kLayers = 28;
constexpr int kDim = 1024;       // hidden width
constexpr int kQDim = 2048;      // 16 query heads x 128
constexpr int kKvDim = 1024;     // 8 key / value heads x 128
constexpr int kQkv = kQDim + 2 * kKvDim;
constexpr int kHeadDim = 128;
constexpr int kQHeads = 16;
constexpr int kKvHeads = 8;
constexpr int kFfn = 3072;
constexpr int kVocab = 151936;
constexpr uint32_t kEos = 151643;
constexpr int kCap = 4096;       // KV capacity (gptKvCacheCreate(28, 4096, 1024))
constexpr int kMaxPrompt = 3072;
constexpr int kMaxGenerate = 1024;
constexpr float kEps = 1e-6f;
constexpr int kAttnChunk = 64;   // keys per decode-attention partial
constexpr int kMaxChunks = kCap / kAttnChunk;
constexpr int kPartStride = 2 + kHeadDim;  // max, sum, 128 outputs
constexpr int kGemvRows = 8;     // rows per CTA of the decode GEMVs (one per warp)
constexpr int kHeadCtas = kVocab / kGemvRows;

struct LayerW {
    const float *ln1, *ln2, *qn, *kn;
    const float* w_qkv;   // [4096][1024]: q rows, then k, then v
    const float* w_o;     // [1024][2048]
    const float* w_gu;    // [6144][1024]: row 2r = gate_r, 2r + 1 = up_r
    const float* w_down;  // [1024][3072]
};
struct Weights {
    LayerW layer[kLayers];
    const float* embed;  // [151936][1024], also the head (tied)
    const float* norm;   // [1024]
};

// Device-resident decode state, advanced by the argmax kernel of every step.
struct State {
    uint32_t token;   // input of the next step: the last selected id
    uint32_t pos;     // its position (cached tokens before it)
    uint32_t done;    // EOS selected or the step budget spent: later kernels return at once
    uint32_t n_out;   // ids selected so far (out[0 .. n_out))
    uint32_t max_out; // ids the run may select
    uint32_t pad[3];
};

// Scratch of one context (device pointers).
struct Buffers {
    float* hidden;   // [kMaxPrompt][1024] residual stream
    float* qkv;      // [kMaxPrompt][4096]
    float *x_hi, *x_lo;    // [kMaxPrompt][1024] RMSNorm output, split
    float *att_hi, *att_lo;  // [kMaxPrompt][2048] attention output, split (decode: att_hi plain)
    float *gu_hi, *gu_lo;    // [kMaxPrompt][3072] silu(gate) * up, split (decode: gu_hi plain)
    float* part;     // decode attention partials [16][kMaxChunks][kPartStride]
    float* logits;   // [151936]
    float* best;     // per-CTA (value, index) of the head GEMV [kHeadCtas][2]
    float* kv;       // [layer][K | V][4096][1024]
    uint32_t* ids;   // [kMaxPrompt] prompt ids
    uint32_t* out;   // [kMaxGenerate] selected ids
    State* st;
    int* cnt;        // arrival counters: [0, 8) attention per KV head, [8] head GEMV (the last arriver resets)
    int* status;
};

cudaError_t init_tables();
cudaError_t prepare_kernels();  // shared-memory attributes of the attention kernels (per device)
cudaError_t launch_embed(const Weights& w, const Buffers& b, int T, cudaStream_t s);
cudaError_t launch_rmsnorm_split(const float* x, const float* g, float* hi, float* lo, int T, cudaStream_t s);
cudaError_t launch_qk_norm_rope(const LayerW& L, const Buffers& b, int layer, int T, bool decode, cudaStream_t s);
cudaError_t launch_attn_prefill(const Buffers& b, int layer, int T, cudaStream_t s);
cudaError_t launch_decode_layer(const LayerW& L, const Buffers& b, int layer, cudaStream_t s);
cudaError_t launch_head(const Weights& w, const Buffers& b, const float* last_row, bool decode, cudaStream_t s);
cudaError_t launch_decode_embed(const Weights& w, const Buffers& b, cudaStream_t s);
cudaError_t launch_interleave_rows(const float* a, const float* b, float* out, int rows, int cols, cudaStream_t s);

}  // namespace qwen
}  // namespace itts
