// Device-side model description and kernel arguments of the B200 GPT decoder.
// Plain structs shared by the host runtime (itts_gpt.cpp) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace itts {

// Device status word (int32[4]): {code, where, cta, detail}.  Written once by
// the first failing CTA (atomicCAS on code) and read by the host after a sync.
enum DeviceStatus : int {
    kStatusOk = 0,
    kStatusBarrierTimeout = 1,   // a grid barrier wait exceeded its time limit
    kStatusInvalidCode = 2,      // sampled code 8192 (gpt_sampling.cpp:182)
    kStatusNoFiniteLogits = 3,   // sampling/top-p saw no finite score
    kStatusZeroMass = 4,         // probability mass was zero
    kStatusRingTimeout = 5,      // a weight-ring slot did not arrive in time
};


// One transformer block.  Matrices are row-major [out, in] fp32 (the Conv1D
// [in, out] tensors of the bundle are transposed once on the device at load,
// the transpose the reference caches on the CPU in gpt.cpp:24-33).
struct LayerW {
    const float *ln1_g, *ln1_b;
    const float *w_qkv, *b_qkv;  // [3840, 1280]
    const float *w_o, *b_o;      // [1280, 1280]
    const float *ln2_g, *ln2_b;
    const float *w_fc, *b_fc;    // [5120, 1280]
    const float *w_mp, *b_mp;    // [1280, 5120]
};

struct ModelW {
    LayerW layer[24];
    int layers;
    const float *lnf_g, *lnf_b;  // gpt.gpt.ln_f
    const float *fn_g, *fn_b;    // gpt.final_norm
    const float *w_head, *b_head;  // gpt.mel_head [8194, 1280] (nn.Linear layout)
    const float *mel_emb, *mel_pos;
};

// Sampling options after GenerationOptions validation (gpt_sampling.cpp:168-173).
struct SampleOpts {
    int do_sample;
    uint32_t top_k;
    uint64_t seed;
    float temperature;
    float top_p;
    float rp;  // repetition penalty
    uint32_t num_beams;
    int rng;   // 0 SplitMix64, 1 Philox4x32-10
};

// Small control block, zeroed before every decode launch.
struct DecodeCtl {
    int status[4];       // {code, where, cta, detail}
    uint32_t info[4];    // {n_codes, stopped, status, forward_steps}
    unsigned bar;        // grid-barrier arrival counter (monotonic per launch)
    unsigned head_cnt[24][20];  // split-K attention arrivals per (layer, head); the last resets it
    unsigned f_cnt[24];         // CTAs that published their GELU outputs, per layer (all steps)
    uint32_t token;      // current code (layered mode)
    int done;            // layered mode: loop finished
    unsigned pad[5];
};

struct SamplerBig;

// Decode-time device buffers (activations live in L2; KV cache in HBM).
struct DecodeBuffers {
    float* kv;        // [layer][K|V][head][4096][64] fp32
    // Activations handed between CTAs as tagged words: (epoch << 32) | float
    // bits, written once per layer; a reader polls until every word it needs
    // carries the epoch of the layer it wants (zeroed before each launch).
    unsigned long long* qkv;   // [3840]
    unsigned long long* h;     // [1280] residual stream leaving a layer
    unsigned long long* hm;    // [1280] residual stream after the attention block
    unsigned long long* attn;  // [1280] merged attention output
    float* f;                  // [5120] GELU(c_fc), published by DecodeCtl::f_cnt
    float* logits;    // [8194]
    float* part;      // split-K attention partials [20 * 256 * 68]
    SamplerBig* sampler_big;  // one large-survivor workspace per CTA
    DecodeCtl* ctl;
};

enum DecodeMode : int { kModeStep = 0, kModeGenerate = 1 };

struct DecodeArgs {
    const ModelW* w;  // device copy
    DecodeBuffers b;
    int mode;
    uint32_t n_iter;      // kModeStep: 1; kModeGenerate: max_tokens
    uint32_t s0;          // cached tokens before the first forward step
    uint32_t pos0;        // mel position of the first forward step
    uint32_t first_code;  // kModeStep: the input code
    SampleOpts opts;
    const uint32_t* history;  // initial repetition-penalty history ({1, 8192})
    uint32_t history_n;
    uint32_t* codes;      // kModeGenerate output [n_iter]
    uint32_t* info_out;   // optional copy of ctl->info (may be null)
    const float* head_src;  // prefill: last hidden row fed to the head phase
    unsigned long long wait_ns;  // time limit of every device-side wait; 0: the default (2 s)
};

// ---- batched decode (M rows per step) ------------------------------------
// Up to kMaxBatch independent rows (requests or beam hypotheses) advance one
// token per step together; each weight byte is read once per step for all
// rows.  Per-row arithmetic is that of the batch-1 kernels, so every row's
// logits are bit-identical to a batch-1 decode of the same row.
constexpr int kMaxBatch = 16;

// Device-resident per-step state of a batched decode (read by every kernel of
// a step, advanced by the sampler kernel), so one launch sequence serves every
// step.
struct BatchState {
    uint32_t token[kMaxBatch];    // code each row feeds to the next forward step
    uint32_t s0[kMaxBatch];       // cached tokens of the row before its first forward step
    uint32_t arena[kMaxBatch];    // KV arena of the row
    uint32_t n_codes[kMaxBatch];  // codes generated so far
    uint32_t stopped[kMaxBatch];  // 1 when the stop code ended the row
    uint32_t base[kMaxBatch];     // global step of the row's draw 0 (rows join at different steps)
    uint32_t maxc[kMaxBatch];     // codes the row may generate
    uint32_t active;              // bit m: row m still decodes
    uint32_t step;                // global index of the next draw; a row's draw i is step base + i
    uint32_t sample_arrivals;     // sampler CTAs that finished the current draw (layered mode)
    uint32_t pad[5];
};
// A row's draw i feeds its code to forward step i: mel position 2 + i over
// s0 + i cached tokens (gpt_sampling.cpp:184-186).

struct BatchArgs {
    DecodeArgs d;      // weight table, status word, wait limit (ring and waits of the shared code)
    uint32_t M;        // rows (1..kMaxBatch)
    float* x;          // [kMaxBatch][1280] residual stream entering / leaving a layer
    float* qkv;        // [kMaxBatch][3840]
    float* attn;       // [kMaxBatch][1280]
    float* hm;         // [kMaxBatch][1280]
    float* f;          // [kMaxBatch][5120]
    float* logits;     // [kMaxBatch][8448]
    float* part;       // [kMaxBatch][20][8][68] split-K attention partials
    unsigned* head_cnt;  // [24][kMaxBatch][20] attention arrivals (the last arriver resets)
    float* kv;         // arena 0; arena a starts at kv + a * arena_floats
    size_t arena_floats;
    BatchState* st;
    uint32_t* codes;   // generate: code i of row m at codes[m * codes_stride + i]
    uint32_t codes_stride;
    uint32_t* seen;    // [kMaxBatch][257] repetition-penalty sets
    SamplerBig* big;   // [kMaxBatch] sampler workspaces
    SampleOpts opts[kMaxBatch];
    int scaled_head;   // head applies repetition penalty and temperature (generate loop)
};
constexpr size_t kBatchLogitsStride = 8448;
constexpr int kSeenWords = 257;  // ceil(8194 / 32)

// ---- host-side launchers ----------------------------------------------------
// decode_body.cuh, once per weight type: wf32 (decode.cu), wbf16 (decode_bf16.cu)
#define ITTS_DECLARE_DECODE_LAUNCHERS(NS)                                                                      \
    namespace NS {                                                                                             \
    size_t decode_smem_bytes();                                                                                \
    cudaError_t decode_configure(int* blocks_per_sm);                                                          \
    cudaError_t launch_decode_persistent(const DecodeArgs& a, int ncta, cudaStream_t s);                       \
    cudaError_t launch_decode_layered(const DecodeArgs& a, int layers, int ncta, cudaStream_t s,               \
                                      uint64_t* launches);                                                     \
    cudaError_t launch_head(const DecodeArgs& a, int ncta, cudaStream_t s);                                    \
    cudaError_t launch_wait_probe(const DecodeArgs& a, int ncta, cudaStream_t s);                              \
    cudaError_t batch_configure();                                                                             \
    cudaError_t launch_batch_forward(const BatchArgs& a, int layers, int ncta, cudaStream_t s,                 \
                                     uint64_t* launches);                                                      \
    cudaError_t launch_batch_persistent(const BatchArgs& a, uint32_t iters, int sample, int ncta,              \
                                        cudaStream_t s);                                                       \
    }
ITTS_DECLARE_DECODE_LAUNCHERS(wf32)
ITTS_DECLARE_DECODE_LAUNCHERS(wbf16)
#undef ITTS_DECLARE_DECODE_LAUNCHERS

// sampler_kernels.cu
size_t sampler_big_bytes();
size_t sampler_dyn_smem_bytes();
cudaError_t sampler_configure();
cudaError_t launch_layer_sample(const DecodeArgs& a, uint32_t i, cudaStream_t s);
cudaError_t launch_layer_finish(const DecodeArgs& a, cudaStream_t s);
cudaError_t launch_processors(const float* logits, const SampleOpts& o, const uint32_t* hist, uint32_t hist_n,
                              float* out, int* status, cudaStream_t s);
cudaError_t launch_batch_sample(const BatchArgs& a, cudaStream_t s);
cudaError_t launch_beam_scores(const float* logits, const SampleOpts& o, const uint32_t* hist, uint32_t hist_n,
                               float beam_score, float* tmp, float* out, int* status, cudaStream_t s);

// Tensor-core prefill (gemm_tma.cu).  Every GEMM operand is held as two
// TF32-exact fp32 arrays, hi = x rounded to TF32 and lo = (x - hi) rounded to
// TF32: the weights split once when the context is created (bf16 weights are
// exact in TF32: hi is the widened matrix, lo a zero matrix), the activations
// by the kernel that produces them.  `maps` holds the
// TMA tensor maps of the split weights (host memory, encoded once).
enum TmaMatrix : int { kMatQkv = 0, kMatO = 1, kMatFc = 2, kMatMp = 3 };
struct TmaPrefill {
    static constexpr int kCounters = 320;  // output tiles of the largest GEMM (c_fc, 1024 rows)
    float* wsplit = nullptr;  // device: per layer and matrix, hi [N][K] then lo [N][K]
    float *x_hi = nullptr, *x_lo = nullptr;      // [1024, 1280] LayerNorm output
    float *att_hi = nullptr, *att_lo = nullptr;  // [1024, 1280] attention output
    float *ff_hi = nullptr, *ff_lo = nullptr;    // [1024, 5120] GELU(c_fc) output
    float* ws = nullptr;                         // split-K partial tiles
    int* counters = nullptr;                     // split-K arrival counter per output tile
    void* maps = nullptr;                        // host: CUtensorMap [layers][4][hi, lo]
    int layers = 0;
    int act_rows = -1;                           // rows the activation maps were encoded for
    alignas(64) unsigned char act_maps[6][128];  // x, att, ff (hi, lo) tensor maps for act_rows (64-byte aligned)
};
cudaError_t tma_prefill_init(TmaPrefill* p, const ModelW& hw, bool wbf16, cudaStream_t s);

// The same GEMM for other models (gemm_tma.cu): C = epi(A W^T + bias), A
// [M][K] and W [N][K] each given by the tensor maps of its TF32 hi and lo
// arrays (tma_make_map; split with tma_split).  N % 128 == 0, K % 32 == 0.
enum TmaEpi : int {
    TmaEpiBias = 0,    // C = A W^T + bias (bias may be null)
    TmaEpiGelu = 1,    // GELU (GPT-2 tanh form); with C_lo the output is split hi / lo
    TmaEpiResid = 2,   // C = R + A W^T + bias
    TmaEpiSwiGLU = 3,  // W rows interleave gate / up: C, C_lo [M][N/2] = split(silu(gate) * up)
    TmaEpiGeluErf = 4,     // GELU (erf form of the codec); with C_lo the output is split hi / lo
    TmaEpiScaleResid = 5,  // C = R + (A W^T + bias) * gamma (layer scale + residual)
};
struct TmaMap {
    alignas(64) unsigned char bytes[128];
};
struct TmaGemm {
    const TmaMap* a;  // [2]: A hi, A lo
    const TmaMap* w;  // [2]: W hi, W lo
    const float* bias;
    const float* R;
    float* C;
    float* C_lo;
    int M, N, K, epi;
    float* ws;         // tma_workspace_floats() floats
    int* counters;     // >= output tiles, zeroed
    int counters_n;
    int* status;
    const float* gamma = nullptr;  // [N] layer scale (TmaEpiScaleResid)
};
cudaError_t tma_make_map(TmaMap* m, const float* base, uint64_t rows, uint64_t cols);
cudaError_t tma_split(const float* src, float* hi, float* lo, size_t n, cudaStream_t s);
size_t tma_workspace_floats();
cudaError_t tma_gemm(const TmaGemm& g, cudaStream_t s);
void tma_prefill_free(TmaPrefill* p);

struct PrefillArgs {
    const ModelW* hw;  // host copy (pointers to device memory)
    float* hidden;     // [T, 1280] in: prefix, out: last hidden state
    float* x;          // [T, 1280]
    float* qkv;        // [T, 3840]
    float* att;        // [T, 1280]
    float* r;          // [T, 1280]
    float* ff;         // [T, 5120]
    float* kv;
    int T;
    bool wbf16;   // matrices stored bf16
    int* status;  // device status word (bounded waits of the tensor-core GEMM)
    TmaPrefill* tma;  // the TMA-fed tensor-core GEMM; null: CUDA-core tiles
    float* att_part;  // attention key-chunk partials [kHeads][kAttMaxBlocks][kAttMaxChunks][64][kAttPartLd]
    int* att_cnt;     // chunk arrivals per (head, query block) [kHeads * kAttMaxBlocks], zero between launches
};
// Prefill attention split: 64-query blocks, key chunks of kAttChunk keys.
constexpr int kAttChunk = 128;
constexpr int kAttMaxBlocks = 16;  // 1024 prefix rows
constexpr int kAttMaxChunks = kAttMaxBlocks * 64 / kAttChunk;
constexpr int kAttPartLd = 68;
constexpr size_t kAttPartFloats = size_t(20) * kAttMaxBlocks * kAttMaxChunks * 64 * kAttPartLd;
constexpr int kAttCounters = 20 * kAttMaxBlocks;
cudaError_t launch_prefill_layers(const PrefillArgs& p, cudaStream_t s, uint64_t* launches);

cudaError_t launch_transpose(const float* in, float* out, int rows_in, int cols_in, cudaStream_t s);
cudaError_t launch_transpose_bf16(const float* in, void* out, int rows_in, int cols_in, cudaStream_t s);
cudaError_t launch_to_bf16(const float* in, void* out, size_t n, cudaStream_t s);
struct PrepareArgs {
    const float *spk_w, *spk_b, *text_emb, *text_pos, *lang_emb, *mel_emb, *mel_pos;
    const float *speaker, *emotion;
    const uint32_t* ids;
    uint32_t n_ids, language;
    float* out;  // [(3 + n_ids + 1), 1280]
};
cudaError_t launch_prepare(const PrepareArgs& a, cudaStream_t s);

}  // namespace itts
