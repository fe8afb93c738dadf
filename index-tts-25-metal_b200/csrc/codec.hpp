// Device-side description of the IndexTTS 2.5 semantic codec's decoder
// (weights in device memory, scratch buffers) shared by codec.cu and the host
// runtime itts_codec.cpp.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "model.hpp"

namespace itts {

struct CodecBlockW {  // codec.decoder.0.convnext.i
    const float *dw_w, *dw_b;    // depthwise conv [384, 1, 7]
    const float *ln_g, *ln_b;    // LayerNorm 384, eps 1e-6
    const float *pw1_w, *pw1_b;  // [2048, 384]
    const float *pw2_w, *pw2_b;  // [384, 2048]
    const float* gamma;          // [384] layer scale
};

struct CodecWeights {
    const float* codebook;        // [8192, 8]
    const float *out_w, *out_b;   // quantizer out_project [1024, 8]
    const float *embed_w, *embed_b;  // decoder embed conv [384, 1024, 7]
    const float *norm_g, *norm_b;
    CodecBlockW block[12];
    const float *final_g, *final_b;
    const float *head_w, *head_b;  // codec.decoder.1 [1024, 384]
    const float *up_w, *up_b;      // codec.up [1024, 1024, 3]
};

struct CodecScratch {  // sized for the largest T decoded so far
    float* hidden;  // [T, 1024]
    float* h;       // [T, 384]
    float* x;       // [T, 384]
    float* u;       // [T, 2048]
};

// The tensor-core GEMMs of the decode (gemm_tma.cu): the 27 weight matrices
// split into TF32 hi / lo once, their tensor maps, the split activations that
// feed them and the stream-K workspace.  The convolutions' A operands are
// written out as im2col rows (K order c * k + j, the weights' [out][in][k]).
struct CodecTc {
    float* wsplit = nullptr;  // hi, lo of every matrix
    TmaMap w_embed[2], w_pw1[12][2], w_pw2[12][2], w_head[2], w_up[2];
    float* act = nullptr;     // activation block for act_cap rows (see codec_tc_rows)
    int act_cap = 0, rows = -1;
    float *col_e[2], *ln[2], *u[2], *col_u[2];  // hi, lo: [T][7168], [T][384], [T][2048], [2T][3072]
    TmaMap a_col_e[2], a_ln[2], a_u[2], a_col_u[2];
    float* ws = nullptr;      // stream-K partial tiles
    int* counters = nullptr;  // kCodecCounters per-tile arrivals, zeroed before each decode
    int* status = nullptr;    // device status word of the GEMMs' bounded waits
};
constexpr int kCodecCounters = 1024;  // >= the output tiles of any codec GEMM at 5000 codes
cudaError_t codec_tc_init(CodecTc* tc, const CodecWeights& w, cudaStream_t s);
void codec_tc_free(CodecTc* tc);

// Kernels one decode launches.  CUDA-core path: the lookup, the embed conv and
// its LayerNorm, four per ConvNeXt block, the final LayerNorm, linear and up
// conv.  Tensor-core path: two im2col kernels more.
constexpr int kCodecLaunches = 3 + 12 * 4 + 3;
constexpr int kCodecLaunchesTc = kCodecLaunches + 2;
// tc == nullptr: the CUDA-core GEMMs; otherwise the tensor-core GEMMs (the
// activation maps are re-encoded for T rows when T changes).
cudaError_t codec_decode_device(const CodecWeights& w, const CodecScratch& sc, CodecTc* tc, const uint32_t* d_codes,
                                int T, float* out, cudaStream_t s);

}  // namespace itts
