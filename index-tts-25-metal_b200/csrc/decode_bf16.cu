// The decode kernels with bf16 weight matrices (see decode_body.cuh): the
// streamed rows of c_attn, attn.c_proj, c_fc, mlp.c_proj and mel_head are
// bf16 (half the bytes per step), LayerNorm vectors, biases, activations,
// the KV cache and all arithmetic stay fp32.
#define ITTS_WNS wbf16
#define ITTS_WBF16 1
#include "decode_body.cuh"
#include "decode_batch.cuh"
