// Load-time and conditioning kernels: the Conv1D weight transpose and
// GptDecoder::prepare on the device.
#include <cuda_bf16.h>

#include "common.cuh"
#include "model.hpp"

namespace itts {

// out[c, r] = in[r, c] for in [rows_in, cols_in] (HF Conv1D [in, out] ->
// row-major [out, in], the transpose gpt.cpp:24-33 caches on the CPU).
__device__ __forceinline__ void store_w(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_w(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <class T>
__global__ void k_transpose(const float* __restrict__ in, T* __restrict__ out, int rows_in, int cols_in) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows_in && c < cols_in) tile[i][threadIdx.x] = in[(size_t)r * cols_in + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows_in && c < cols_in) store_w(out + (size_t)c * rows_in + r, tile[threadIdx.x][i]);
    }
}

cudaError_t launch_transpose(const float* in, float* out, int rows_in, int cols_in, cudaStream_t s) {
    dim3 grid((cols_in + 31) / 32, (rows_in + 31) / 32);
    k_transpose<float><<<grid, dim3(32, 8), 0, s>>>(in, out, rows_in, cols_in);
    return cudaGetLastError();
}

cudaError_t launch_transpose_bf16(const float* in, void* out, int rows_in, int cols_in, cudaStream_t s) {
    dim3 grid((cols_in + 31) / 32, (rows_in + 31) / 32);
    k_transpose<__nv_bfloat16><<<grid, dim3(32, 8), 0, s>>>(in, static_cast<__nv_bfloat16*>(out), rows_in, cols_in);
    return cudaGetLastError();
}

__global__ void k_to_bf16(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __float2bfloat16_rn(in[i]);
}

cudaError_t launch_to_bf16(const float* in, void* out, size_t n, cudaStream_t s) {
    k_to_bf16<<<1184, 256, 0, s>>>(in, static_cast<__nv_bfloat16*>(out), n);
    return cudaGetLastError();
}

// GptDecoder::prepare (gpt.cpp:42-71) after host-side id framing:
//   row 0      speaker_cond = (spk_emb_proj . speaker + bias) + emotion
//   rows 1, 2  zeros
//   rows 3..   (text_embedding[id] + text_pos[i]) + lang_embedding[language]
//   last row   mel_embedding[8192] + mel_pos_embedding[0]
__global__ void __launch_bounds__(256) k_prepare(PrepareArgs a) {
    const int row = blockIdx.x;
    float* o = a.out + (size_t)row * kWidth;
    if (row == 0) {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int r = warp; r < kWidth; r += 8) {
            const float* w = a.spk_w + (size_t)r * 192;
            float acc = 0.f;
            for (int c = lane; c < 192; c += 32) acc = fmaf(w[c], a.speaker[c], acc);
            acc = warp_sum(acc);
            if (lane == 0) o[r] = (acc + a.spk_b[r]) + a.emotion[r];
        }
    } else if (row < 3) {
        for (int c = threadIdx.x; c < kWidth; c += blockDim.x) o[c] = 0.f;
    } else if (row < 3 + (int)a.n_ids) {
        const int i = row - 3;
        const float* te = a.text_emb + (size_t)a.ids[i] * kWidth;
        const float* tp = a.text_pos + (size_t)i * kWidth;
        const float* le = a.lang_emb + (size_t)a.language * kWidth;
        for (int c = threadIdx.x; c < kWidth; c += blockDim.x) o[c] = (te[c] + tp[c]) + le[c];
    } else {
        const float* me = a.mel_emb + (size_t)kStartCode * kWidth;
        for (int c = threadIdx.x; c < kWidth; c += blockDim.x) o[c] = me[c] + a.mel_pos[c];
    }
}

cudaError_t launch_prepare(const PrepareArgs& a, cudaStream_t s) {
    k_prepare<<<3 + a.n_ids + 1, 256, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace itts
