// Shared device-side definitions for the B200 GPT decoder.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "model.hpp"

namespace itts {

// Model dimensions of the IndexTTS 2.5 UnifiedVoice GPT (src/gpt.cpp:7-23).
constexpr int kWidth = 1280;
constexpr int kHeads = 20;
constexpr int kHeadDim = 64;
constexpr int kQkv = 3 * kWidth;
constexpr int kFfn = 5120;
constexpr int kVocab = 8194;
constexpr int kStopCode = 8193;
constexpr int kStartCode = 8192;
constexpr int kKvCapacity = 4096;
constexpr int kMaxLayers = 24;
constexpr int kMaxPrefix = 1024;
constexpr float kLnEps = 1e-5f;

// Decode kernels run 512 threads (16 warps) per CTA, one CTA per SM.
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

// Wall-clock limit of every device-side spin-wait.  A legitimate wait lasts
// microseconds; the limit only turns a lost peer into an error status.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ int ld_volatile(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

// Weights are streamed once per decode step: read-only loads without L1 allocation.
__device__ __forceinline__ float4 ld_stream(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float dot4(float4 a, float4 b, float acc) {
    acc = fmaf(a.x, b.x, acc);
    acc = fmaf(a.y, b.y, acc);
    acc = fmaf(a.z, b.z, acc);
    acc = fmaf(a.w, b.w, acc);
    return acc;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum over all threads of the CTA; `red` holds >= 32 floats.
// Every thread receives the total.  Contains two __syncthreads().
__device__ __forceinline__ float block_sum(float v, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
    return warp_sum(t);
}

__device__ __forceinline__ float block_max(float v, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
    return warp_max(t);
}

// Named barrier 1 over the kThreads consumer threads of a CTA: every thread of
// a kernel launched with kThreads, or the 16 consumer warps of the decode
// kernels, whose extra producer warp never joins it.
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kThreads) : "memory"); }

// csync() that also ORs a predicate across the consumer threads.
__device__ __forceinline__ bool csync_or(bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, 1, %2, pi;\n\t"
        "selp.u32 %0, 1, 0, po;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)p), "n"(kThreads)
        : "memory");
    return r != 0;
}

// Sum / max over the kThreads consumer threads (two csync()).
__device__ __forceinline__ float cblock_sum(float v, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_sum(v);
    csync();
    if (lane == 0) red[warp] = v;
    csync();
    return warp_sum(lane < kWarps ? red[lane] : 0.0f);
}

__device__ __forceinline__ float cblock_max(float v, float* red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    v = warp_max(v);
    csync();
    if (lane == 0) red[warp] = v;
    csync();
    return warp_max(lane < kWarps ? red[lane] : -INFINITY);
}

__device__ __forceinline__ void set_status(int* status, int code, int where, int detail) {
    if (atomicCAS(status, 0, code) == 0) {
        status[1] = where;
        status[2] = blockIdx.x;
        status[3] = detail;
    }
}

// tanh GELU with the clamps of mit2_gelu_f32 (kernels.metal:486-503).
// TF32 rounding to nearest (ties away from zero) of an fp32 value: the top 19
// bits of the word after adding half of the dropped part.  x - rn_tf32(x) is
// exact in fp32; the pair is the hi / lo split of the tensor-core GEMMs.
__device__ __forceinline__ float rn_tf32(float x) {
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

__device__ __forceinline__ float gelu_ref(float v) {
    if (v > 10.0f) return v;
    if (v < -10.0f) return 0.0f;
    return 0.5f * v * (1.0f + tanhf(0.7978845608028654f * (v + 0.044715f * v * v * v)));
}

// GELU 0.5 x (1 + erf(x / sqrt 2)) with erf from the Abramowitz-Stegun 7.1.26
// rational approximation (max error 1.5e-7), the form of itts25_codec_gelu
// (kernels.metal:3132-3137).
__device__ __forceinline__ float gelu_erf(float x) {
    const float v = x * 0.7071067811865475f, a = fabsf(v), t = 1.0f / (1.0f + 0.3275911f * a);
    const float p = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    float erf = 1.0f - p * expf(-a * a);
    if (v < 0.0f) erf = -erf;
    return 0.5f * x * (1.0f + erf);
}

// Two independent fp32 fused multiply-adds (round to nearest even, as fmaf)
// in one instruction: (a.x * b.x + c.x, a.y * b.y + c.y).  Each lane of the
// pair is exactly fmaf of its operands, so a kernel issuing these for two
// independent fma chains computes the same values with half the FMA issue.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// Programmatic dependent launch (PDL).  A kernel launched with programmatic
// stream serialization may start while its predecessor in the stream drains:
// it does what does not depend on it (setup, weight loads), waits for it with
// pdl_wait() before touching the buffers they share, and calls pdl_trigger()
// to let its own successor launch early.  Both are no-ops in a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialization (a programmatic edge when the
// stream is being captured into a graph).
template <class... P, class... A>
cudaError_t launch_pdl(void (*kernel)(P...), dim3 grid, int block, size_t smem, cudaStream_t s, A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

}  // namespace itts
