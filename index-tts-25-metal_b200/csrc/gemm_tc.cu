// Prefill linears on the 5th-generation tensor cores (tcgen05, sm_100a):
//   C[m, n] = epi(sum_k A[m, k] * W[n, k] + bias[n])
// A [M, K] fp32 row-major (activations), W [N, K] row-major (fp32, or bf16 in a
// bf16-weight context), both K-major.  fp32 accuracy from three TF32 products:
// every operand is split into hi (its top 19 bits, exactly representable in
// TF32) and lo = x - hi (exact in fp32, used as TF32), and the accumulator
// takes hi*hi + hi*lo + lo*hi (the dropped lo*lo and the truncation of lo are
// about 2^-21 relative).
//
// One CTA per 128 x 64 output tile, 128 threads (4 warps).  Per 32-wide K
// block the threads load A and W with coalesced 16-byte loads, split them and
// store hi and lo tiles in shared memory in the 128-byte-swizzled K-major
// layout the tensor core reads (row r at r * 128 bytes, 16-byte chunk c at
// position c ^ (r % 8)); one thread issues the 12 MMAs of the block
// (3 products x 4 K-steps of 8) into a 128 x 64 fp32 accumulator in tensor
// memory and commits them to the stage's mbarrier, which the threads wait on
// before refilling that stage (two stages).  The tensor core's fp32
// accumulation does not round to nearest, so its error grows with K: every
// 256 K the accumulator is drained (tcgen05.ld, warp w owns rows
// 32w..32w+31, thread = row) into fp32 registers with round-to-nearest adds and
// the next chunk starts afresh.  The epilogue applies bias, GELU or the
// residual.  Every mbarrier wait is bounded; on timeout the kernel records a
// status, waits (bounded) for its MMAs and frees its tensor memory before
// returning.
#include <cuda_bf16.h>

#include "common.cuh"
#include "model.hpp"

namespace itts {
namespace {

constexpr int TBM = 128, TBN = 64, TBK = 32;
constexpr int kChunkBlocks = 8;  // K blocks per tensor-memory accumulation chunk (256 K)
constexpr uint32_t kTmemCols = TBN;

struct TcSmem {
    float a[2][2][TBM * TBK];  // [stage][hi, lo], 16 KB each
    float b[2][2][TBN * TBK];  // 8 KB each
    unsigned long long mbar[2];
    unsigned long long chunk_bar;
    uint32_t tmem_base;
};
constexpr size_t kTcSmemBytes = sizeof(TcSmem) + 1024;  // + alignment of the tiles to 1024 bytes

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
           (uint64_t(2) << 61);
}

// Instruction descriptor: D f32, A and B tf32, both K-major, N = 64, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(TBN >> 3) << 17) | (uint32_t(TBM >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer_ns();
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(su32(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ void split(float x, float& hi, float& lo) {
    hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    lo = x - hi;
}

// Loads one ROWS x 32 operand block (rows r0.., K columns k0..) into the hi
// and lo tiles; rows at or beyond `rows` are zero.
template <int ROWS, bool BF16>
__device__ __forceinline__ void load_block(const void* src, int ld, int r0, int rows, int k0, float* hi, float* lo) {
    const int t = threadIdx.x;
#pragma unroll
    for (int i = 0; i < ROWS / 16; ++i) {
        const int idx = t + 128 * i, r = idx >> 3, c = idx & 7;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r0 + r < rows) {
            if (BF16) {
                const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(src) +
                                                                     (size_t)(r0 + r) * ld + k0 + 4 * c));
                v = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                                __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
            } else {
                v = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(src) + (size_t)(r0 + r) * ld + k0) +
                          c);
            }
        }
        float4 h, l;
        split(v.x, h.x, l.x);
        split(v.y, h.y, l.y);
        split(v.z, h.z, l.z);
        split(v.w, h.w, l.w);
        const int off = r * TBK + ((c ^ (r & 7)) << 2);  // 128-byte swizzle within the 8-row group
        *reinterpret_cast<float4*>(hi + off) = h;
        *reinterpret_cast<float4*>(lo + off) = l;
    }
}

template <int EPI, bool WB>
__global__ void __launch_bounds__(128, 1) k_gemm_tc(const float* __restrict__ A, const void* __restrict__ W,
                                                    const float* __restrict__ bias, const float* __restrict__ R,
                                                    float* __restrict__ C, int M, int N, int K, int* status) {
    extern __shared__ unsigned char smem_raw[];
    TcSmem& sm = *reinterpret_cast<TcSmem*>(smem_raw + ((1024 - (su32(smem_raw) & 1023)) & 1023));
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int m0 = blockIdx.y * TBM, n0 = blockIdx.x * TBN;
    if (t == 0) {
        for (int s = 0; s < 2; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&sm.mbar[s])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&sm.chunk_bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = sm.tmem_base;
    const uint32_t row_addr = tmem + (uint32_t(32 * warp) << 16);  // this warp's 32 accumulator rows

    float racc[TBN];
#pragma unroll
    for (int j = 0; j < TBN; ++j) racc[j] = 0.f;
    const int nkb = K / TBK;
    int pending = -1;  // last K block whose MMAs may still be running (-1: none)
    bool ok = true;
    for (int kb = 0; kb < nkb && ok; ++kb) {
        const int st = kb & 1;
        if (kb >= 2 && !mbar_wait(&sm.mbar[st], uint32_t((kb - 2) >> 1) & 1u)) ok = false;
        if (__syncthreads_or(!ok)) break;
        load_block<TBM, false>(A, K, m0, M, kb * TBK, sm.a[st][0], sm.a[st][1]);
        load_block<TBN, WB>(W, K, n0, N, kb * TBK, sm.b[st][0], sm.b[st][1]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> tensor-core reads
        __syncthreads();
        const bool chunk_start = kb % kChunkBlocks == 0;
        const bool chunk_end = kb % kChunkBlocks == kChunkBlocks - 1 || kb == nkb - 1;
        if (t == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ah = su32(sm.a[st][0]), al = su32(sm.a[st][1]);
            const uint32_t bh = su32(sm.b[st][0]), bl = su32(sm.b[st][1]);
#pragma unroll
            for (int ks = 0; ks < TBK / 8; ++ks) {  // 8 TF32 = 32 bytes per K step
                const uint32_t o = 32u * ks;
                mma_tf32(tmem, smem_desc(al + o), smem_desc(bh + o), !(chunk_start && ks == 0));
                mma_tf32(tmem, smem_desc(ah + o), smem_desc(bl + o), 1);
                mma_tf32(tmem, smem_desc(ah + o), smem_desc(bh + o), 1);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             su32(&sm.mbar[st]))
                         : "memory");
            if (chunk_end)
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 su32(&sm.chunk_bar))
                             : "memory");
        }
        pending = kb;
        if (chunk_end) {  // drain: every MMA so far has completed once the chunk barrier flips
            if (!mbar_wait(&sm.chunk_bar, uint32_t(kb / kChunkBlocks) & 1u)) ok = false;
            if (__syncthreads_or(!ok)) break;
            pending = -1;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int c0 = 0; c0 < TBN; c0 += 16) {
                uint32_t v[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
                    "%13, %14, %15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                      "=r"(v[15])
                    : "r"(row_addr + uint32_t(c0)));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 16; ++j) racc[c0 + j] += __uint_as_float(v[j]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncthreads();  // the next chunk overwrites the accumulator
        }
    }
    if (pending >= 0) {  // aborted with MMAs possibly in flight: wait (bounded) before freeing
        if (t == 0)
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             su32(&sm.chunk_bar))
                         : "memory");
        mbar_wait(&sm.chunk_bar, uint32_t(pending / kChunkBlocks) & 1u);
    }
    ok = !__syncthreads_or(!ok);
    if (ok) {
        const int m = m0 + 32 * warp + lane;
        if (m < M) {
#pragma unroll
            for (int j = 0; j < TBN; ++j) {
                const int n = n0 + j;
                const float y = racc[j] + bias[n];
                float out;
                if (EPI == 1)
                    out = gelu_ref(y);
                else if (EPI == 2)
                    out = R[(size_t)m * N + n] + y;
                else
                    out = y;
                C[(size_t)m * N + n] = out;
            }
        }
    } else if (t == 0) {
        set_status(status, kStatusRingTimeout, 500, blockIdx.y * gridDim.x + blockIdx.x);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

template <int EPI, bool WB>
cudaError_t launch_one(const float* A, const void* W, const float* bias, const float* R, float* C, int M, int N, int K,
                       int* status, cudaStream_t s) {
    static bool configured[64] = {};  // the attribute is per function and device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(k_gemm_tc<EPI, WB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTcSmemBytes);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    dim3 grid(N / TBN, (M + TBM - 1) / TBM);
    k_gemm_tc<EPI, WB><<<grid, 128, kTcSmemBytes, s>>>(A, W, bias, R, C, M, N, K, status);
    return cudaGetLastError();
}

}  // namespace

bool gemm_tc_supported(int N, int K) { return N % TBN == 0 && K % TBK == 0; }

cudaError_t launch_gemm_tc(int epi, bool wbf16, const float* A, const void* W, const float* bias, const float* R,
                           float* C, int M, int N, int K, int* status, cudaStream_t s) {
    switch (epi * 2 + (wbf16 ? 1 : 0)) {
        case 0: return launch_one<0, false>(A, W, bias, R, C, M, N, K, status, s);
        case 1: return launch_one<0, true>(A, W, bias, R, C, M, N, K, status, s);
        case 2: return launch_one<1, false>(A, W, bias, R, C, M, N, K, status, s);
        case 3: return launch_one<1, true>(A, W, bias, R, C, M, N, K, status, s);
        case 4: return launch_one<2, false>(A, W, bias, R, C, M, N, K, status, s);
        default: return launch_one<2, true>(A, W, bias, R, C, M, N, K, status, s);
    }
}

}  // namespace itts
