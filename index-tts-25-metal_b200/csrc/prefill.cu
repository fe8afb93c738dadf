// Prefill of the GPT prefix (src/gpt.cpp:88-125 with initial=true) on B200.
//
// T <= 1024 rows.  Per layer: LayerNorm rows, the QKV GEMM, the K/V store into
// the cache (head-major layout), causal attention, c_proj GEMM with the
// residual fused, LayerNorm, c_fc GEMM with GELU fused, mlp.c_proj GEMM with
// the residual fused.  GEMMs are C[T, N] = A[T, K] . W[N, K]^T with fp32
// accuracy (the reference's MPS fp32 GEMMs, metal_context.mm:368-410): by
// default on the tensor cores (gemm_tma.cu, TF32 hi / lo operands, the chain
// launched with PDL); in prefill mode 1 on the CUDA cores (k_gemm_nt below).
#include "common.cuh"
#include "model.hpp"

namespace itts {

// mit2_layernorm_f32_rows (kernels.metal:618-669): one CTA per row.
// With `out_lo` the row is written split for the tensor-core GEMM: out =
// rn_tf32(y), out_lo = rn_tf32(y - out).
__global__ void __launch_bounds__(256) k_ln_rows(const float* __restrict__ x, const float* __restrict__ g,
                                                 const float* __restrict__ b, float* __restrict__ out,
                                                 float* __restrict__ out_lo) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();  // x is the previous kernel's output
    const float* row = x + (size_t)blockIdx.x * kWidth;
    float v[5];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        v[j] = row[threadIdx.x + 256 * j];
        s += v[j];
    }
    const float mean = block_sum(s, red) * (1.0f / kWidth);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        const float d = v[j] - mean;
        q = fmaf(d, d, q);
    }
    const float var = block_sum(q, red) * (1.0f / kWidth);
    const float inv = 1.0f / sqrtf(var + kLnEps);
    float* o = out + (size_t)blockIdx.x * kWidth;
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        const int c = threadIdx.x + 256 * j;
        const float y = (v[j] - mean) * inv * g[c] + b[c];
        if (out_lo) {
            const float h = rn_tf32(y);
            o[c] = h;
            out_lo[(size_t)blockIdx.x * kWidth + c] = rn_tf32(y - h);
        } else {
            o[c] = y;
        }
    }
}

enum GemmEpi : int { kEpiBias = 0, kEpiGelu = 1, kEpiResid = 2 };

// W is fp32, or bf16 when WB (widened to fp32 on load: bf16 is the high half
// of an fp32 word).  64x64 output tile, 4x4 per thread, k-tiles of 32 (K must
// be a multiple of 32): the next tile's global loads are in flight while the
// current one is multiplied, and 32 k-steps per tile cover most of their L2
// latency.  Each output sums its K products in k order.
template <int EPI, bool WB>
__global__ void __launch_bounds__(256) k_gemm_nt(const float* __restrict__ A, const void* __restrict__ Wv,
                                                 const float* __restrict__ bias, const float* __restrict__ R,
                                                 float* __restrict__ C, int M, int N, int K) {
    constexpr int BM = 64, BN = 64, BK = 32;
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Ws[2][BK][BN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int lr = tid >> 2, lk = (tid & 3) * 4;  // and lk + 16
    float4 ra[2], rw[2];
    auto gload = [&](int k0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kk = k0 + lk + 16 * h;
            ra[h] = (m0 + lr < M) ? *reinterpret_cast<const float4*>(A + (size_t)(m0 + lr) * K + kk)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            if (n0 + lr >= N) {
                rw[h] = make_float4(0.f, 0.f, 0.f, 0.f);
            } else if (WB) {
                const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(Wv) +
                                                                     (size_t)(n0 + lr) * K + kk));
                rw[h] = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                                    __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
            } else {
                rw[h] = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(Wv) + (size_t)(n0 + lr) * K + kk));
            }
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kk = lk + 16 * h;
            As[buf][kk + 0][lr] = ra[h].x;
            As[buf][kk + 1][lr] = ra[h].y;
            As[buf][kk + 2][lr] = ra[h].z;
            As[buf][kk + 3][lr] = ra[h].w;
            Ws[buf][kk + 0][lr] = rw[h].x;
            Ws[buf][kk + 1][lr] = rw[h].y;
            Ws[buf][kk + 2][lr] = rw[h].z;
            Ws[buf][kk + 3][lr] = rw[h].w;
        }
    };
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    gload(0);
    sstore(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += BK) {
        const bool more = k0 + BK < K;
        if (more) gload(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 w = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
            const float av[4] = {a.x, a.y, a.z, a.w}, wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], wv[j], acc[i][j]);
        }
        if (more) sstore(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n >= N) continue;
            const float y = acc[i][j] + bias[n];
            float out;
            if (EPI == kEpiGelu)
                out = gelu_ref(y);
            else if (EPI == kEpiResid)
                out = R[(size_t)m * N + n] + y;
            else
                out = y;
            C[(size_t)m * N + n] = out;
        }
    }
}

// mit2_gpt_kv_store_f32 (kernels.metal:1250-1266) into the head-major cache
// [K|V][head][4096][64] of one layer.
__global__ void k_kv_store(const float* __restrict__ qkv, float* __restrict__ kv_layer, int T) {
    pdl_trigger();
    pdl_wait();
    const size_t n = (size_t)T * 2 * kWidth;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (2 * kWidth)), rem = (int)(i % (2 * kWidth));
        const int sel = rem / kWidth, c = rem % kWidth, h = c / kHeadDim, d = c % kHeadDim;
        kv_layer[(((size_t)sel * kHeads + h) * kKvCapacity + t) * kHeadDim + d] = qkv[(size_t)t * kQkv + kWidth + rem];
    }
}

// Causal multi-head attention over packed qkv [T, 3840] (q | k | v, head h at
// h*64), scale 1/8, as mit2_gpt_causal_attention_sgq_f32
// (kernels.metal:2249-2290), with an online softmax over 64-key tiles.
// CTA = (head, 64 queries, chunk of kAttChunk keys): the keys a query block
// reaches are split into chunks so that no CTA walks more than two tiles (a
// single CTA per block left the last blocks of long prefixes as the critical
// path).  256 threads as 16 x 16: thread (ty, tx) owns the scores of queries
// 4ty..4ty+3 x keys 4tx..4tx+3 of a tile and the outputs of those queries x
// dims 4tx..4tx+3.  Q and K are staged d-major (QT[d][q], KT[d][k]) and V and
// the tile's probabilities row-major, so every inner step is two or eight
// 16-byte shared loads per 16 or 64 FMAs.  A query row's 64 scores live in one
// half-warp, reduced with shuffles.
// A block with one chunk writes its output; otherwise every chunk writes its
// (max, sum, unnormalised output) partial and the last of the block's chunks to
// arrive merges them in chunk order (deterministic whichever arrives last).
// With `out_lo` the output is written split (as k_ln_rows).
constexpr int kAttLd = 68;  // row stride of the staged 64 x 64 tiles (floats)
constexpr size_t kAttSmem = 4 * 64 * kAttLd * sizeof(float);
static_assert(kAttChunk % 64 == 0, "key chunks are whole tiles");
static_assert(kAttPartLd >= 66 && kAttPartLd % 4 == 0, "partial rows: 64 outputs, max, sum");

__device__ __forceinline__ float half_max(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float half_sum(float v) {
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void attn_store(float* out, float* out_lo, size_t o, float4 y) {
    if (out_lo) {
        const float4 hv = make_float4(rn_tf32(y.x), rn_tf32(y.y), rn_tf32(y.z), rn_tf32(y.w));
        *reinterpret_cast<float4*>(out + o) = hv;
        *reinterpret_cast<float4*>(out_lo + o) =
            make_float4(rn_tf32(y.x - hv.x), rn_tf32(y.y - hv.y), rn_tf32(y.z - hv.z), rn_tf32(y.w - hv.w));
    } else {
        *reinterpret_cast<float4*>(out + o) = y;
    }
}

__global__ void __launch_bounds__(256) k_causal_attn(const float* __restrict__ qkv, float* __restrict__ out,
                                                     float* __restrict__ out_lo, int T, float* part, int* cnt) {
    extern __shared__ __align__(16) float att_smem[];
    __shared__ int is_last;
    float* QT = att_smem;             // [64 d][kAttLd]: Q of the block, d-major
    float* KT = QT + 64 * kAttLd;     // [64 d][kAttLd]: K of the tile, d-major
    float* Vs = KT + 64 * kAttLd;     // [64 k][kAttLd]
    float* Ps = Vs + 64 * kAttLd;     // [64 q][kAttLd]: the tile's probabilities
    const int h = blockIdx.x, qb = blockIdx.y, q0 = qb * 64, tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int lr = tid & 63, ld4 = tid >> 6;  // staging: row lr, 16-byte column groups ld4, ld4 + 4, ...
    const int kend = min(T, q0 + 64);  // keys 0 .. kend-1 reach some query of the block
    const int nck = (kend + kAttChunk - 1) / kAttChunk;
    pdl_trigger();
    if ((int)blockIdx.z >= nck) return;  // the grid covers the longest block's chunks
    const int kb = blockIdx.z * kAttChunk, ke = min(kend, kb + kAttChunk);
    pdl_wait();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int d = 4 * (ld4 + 4 * j), q = q0 + lr;
        const float4 v = q < T ? *reinterpret_cast<const float4*>(qkv + (size_t)q * kQkv + h * kHeadDim + d)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        QT[(d + 0) * kAttLd + lr] = v.x;
        QT[(d + 1) * kAttLd + lr] = v.y;
        QT[(d + 2) * kAttLd + lr] = v.z;
        QT[(d + 3) * kAttLd + lr] = v.w;
    }
    float m[4], l[4], acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -INFINITY;
        l[a] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;
    }
    for (int k0 = kb; k0 < ke; k0 += 64) {
        __syncthreads();  // the previous tile's K, V and P are consumed
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int d = 4 * (ld4 + 4 * j), key = k0 + lr;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (key < ke) {
                const float* row = qkv + (size_t)key * kQkv + h * kHeadDim + d;
                kv = *reinterpret_cast<const float4*>(row + kWidth);
                vv = *reinterpret_cast<const float4*>(row + 2 * kWidth);
            }
            KT[(d + 0) * kAttLd + lr] = kv.x;
            KT[(d + 1) * kAttLd + lr] = kv.y;
            KT[(d + 2) * kAttLd + lr] = kv.z;
            KT[(d + 3) * kAttLd + lr] = kv.w;
            *reinterpret_cast<float4*>(Vs + lr * kAttLd + d) = vv;
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) sc[a][b] = 0.f;
#pragma unroll 8
        for (int d = 0; d < 64; ++d) {
            const float4 qv = *reinterpret_cast<const float4*>(QT + d * kAttLd + 4 * ty);
            const float4 kv = *reinterpret_cast<const float4*>(KT + d * kAttLd + 4 * tx);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
            const float2 k01 = make_float2(kv.x, kv.y), k23 = make_float2(kv.z, kv.w);
#pragma unroll
            for (int a = 0; a < 4; ++a) {  // paired fmas: each half is fmaf(qa[a], kb[b], sc[a][b])
                const float2 q2 = make_float2(qa[a], qa[a]);
                const float2 s01 = fma2(q2, k01, make_float2(sc[a][0], sc[a][1]));
                const float2 s23 = fma2(q2, k23, make_float2(sc[a][2], sc[a][3]));
                sc[a][0] = s01.x, sc[a][1] = s01.y, sc[a][2] = s23.x, sc[a][3] = s23.y;
            }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int q = q0 + 4 * ty + a;
            float mx = -INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int key = k0 + 4 * tx + b;
                sc[a][b] = (key <= q && key < ke) ? sc[a][b] * 0.125f : -INFINITY;
                mx = fmaxf(mx, sc[a][b]);
            }
            const float mn = fmaxf(m[a], half_max(mx));
            const float corr = mn == -INFINITY ? 1.f : expf(m[a] - mn);
            float ps = 0.f;
            float4 pv;
            float* pp = &pv.x;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                pp[b] = sc[a][b] == -INFINITY ? 0.f : expf(sc[a][b] - mn);
                ps += pp[b];
            }
            *reinterpret_cast<float4*>(Ps + (4 * ty + a) * kAttLd + 4 * tx) = pv;
            l[a] = l[a] * corr + half_sum(ps);
            m[a] = mn;
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][c] *= corr;
        }
        __syncthreads();
#pragma unroll 4
        for (int k = 0; k < 64; k += 4) {
            float4 pr[4], vr[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) pr[a] = *reinterpret_cast<const float4*>(Ps + (4 * ty + a) * kAttLd + k);
#pragma unroll
            for (int i = 0; i < 4; ++i) vr[i] = *reinterpret_cast<const float4*>(Vs + (k + i) * kAttLd + 4 * tx);
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                const float p4[4] = {pr[a].x, pr[a].y, pr[a].z, pr[a].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {  // paired fmas, each half fmaf(p, v, acc)
                    const float2 p2 = make_float2(p4[i], p4[i]);
                    const float2 a01 = fma2(p2, make_float2(vr[i].x, vr[i].y), make_float2(acc[a][0], acc[a][1]));
                    const float2 a23 = fma2(p2, make_float2(vr[i].z, vr[i].w), make_float2(acc[a][2], acc[a][3]));
                    acc[a][0] = a01.x, acc[a][1] = a01.y, acc[a][2] = a23.x, acc[a][3] = a23.y;
                }
            }
        }
    }
    if (nck == 1) {
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int q = q0 + 4 * ty + a;
            if (q >= T) continue;
            const float inv = 1.0f / l[a];
            attn_store(out, out_lo, (size_t)q * kWidth + h * kHeadDim + 4 * tx,
                       make_float4(acc[a][0] * inv, acc[a][1] * inv, acc[a][2] * inv, acc[a][3] * inv));
        }
        return;
    }
    // partial of chunk z: row r = [64 outputs | max | sum | pad]
    float* blk = part + ((size_t)h * kAttMaxBlocks + qb) * kAttMaxChunks * 64 * kAttPartLd;
    float* mine = blk + (size_t)blockIdx.z * 64 * kAttPartLd;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        float* row = mine + (4 * ty + a) * kAttPartLd;
        *reinterpret_cast<float4*>(row + 4 * tx) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
        if (tx == 0) *reinterpret_cast<float2*>(row + 64) = make_float2(m[a], l[a]);
    }
    __syncthreads();  // every partial store of this CTA is issued
    if (tid == 0) {
        // The acq_rel add releases the stores the barrier ordered before it
        // and, for the last arriver, acquires the other chunks'.
        int* c = cnt + h * kAttMaxBlocks + qb;
        int prev;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(c) : "memory");
        const int last = prev == nck - 1;
        if (last) *c = 0;
        is_last = last;
    }
    __syncthreads();
    if (!is_last) return;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int r = 4 * ty + a, q = q0 + r;
        if (q >= T) continue;  // (no key reaches a padding row: its max is -inf)
        float mx = -INFINITY;
        for (int c = 0; c < nck; ++c) mx = fmaxf(mx, __ldcg(blk + ((size_t)c * 64 + r) * kAttPartLd + 64));
        float sum = 0.f;
        float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < nck; ++c) {  // chunk order
            const float* row = blk + ((size_t)c * 64 + r) * kAttPartLd;
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(row + 64));
            const float4 v = __ldcg(reinterpret_cast<const float4*>(row + 4 * tx));
            const float w = expf(ml.x - mx);  // every chunk holds key 0 or a key <= the block's first query
            sum = fmaf(ml.y, w, sum);
            y.x = fmaf(v.x, w, y.x);
            y.y = fmaf(v.y, w, y.y);
            y.z = fmaf(v.z, w, y.z);
            y.w = fmaf(v.w, w, y.w);
        }
        const float inv = 1.0f / sum;
        attn_store(out, out_lo, (size_t)q * kWidth + h * kHeadDim + 4 * tx,
                   make_float4(y.x * inv, y.y * inv, y.z * inv, y.w * inv));
    }
}

static cudaError_t launch_attn(const PrefillArgs& p, float* out, float* out_lo, cudaStream_t s) {
    const int T = p.T;
    if (T < 1 || T > kAttMaxBlocks * 64) return cudaErrorInvalidValue;
    static bool configured[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        e = cudaFuncSetAttribute(k_causal_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttSmem);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    const dim3 grid(kHeads, (T + 63) / 64, (T + kAttChunk - 1) / kAttChunk);
    return launch_pdl(k_causal_attn, grid, 256, kAttSmem, s, (const float*)p.qkv, out, out_lo, T, p.att_part,
                      p.att_cnt);
}

cudaError_t launch_gemm_tma(TmaPrefill* p, int layer, int mat, const float* bias, const float* R, float* C,
                            float* C_lo, int M, int* status, cudaStream_t s);

// Prefill mode 1: the CUDA-core tiles above (fp32 or bf16 weights).
static_assert(kWidth % 32 == 0 && kFfn % 32 == 0, "k_gemm_nt k-tiles of 32");
template <int EPI>
static void gemm(const float* A, const float* W, bool wb, const float* bias, const float* R, float* C, int M, int N,
                 int K, cudaStream_t s) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    if (wb)
        k_gemm_nt<EPI, true><<<grid, 256, 0, s>>>(A, W, bias, R, C, M, N, K);
    else
        k_gemm_nt<EPI, false><<<grid, 256, 0, s>>>(A, W, bias, R, C, M, N, K);
}

// Prefill mode 0: the TMA-fed tensor-core GEMM (gemm_tma.cu); the operands of
// every GEMM are split into TF32 hi / lo by the kernel that produces them.
// Every kernel of the chain is launched with PDL: it starts while its
// predecessor drains (the GEMM requests its first weight tiles then) and
// waits for it before touching shared buffers, so a kernel completes only
// after all before it have.
static cudaError_t prefill_layers_tma(const PrefillArgs& p, cudaStream_t s, uint64_t* launches) {
    const int T = p.T;
    TmaPrefill* q = p.tma;
    // A CTA that gave up leaves its tile's split-K counter behind.
    cudaError_t e = cudaMemsetAsync(q->counters, 0, TmaPrefill::kCounters * sizeof(int), s);
    if (e != cudaSuccess) return e;
    const int kv_grid = min(1184, (T * 2 * kWidth + 255) / 256);
    for (int l = 0; l < p.hw->layers; ++l) {
        const LayerW& L = p.hw->layer[l];
        if ((e = launch_pdl(k_ln_rows, dim3(T), 256, 0, s, p.hidden, L.ln1_g, L.ln1_b, q->x_hi, q->x_lo)) !=
            cudaSuccess)
            return e;
        if ((e = launch_gemm_tma(q, l, kMatQkv, L.b_qkv, nullptr, p.qkv, nullptr, T, p.status, s)) != cudaSuccess)
            return e;
        if ((e = launch_pdl(k_kv_store, dim3(kv_grid), 256, 0, s, p.qkv,
                            p.kv + (size_t)l * 2 * kHeads * kKvCapacity * kHeadDim, T)) != cudaSuccess)
            return e;
        if ((e = launch_attn(p, q->att_hi, q->att_lo, s)) != cudaSuccess) return e;
        if ((e = launch_gemm_tma(q, l, kMatO, L.b_o, p.hidden, p.r, nullptr, T, p.status, s)) != cudaSuccess)
            return e;
        if ((e = launch_pdl(k_ln_rows, dim3(T), 256, 0, s, p.r, L.ln2_g, L.ln2_b, q->x_hi, q->x_lo)) != cudaSuccess)
            return e;
        if ((e = launch_gemm_tma(q, l, kMatFc, L.b_fc, nullptr, q->ff_hi, q->ff_lo, T, p.status, s)) != cudaSuccess)
            return e;
        if ((e = launch_gemm_tma(q, l, kMatMp, L.b_mp, p.r, p.hidden, nullptr, T, p.status, s)) != cudaSuccess)
            return e;
        *launches += 8;
    }
    return cudaGetLastError();
}

cudaError_t launch_prefill_layers(const PrefillArgs& p, cudaStream_t s, uint64_t* launches) {
    if (p.tma) return prefill_layers_tma(p, s, launches);
    const int T = p.T;
    for (int l = 0; l < p.hw->layers; ++l) {
        const LayerW& L = p.hw->layer[l];
        k_ln_rows<<<T, 256, 0, s>>>(p.hidden, L.ln1_g, L.ln1_b, p.x, nullptr);
        gemm<kEpiBias>(p.x, L.w_qkv, p.wbf16, L.b_qkv, nullptr, p.qkv, T, kQkv, kWidth, s);
        k_kv_store<<<min(1184, (T * 2 * kWidth + 255) / 256), 256, 0, s>>>(
            p.qkv, p.kv + (size_t)l * 2 * kHeads * kKvCapacity * kHeadDim, T);
        if (cudaError_t e = launch_attn(p, p.att, nullptr, s); e != cudaSuccess) return e;
        gemm<kEpiResid>(p.att, L.w_o, p.wbf16, L.b_o, p.hidden, p.r, T, kWidth, kWidth, s);
        k_ln_rows<<<T, 256, 0, s>>>(p.r, L.ln2_g, L.ln2_b, p.x, nullptr);
        gemm<kEpiGelu>(p.x, L.w_fc, p.wbf16, L.b_fc, nullptr, p.ff, T, kFfn, kWidth, s);
        gemm<kEpiResid>(p.ff, L.w_mp, p.wbf16, L.b_mp, p.r, p.hidden, T, kWidth, kFfn, s);
        *launches += 8;
    }
    return cudaGetLastError();
}

}  // namespace itts
