// Prefill of the GPT prefix (src/gpt.cpp:88-125 with initial=true) on B200.
//
// T <= 1024 rows.  Per layer: LayerNorm rows, the QKV GEMM, the K/V store into
// the cache (head-major layout), causal attention, c_proj GEMM with the
// residual fused, LayerNorm, c_fc GEMM with GELU fused, mlp.c_proj GEMM with
// the residual fused.  GEMMs are C[T, N] = A[T, K] . W[N, K]^T in fp32 on the
// CUDA cores (64x64 tiles, double-buffered shared memory), which keeps fp32
// parity with the reference's MPS fp32 GEMMs (metal_context.mm:368-410).
#include "common.cuh"
#include "model.hpp"

namespace itts {

// mit2_layernorm_f32_rows (kernels.metal:618-669): one CTA per row.
__global__ void __launch_bounds__(256) k_ln_rows(const float* __restrict__ x, const float* __restrict__ g,
                                                 const float* __restrict__ b, float* __restrict__ out) {
    __shared__ float red[32];
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
        o[c] = (v[j] - mean) * inv * g[c] + b[c];
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
    const size_t n = (size_t)T * 2 * kWidth;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (2 * kWidth)), rem = (int)(i % (2 * kWidth));
        const int sel = rem / kWidth, c = rem % kWidth, h = c / kHeadDim, d = c % kHeadDim;
        kv_layer[(((size_t)sel * kHeads + h) * kKvCapacity + t) * kHeadDim + d] = qkv[(size_t)t * kQkv + kWidth + rem];
    }
}

// Causal multi-head attention over packed qkv [T, 3840] (q | k | v, head h at
// h*64), scale 1/8, as mit2_gpt_causal_attention_sgq_f32
// (kernels.metal:2249-2290).  CTA = (head, 16 queries); warp = one query with
// an online softmax over 64-key tiles staged in shared memory.
__global__ void __launch_bounds__(512) k_causal_attn(const float* __restrict__ qkv, float* __restrict__ out, int T) {
    __shared__ float Ks[64][65];
    __shared__ __align__(16) float Vs[64][64];
    __shared__ float Qs[16][64];
    const int h = blockIdx.x, q0 = blockIdx.y * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tq = q0 + warp;
    for (int i = threadIdx.x; i < 16 * 64; i += 512) {
        const int w = i / 64, d = i % 64;
        Qs[w][d] = (q0 + w < T) ? qkv[(size_t)(q0 + w) * kQkv + h * kHeadDim + d] : 0.f;
    }
    const int kmax = min(T, q0 + 16);
    float m = -INFINITY, l = 0.f, acc0 = 0.f, acc1 = 0.f;
    for (int kt = 0; kt < kmax; kt += 64) {
        __syncthreads();
        for (int i = threadIdx.x; i < 64 * 64; i += 512) {
            const int r = i / 64, d = i % 64, key = kt + r;
            const bool ok = key < kmax;
            Ks[r][d] = ok ? qkv[(size_t)key * kQkv + kWidth + h * kHeadDim + d] : 0.f;
            Vs[r][d] = ok ? qkv[(size_t)key * kQkv + 2 * kWidth + h * kHeadDim + d] : 0.f;
        }
        __syncthreads();
        if (tq < T && kt <= tq) {
            float s[2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int j = lane + 32 * hh, key = kt + j;
                float d0 = 0.f;
                if (key <= tq) {
#pragma unroll 16
                    for (int d = 0; d < 64; ++d) d0 = fmaf(Qs[warp][d], Ks[j][d], d0);
                    s[hh] = d0 * 0.125f;
                } else {
                    s[hh] = -INFINITY;
                }
            }
            const float mt = warp_max(fmaxf(s[0], s[1]));
            const float mn = fmaxf(m, mt);
            const float corr = expf(m - mn);
            const float p0 = s[0] == -INFINITY ? 0.f : expf(s[0] - mn);
            const float p1 = s[1] == -INFINITY ? 0.f : expf(s[1] - mn);
            l = l * corr + warp_sum(p0 + p1);
            acc0 *= corr;
            acc1 *= corr;
#pragma unroll 8
            for (int j = 0; j < 64; ++j) {
                const float pj = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
                const float2 v = *reinterpret_cast<const float2*>(&Vs[j][2 * lane]);
                acc0 = fmaf(pj, v.x, acc0);
                acc1 = fmaf(pj, v.y, acc1);
            }
            m = mn;
        }
    }
    if (tq < T) {
        float* o = out + (size_t)tq * kWidth + h * kHeadDim;
        o[2 * lane] = acc0 / l;
        o[2 * lane + 1] = acc1 / l;
    }
}

bool gemm_tc_supported(int N, int K);
cudaError_t launch_gemm_tc(int epi, bool wbf16, const float* A, const void* W, const float* bias, const float* R,
                           float* C, int M, int N, int K, int* status, cudaStream_t s);

// The tensor-core GEMM (gemm_tc.cu, three TF32 products) serves the bf16-
// weight path.  fp32 weights keep the SIMT tiles above: the tensor core's fp32
// accumulation, even drained every 256 K, leaves prefill logits about 3x
// further from the reference (8e-6 vs 3e-6 max_abs on the 24-layer model),
// enough to change a 1024-code sampled run that the fp32 path reproduces.
static_assert(kWidth % 32 == 0 && kFfn % 32 == 0, "k_gemm_nt k-tiles of 32");
template <int EPI>
static void gemm(const float* A, const float* W, bool wb, const float* bias, const float* R, float* C, int M, int N,
                 int K, int* status, cudaStream_t s) {
    if (wb && gemm_tc_supported(N, K)) {
        launch_gemm_tc(EPI, wb, A, W, bias, R, C, M, N, K, status, s);
        return;
    }
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    if (wb)
        k_gemm_nt<EPI, true><<<grid, 256, 0, s>>>(A, W, bias, R, C, M, N, K);
    else
        k_gemm_nt<EPI, false><<<grid, 256, 0, s>>>(A, W, bias, R, C, M, N, K);
}

cudaError_t launch_prefill_layers(const PrefillArgs& p, cudaStream_t s, uint64_t* launches) {
    const int T = p.T;
    for (int l = 0; l < p.hw->layers; ++l) {
        const LayerW& L = p.hw->layer[l];
        k_ln_rows<<<T, 256, 0, s>>>(p.hidden, L.ln1_g, L.ln1_b, p.x);
        gemm<kEpiBias>(p.x, L.w_qkv, p.wbf16, L.b_qkv, nullptr, p.qkv, T, kQkv, kWidth, p.status, s);
        k_kv_store<<<min(1184, (T * 2 * kWidth + 255) / 256), 256, 0, s>>>(
            p.qkv, p.kv + (size_t)l * 2 * kHeads * kKvCapacity * kHeadDim, T);
        k_causal_attn<<<dim3(kHeads, (T + 15) / 16), 512, 0, s>>>(p.qkv, p.att, T);
        gemm<kEpiResid>(p.att, L.w_o, p.wbf16, L.b_o, p.hidden, p.r, T, kWidth, kWidth, p.status, s);
        k_ln_rows<<<T, 256, 0, s>>>(p.r, L.ln2_g, L.ln2_b, p.x);
        gemm<kEpiGelu>(p.x, L.w_fc, p.wbf16, L.b_fc, nullptr, p.ff, T, kFfn, kWidth, p.status, s);
        gemm<kEpiResid>(p.ff, L.w_mp, p.wbf16, L.b_mp, p.r, p.hidden, T, kWidth, kFfn, p.status, s);
        *launches += 8;
    }
    return cudaGetLastError();
}

}  // namespace itts
