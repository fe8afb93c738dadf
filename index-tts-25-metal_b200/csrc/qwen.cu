// Qwen3-0.6B decoder (src/qwen.cpp) on B200: the kernels of one prefill and
// of one decode step.
//
// Prefill of T prompt tokens (the GEMMs run on the tensor cores through
// gemm_tma.cu, operands split into TF32 hi / lo):
//   embedding rows -> 28 x { RMSNorm (split) -> q|k|v GEMM -> per-head
//   q/k RMSNorm + RoPE, K/V into the cache -> causal GQA attention (split)
//   -> o_proj GEMM + residual -> RMSNorm (split) -> gate|up GEMM with the
//   SwiGLU epilogue (split) -> down GEMM + residual } -> final RMSNorm of the
//   last row fused into the tied-head GEMV -> argmax.
// One decode step (a CUDA graph replayed per token; every kernel reads the
// token and position from the device State and returns at once after EOS):
//   embedding row -> 28 x { RMSNorm fused into the q|k|v GEMV -> q/k RMSNorm
//   + RoPE + K/V append -> split-K attention over 64-key chunks (both query
//   heads of a KV head per CTA) -> merge -> o_proj GEMV + residual -> RMSNorm
//   fused into the gate|up GEMV with SiLU(gate) * up -> down GEMV + residual }
//   -> head GEMV -> argmax, which advances the State.
// The GEMVs stream fp32 weights with read-only, L1-bypassing 16-byte loads, one
// warp per row, every lane with K/128 loads in flight; each output sums its
// products in a fixed order, so results are deterministic.
//
// Kernel math follows vendor/metal-runtime/metal/kernels.metal:
// mit2_rmsnorm_f32_rows_eps (:995-1030, x * rsqrt(mean(x^2) + eps) * g),
// itts25_qwen_rope (:3111-3115, half rotation, theta 1e6),
// itts25_qwen_attention (:3119-3131, scale 1/sqrt(128), KV head = head / 2),
// mit2_silu_mul_f32 (:363-374), mit2_gpt_argmax_f32 (:1269-1305, first index of
// the maximum) and mit2_embedding_f32 (:281-294).
#include <cmath>
#include <utility>

#include "common.cuh"
#include "qwen.hpp"

namespace itts {
namespace qwen {
namespace {

// RoPE inverse frequencies 1e6^(-j/64), j < 64: the correctly rounded floats
// (set once by init_tables); the angle is their float product with the position.
__constant__ float c_inv_freq[64];

constexpr float kScale = 0.08838834764831844f;  // 1 / sqrt(128)

__device__ __forceinline__ bool finished(const State* st) { return st && *reinterpret_cast<const volatile uint32_t*>(&st->done); }

// Sum over a CTA of 128 or 256 threads (every thread receives it).
template <int kThreadsT>
__device__ __forceinline__ float cta_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < kThreadsT / 32; ++i) t += red[i];
    return t;
}

__global__ void __launch_bounds__(256) k_embed(const float* __restrict__ table, const uint32_t* __restrict__ ids,
                                               float* __restrict__ out, const State* st) {
    if (finished(st)) return;
    const uint32_t id = st ? st->token : ids[blockIdx.x];
    reinterpret_cast<float4*>(out + (size_t)blockIdx.x * kDim)[threadIdx.x] =
        reinterpret_cast<const float4*>(table + (size_t)id * kDim)[threadIdx.x];
}

// RMSNorm rows (width 1024) written as TF32 hi / lo for the tensor-core GEMMs.
__global__ void __launch_bounds__(256) k_rmsnorm_split(const float* __restrict__ x, const float* __restrict__ g,
                                                       float* __restrict__ hi, float* __restrict__ lo) {
    __shared__ float red[8];
    const size_t row = (size_t)blockIdx.x * kDim;
    const float4 v = reinterpret_cast<const float4*>(x + row)[threadIdx.x];
    const float ss = cta_sum<256>(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w, red);
    const float inv = 1.0f / sqrtf(ss / float(kDim) + kEps);
    const float4 gv = reinterpret_cast<const float4*>(g)[threadIdx.x];
    const float4 y = make_float4(v.x * inv * gv.x, v.y * inv * gv.y, v.z * inv * gv.z, v.w * inv * gv.w);
    const float4 h = make_float4(rn_tf32(y.x), rn_tf32(y.y), rn_tf32(y.z), rn_tf32(y.w));
    reinterpret_cast<float4*>(hi + row)[threadIdx.x] = h;
    reinterpret_cast<float4*>(lo + row)[threadIdx.x] =
        make_float4(rn_tf32(y.x - h.x), rn_tf32(y.y - h.y), rn_tf32(y.z - h.z), rn_tf32(y.w - h.w));
}

// Per-head RMSNorm (q_norm / k_norm, width 128) and RoPE of token t's 16
// query heads (in place) and 8 key heads (into the K cache at position
// pos0 + t, with the token's value row into the V cache).  CTA = (t, head):
// heads 0-15 query, 16-23 key.
__global__ void __launch_bounds__(128) k_qk_norm_rope(float* __restrict__ qkv, const float* __restrict__ qn,
                                                      const float* __restrict__ kn, float* __restrict__ kc,
                                                      float* __restrict__ vc, int pos0, const State* st) {
    __shared__ float xs[kHeadDim];
    __shared__ float red[4];
    if (st) {
        if (finished(st)) return;
        pos0 = int(st->pos);
    }
    const int t = blockIdx.x, hh = blockIdx.y, d = threadIdx.x;
    const bool isq = hh < kQHeads;
    const int j = isq ? hh : hh - kQHeads;
    float* vec = qkv + (size_t)t * kQkv + (isq ? j * kHeadDim : kQDim + j * kHeadDim);
    const float x = vec[d];
    const float ss = cta_sum<128>(x * x, red);
    const float inv = 1.0f / sqrtf(ss / float(kHeadDim) + kEps);
    const float xn = x * inv * (isq ? qn : kn)[d];
    xs[d] = xn;
    __syncthreads();
    const float angle = float(pos0 + t) * c_inv_freq[d & 63];
    const float rot = d < 64 ? -xs[d + 64] : xs[d - 64];
    const float r = xn * cosf(angle) + rot * sinf(angle);
    if (isq) {
        vec[d] = r;
    } else {
        const size_t o = (size_t)(pos0 + t) * kKvDim + j * kHeadDim + d;
        kc[o] = r;
        vc[o] = qkv[(size_t)t * kQkv + kQDim + kKvDim + j * kHeadDim + d];
    }
}

// Causal GQA attention of T prompt tokens at positions pos0.. over the cache.
// CTA = (query head, 64 queries), 16 x 16 threads: thread (ty, tx) owns the
// scores of queries 4ty..+3 x keys 4tx..+3 of a 64-key tile and the outputs of
// those queries x dims 8tx..+7; online softmax per query row across tiles
// (a row's 64 scores live in one half-warp).  Output split hi / lo.
constexpr int kQLd = 68, kVLd = 132;
constexpr size_t kAttnPrefillSmem = (2 * kHeadDim * kQLd + 64 * kVLd + 64 * kQLd) * sizeof(float);

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

__global__ void __launch_bounds__(256) k_attn_prefill(const float* __restrict__ qkv, const float* __restrict__ kc,
                                                      const float* __restrict__ vc, float* __restrict__ out_hi,
                                                      float* __restrict__ out_lo, int T, int pos0) {
    extern __shared__ __align__(16) float smem[];
    float* QT = smem;                   // [128 d][kQLd]
    float* KT = QT + kHeadDim * kQLd;   // [128 d][kQLd]
    float* Vs = KT + kHeadDim * kQLd;   // [64 k][kVLd]
    float* Ps = Vs + 64 * kVLd;         // [64 q][kQLd]
    const int h = blockIdx.x, kvh = h / 2, q0 = blockIdx.y * 64, tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4, lr = tid & 63, lc = tid >> 6;
    for (int c = lc; c < kHeadDim / 4; c += 4) {
        const int q = q0 + lr, d = 4 * c;
        const float4 v = q < T ? *reinterpret_cast<const float4*>(qkv + (size_t)q * kQkv + h * kHeadDim + d)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        QT[(d + 0) * kQLd + lr] = v.x;
        QT[(d + 1) * kQLd + lr] = v.y;
        QT[(d + 2) * kQLd + lr] = v.z;
        QT[(d + 3) * kQLd + lr] = v.w;
    }
    float m[4], l[4], acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        m[a] = -INFINITY;
        l[a] = 0.f;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[a][c] = 0.f;
    }
    const int kend = pos0 + min(T, q0 + 64);  // keys that reach some query of the block
    for (int k0 = 0; k0 < kend; k0 += 64) {
        __syncthreads();
        for (int c = lc; c < kHeadDim / 4; c += 4) {
            const int key = k0 + lr, d = 4 * c;
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (key < kend) {
                const size_t o = (size_t)key * kKvDim + kvh * kHeadDim + d;
                kv = *reinterpret_cast<const float4*>(kc + o);
                vv = *reinterpret_cast<const float4*>(vc + o);
            }
            KT[(d + 0) * kQLd + lr] = kv.x;
            KT[(d + 1) * kQLd + lr] = kv.y;
            KT[(d + 2) * kQLd + lr] = kv.z;
            KT[(d + 3) * kQLd + lr] = kv.w;
            *reinterpret_cast<float4*>(Vs + lr * kVLd + d) = vv;
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) sc[a][b] = 0.f;
#pragma unroll 8
        for (int d = 0; d < kHeadDim; ++d) {
            const float4 qv = *reinterpret_cast<const float4*>(QT + d * kQLd + 4 * ty);
            const float4 kv = *reinterpret_cast<const float4*>(KT + d * kQLd + 4 * tx);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w}, kb[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) sc[a][b] = fmaf(qa[a], kb[b], sc[a][b]);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            const int qpos = pos0 + q0 + 4 * ty + a;
            float mx = -INFINITY;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int key = k0 + 4 * tx + b;
                sc[a][b] = (key <= qpos && key < kend) ? sc[a][b] * kScale : -INFINITY;
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
            *reinterpret_cast<float4*>(Ps + (4 * ty + a) * kQLd + 4 * tx) = pv;
            l[a] = l[a] * corr + half_sum(ps);
            m[a] = mn;
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[a][c] *= corr;
        }
        __syncthreads();
#pragma unroll 2
        for (int k = 0; k < 64; k += 4) {
            float4 pr[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) pr[a] = *reinterpret_cast<const float4*>(Ps + (4 * ty + a) * kQLd + k);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 v0 = *reinterpret_cast<const float4*>(Vs + (k + i) * kVLd + 8 * tx);
                const float4 v1 = *reinterpret_cast<const float4*>(Vs + (k + i) * kVLd + 8 * tx + 4);
#pragma unroll
                for (int a = 0; a < 4; ++a) {
                    const float p = i == 0 ? pr[a].x : i == 1 ? pr[a].y : i == 2 ? pr[a].z : pr[a].w;
                    acc[a][0] = fmaf(p, v0.x, acc[a][0]);
                    acc[a][1] = fmaf(p, v0.y, acc[a][1]);
                    acc[a][2] = fmaf(p, v0.z, acc[a][2]);
                    acc[a][3] = fmaf(p, v0.w, acc[a][3]);
                    acc[a][4] = fmaf(p, v1.x, acc[a][4]);
                    acc[a][5] = fmaf(p, v1.y, acc[a][5]);
                    acc[a][6] = fmaf(p, v1.z, acc[a][6]);
                    acc[a][7] = fmaf(p, v1.w, acc[a][7]);
                }
            }
        }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int q = q0 + 4 * ty + a;
        if (q >= T) continue;
        const float inv = 1.0f / l[a];
        const size_t o = (size_t)q * kQDim + h * kHeadDim + 8 * tx;
#pragma unroll
        for (int c = 0; c < 8; c += 4) {
            const float4 y =
                make_float4(acc[a][c] * inv, acc[a][c + 1] * inv, acc[a][c + 2] * inv, acc[a][c + 3] * inv);
            const float4 hv = make_float4(rn_tf32(y.x), rn_tf32(y.y), rn_tf32(y.z), rn_tf32(y.w));
            *reinterpret_cast<float4*>(out_hi + o + c) = hv;
            *reinterpret_cast<float4*>(out_lo + o + c) =
                make_float4(rn_tf32(y.x - hv.x), rn_tf32(y.y - hv.y), rn_tf32(y.z - hv.z), rn_tf32(y.w - hv.w));
        }
    }
}

// ---- decode step --------------------------------------------------------
// The decode kernels are launched with programmatic stream serialization
// (PDL): each may start while its predecessor drains, does what does not
// depend on it (the GEMVs load their weight rows), then waits for it.

// Decode attention of one step, with the q/k RMSNorm + RoPE of the step's
// token and its K/V append folded in.  A fixed grid of CTAs walks the work
// items (KV head j, chunk of 64 keys) of S = pos + 1 keys; an item computes
// for query heads 2j and 2j + 1 the chunk's max, sum of exp and exp-weighted
// V (K and V rows staged once for both heads), the chunk holding position pos
// first writes the new K/V row.  The last item of a KV head to arrive (acq_rel
// counter) merges the chunks of its two query heads in chunk order.
constexpr int kKLd = 132;
constexpr int kAttnCtas = 148;
struct AttnSmem {
    float Ks[64 * kKLd];
    float Vs[64 * kHeadDim];
    float qs[2 * kHeadDim];
    float kn[kHeadDim];
    float ps[2 * 64];
    float red[8][2];
    int last;
};

// RMSNorm (width 128, 128 threads of the calling group) and RoPE at `pos` of
// vec -> dst (shared), as k_qk_norm_rope.
__device__ __forceinline__ void norm_rope_128(const float* vec, const float* g, float* dst, float* red2, int pos,
                                              int t, int bar) {
    const float x = vec[t];
    float ss = warp_sum(x * x);
    if ((t & 31) == 0) red2[t >> 5] = ss;
    asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
    ss = red2[0] + red2[1] + red2[2] + red2[3];
    const float xn = x * (1.0f / sqrtf(ss / float(kHeadDim) + kEps)) * g[t];
    dst[t] = xn;
    asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
    const float angle = float(pos) * c_inv_freq[t & 63];
    const float rot = t < 64 ? -dst[t + 64] : dst[t - 64];
    const float r = xn * cosf(angle) + rot * sinf(angle);
    asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
    dst[t] = r;
}

__global__ void __launch_bounds__(256) k_attn_step(float* __restrict__ qkv, const float* __restrict__ qn,
                                                   const float* __restrict__ knw, float* __restrict__ kc,
                                                   float* __restrict__ vc, float* __restrict__ part,
                                                   int* __restrict__ cnt, float* __restrict__ out, const State* st) {
    extern __shared__ __align__(16) unsigned char att_raw[];
    AttnSmem& sm = *reinterpret_cast<AttnSmem*>(att_raw);
    pdl_wait();
    if (finished(st)) return;
    const int pos = int(st->pos), S = pos + 1, nch = (S + 63) / 64, items = kKvHeads * nch;
    const int tid = threadIdx.x, half = tid >> 7, t = tid & 127, lane = tid & 31, warp = tid >> 5;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
        const int j = it % kKvHeads, c = it / kKvHeads, k0 = c * 64, n = min(64, S - k0);
        // the chunk's cached K/V rows (all but position pos) go into registers
        // first, so their latency overlaps the norm / RoPE work below
        float4 kr[8], vr[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * u, r = i >> 5, c4 = i & 31;
            kr[u] = vr[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (r < n && k0 + r != pos) {
                const size_t o = (size_t)(k0 + r) * kKvDim + j * kHeadDim + 4 * c4;
                kr[u] = __ldcg(reinterpret_cast<const float4*>(kc + o));
                vr[u] = __ldcg(reinterpret_cast<const float4*>(vc + o));
            }
        }
        __syncthreads();  // the previous item's shared data is consumed
        // query heads 2j (threads 0-127) and 2j + 1 (128-255), normalised and rotated
        norm_rope_128(qkv + (2 * j + half) * kHeadDim, qn, sm.qs + half * kHeadDim, &sm.red[4 * half][0], pos, t,
                      1 + half);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = tid + 256 * u, r = i >> 5, c4 = i & 31;
            if (k0 + r == pos) continue;  // the appended row is staged below
            *reinterpret_cast<float4*>(sm.Ks + r * kKLd + 4 * c4) = kr[u];
            *reinterpret_cast<float4*>(sm.Vs + r * kHeadDim + 4 * c4) = vr[u];
        }
        if (c == nch - 1) {  // this chunk holds position pos: append the step's K/V (cache and staged row)
            const int r = pos - k0;
            if (half == 0) {
                norm_rope_128(qkv + kQDim + j * kHeadDim, knw, sm.kn, &sm.red[0][1], pos, t, 1);
                kc[(size_t)pos * kKvDim + j * kHeadDim + t] = sm.kn[t];
                sm.Ks[r * kKLd + t] = sm.kn[t];
            } else {
                const float v = qkv[kQDim + kKvDim + j * kHeadDim + t];
                vc[(size_t)pos * kKvDim + j * kHeadDim + t] = v;
                sm.Vs[r * kHeadDim + t] = v;
            }
        }
        __syncthreads();
        // scores: thread (head = half, key = t >> 1, dims (t & 1) * 64 ..)
        const int key = t >> 1, dh = (t & 1) * 64;
        float acc = 0.f;
#pragma unroll 4
        for (int d = 0; d < 64; d += 4) {
            const float4 kv = *reinterpret_cast<const float4*>(sm.Ks + key * kKLd + dh + d);
            const float4 qv = *reinterpret_cast<const float4*>(sm.qs + half * kHeadDim + dh + d);
            acc = fmaf(qv.x, kv.x, acc);
            acc = fmaf(qv.y, kv.y, acc);
            acc = fmaf(qv.z, kv.z, acc);
            acc = fmaf(qv.w, kv.w, acc);
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        const float s = key < n ? acc * kScale : -INFINITY;
        float mx = warp_max(s);
        if (lane == 0) sm.red[warp][0] = mx;
        __syncthreads();
        mx = fmaxf(fmaxf(sm.red[4 * half][0], sm.red[4 * half + 1][0]), fmaxf(sm.red[4 * half + 2][0], sm.red[4 * half + 3][0]));
        const float p = key < n ? expf(s - mx) : 0.f;
        if ((t & 1) == 0) sm.ps[half * 64 + key] = p;
        const float ls = warp_sum((t & 1) == 0 ? p : 0.f);
        if (lane == 0) sm.red[warp][1] = ls;
        __syncthreads();
        const float l = sm.red[4 * half][1] + sm.red[4 * half + 1][1] + sm.red[4 * half + 2][1] + sm.red[4 * half + 3][1];
        // four chains over keys k, k+1, k+2, k+3 (rows past n hold p = 0 and zero V)
        float o4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
        for (int k = 0; k < 64; k += 4)
#pragma unroll
            for (int u = 0; u < 4; ++u) o4[u] = fmaf(sm.ps[half * 64 + k + u], sm.Vs[(k + u) * kHeadDim + t], o4[u]);
        const float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
        float* pp = part + ((size_t)(2 * j + half) * kMaxChunks + c) * kPartStride;
        pp[2 + t] = o;
        if (t == 0) {
            pp[0] = mx;
            pp[1] = l;
        }
        // arrival per KV head; the last of its nch items merges heads 2j, 2j + 1
        // (the acq_rel add releases the partials the barrier ordered before it)
        __syncthreads();
        if (tid == 0) {
            int prev;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(cnt + j) : "memory");
            sm.last = prev == nch - 1;
            if (sm.last) cnt[j] = 0;
        }
        __syncthreads();
        if (sm.last) {  // one pass: the chunks' (max, sum) through shared memory, then the outputs
            const float* ph = part + (size_t)(2 * j + half) * kMaxChunks * kPartStride;
            float* ml = sm.Ks + half * 2 * kMaxChunks;  // the staged keys are consumed
            for (int cc = t; cc < nch; cc += 128) {
                ml[cc] = __ldcg(ph + cc * kPartStride);
                ml[kMaxChunks + cc] = __ldcg(ph + cc * kPartStride + 1);
            }
            __syncthreads();
            float M = -INFINITY;
            for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, ml[cc]);
            float L = 0.f, acco = 0.f;
            for (int cc = 0; cc < nch; ++cc) {
                const float w = expf(ml[cc] - M);
                L = fmaf(ml[kMaxChunks + cc], w, L);
                acco = fmaf(__ldcg(ph + cc * kPartStride + 2 + t), w, acco);
            }
            out[(2 * j + half) * kHeadDim + t] = acco / L;
        }
    }
    pdl_trigger();
}

// Decode GEMVs y = W x over rows of K floats, one warp per row (SwiGLU: per
// gate / up row pair), kGemvRows rows per CTA; x staged in shared memory,
// optionally RMS-normalised with gamma first (width 1024).  The weight rows
// are loaded before the wait for the predecessor.  kGemvHead (the tied head)
// also reduces the CTA's (value, index) maximum, and the last CTA to arrive
// takes the argmax over all of them (the first index of the maximum) and
// advances the State: the selected id is appended to out and becomes the next
// step's input (at the next position when `advance`); EOS or a spent budget
// ends the run.
enum GemvEpi : int { kGemvPlain = 0, kGemvResid = 1, kGemvSwiGLU = 2, kGemvHead = 3 };

template <int K, int EPI, bool NORM>
__global__ void __launch_bounds__(256) k_gemv(const float* __restrict__ W, const float* __restrict__ x,
                                              const float* __restrict__ gamma, float* __restrict__ y,
                                              float* __restrict__ best, int* __restrict__ cnt,
                                              uint32_t* __restrict__ out, State* st, int advance) {
    __shared__ __align__(16) float xs[K];
    __shared__ float red[8];
    __shared__ float bv[32];
    __shared__ uint32_t bi[32];
    __shared__ int last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int kIt = K / 128;  // float4 per lane
    constexpr int kRows = EPI == kGemvSwiGLU ? 2 : 1;
    const size_t row0 = ((size_t)blockIdx.x * kGemvRows + warp) * kRows;
    float4 wv[kRows][kIt];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        const float4* wr = reinterpret_cast<const float4*>(W + (row0 + r) * K);
#pragma unroll
        for (int i = 0; i < kIt; ++i) wv[r][i] = ld_stream(wr + lane + 32 * i);
    }
    pdl_wait();
    if (advance && finished(st)) return;
    for (int i = 4 * tid; i < K; i += 1024) *reinterpret_cast<float4*>(xs + i) = *reinterpret_cast<const float4*>(x + i);
    if (NORM) {
        static_assert(!NORM || K == kDim, "RMSNorm prologue is 1024 wide");
        __syncthreads();
        const float4 v = reinterpret_cast<const float4*>(xs)[tid];
        const float ss = cta_sum<256>(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w, red);
        const float inv = 1.0f / sqrtf(ss / float(kDim) + kEps);
        const float4 g = reinterpret_cast<const float4*>(gamma)[tid];
        reinterpret_cast<float4*>(xs)[tid] = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
    }
    __syncthreads();
    float d[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < kIt; ++i) {
            const float4 xv = reinterpret_cast<const float4*>(xs)[lane + 32 * i];
            a0 = fmaf(wv[r][i].x, xv.x, a0);
            a1 = fmaf(wv[r][i].y, xv.y, a1);
            a0 = fmaf(wv[r][i].z, xv.z, a0);
            a1 = fmaf(wv[r][i].w, xv.w, a1);
        }
        d[r] = warp_sum(a0 + a1);
    }
    pdl_trigger();
    if (EPI != kGemvHead) {
        if (lane == 0) {
            if (EPI == kGemvPlain) y[row0] = d[0];
            if (EPI == kGemvResid) y[row0] += d[0];
            if (EPI == kGemvSwiGLU) y[row0 / 2] = d[0] / (1.0f + expf(-d[0])) * d[1];
        }
        return;
    }
    if (lane == 0) {
        y[row0] = d[0];
        bv[warp] = d[0];
    }
    __syncthreads();
    if (tid == 0) {
        int b = 0;
        for (int i = 1; i < kGemvRows; ++i)
            if (bv[i] > bv[b]) b = i;
        best[2 * blockIdx.x] = bv[b];
        best[2 * blockIdx.x + 1] = __uint_as_float(uint32_t(blockIdx.x * kGemvRows + b));
        __threadfence();
        int prev;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(cnt) : "memory");
        last = prev == int(gridDim.x) - 1;
        if (last) *cnt = 0;
    }
    __syncthreads();
    if (!last) return;
    float v = -INFINITY;
    uint32_t idx = 0xffffffffu;
    for (int i = tid; i < int(gridDim.x); i += 256) {
        const float b = __ldcg(best + 2 * i);
        const uint32_t ii = __float_as_uint(__ldcg(best + 2 * i + 1));
        if (b > v || (b == v && ii < idx)) {
            v = b;
            idx = ii;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
            v = ov;
            idx = oi;
        }
    }
    if (lane == 0) {
        bv[warp] = v;
        bi[warp] = idx;
    }
    __syncthreads();
    if (tid == 0) {
        for (int i = 1; i < 8; ++i)
            if (bv[i] > v || (bv[i] == v && bi[i] < idx)) {
                v = bv[i];
                idx = bi[i];
            }
        if (idx >= uint32_t(kVocab)) idx = 0;  // no finite logit: the reference's initial index
        const uint32_t n = st->n_out;
        out[n] = idx;
        st->n_out = n + 1;
        st->token = idx;
        if (advance) st->pos += 1;
        if (idx == kEos || n + 1 >= st->max_out) st->done = 1;
    }
}

__global__ void __launch_bounds__(256) k_embed_step(const float* __restrict__ table, float* __restrict__ out,
                                                    const State* st) {
    pdl_wait();
    if (finished(st)) return;
    reinterpret_cast<float4*>(out)[threadIdx.x] = reinterpret_cast<const float4*>(table + (size_t)st->token * kDim)[threadIdx.x];
    pdl_trigger();
}

__global__ void k_interleave_rows(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ out,
                                  int rows, int cols) {
    const size_t n = (size_t)rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < 2 * n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, c = i % cols;
        out[i] = (r & 1) ? b[(r >> 1) * cols + c] : a[(r >> 1) * cols + c];
    }
}

template <int K, int EPI, bool NORM>
cudaError_t gemv(const float* W, const float* x, const float* gamma, float* y, float* best, int* cnt, uint32_t* out,
                 State* st, int advance, int rows, cudaStream_t s) {
    const int per = kGemvRows * (EPI == kGemvSwiGLU ? 2 : 1);
    return launch_pdl(k_gemv<K, EPI, NORM>, rows / per, 256, 0, s, W, x, gamma, y, best, cnt, out, st, advance);
}

float* layer_k(const Buffers& b, int layer) { return b.kv + (size_t)layer * 2 * kCap * kKvDim; }
float* layer_v(const Buffers& b, int layer) { return layer_k(b, layer) + (size_t)kCap * kKvDim; }

}  // namespace

cudaError_t init_tables() {
    float f[64];
    for (int j = 0; j < 64; ++j) f[j] = float(std::pow(1000000.0, -double(j) / 64.0));
    return cudaMemcpyToSymbol(c_inv_freq, f, sizeof f);
}

cudaError_t prepare_kernels() {
    cudaError_t e = cudaFuncSetAttribute(k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kAttnPrefillSmem);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_attn_step, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(AttnSmem));
}

cudaError_t launch_embed(const Weights& w, const Buffers& b, int T, cudaStream_t s) {
    k_embed<<<T, 256, 0, s>>>(w.embed, b.ids, b.hidden, nullptr);
    return cudaGetLastError();
}

cudaError_t launch_decode_embed(const Weights& w, const Buffers& b, cudaStream_t s) {
    return launch_pdl(k_embed_step, 1, 256, 0, s, w.embed, b.hidden, (const State*)b.st);
}

cudaError_t launch_rmsnorm_split(const float* x, const float* g, float* hi, float* lo, int T, cudaStream_t s) {
    k_rmsnorm_split<<<T, 256, 0, s>>>(x, g, hi, lo);
    return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope(const LayerW& L, const Buffers& b, int layer, int T, bool decode, cudaStream_t s) {
    k_qk_norm_rope<<<dim3(T, kQHeads + kKvHeads), 128, 0, s>>>(b.qkv, L.qn, L.kn, layer_k(b, layer),
                                                                layer_v(b, layer), 0, decode ? b.st : nullptr);
    return cudaGetLastError();
}

cudaError_t launch_attn_prefill(const Buffers& b, int layer, int T, cudaStream_t s) {
    k_attn_prefill<<<dim3(kQHeads, (T + 63) / 64), 256, kAttnPrefillSmem, s>>>(b.qkv, layer_k(b, layer),
                                                                               layer_v(b, layer), b.att_hi, b.att_lo,
                                                                               T, 0);
    return cudaGetLastError();
}

cudaError_t launch_decode_layer(const LayerW& L, const Buffers& b, int layer, cudaStream_t s) {
    cudaError_t e;
    if ((e = gemv<kDim, kGemvPlain, true>(L.w_qkv, b.hidden, L.ln1, b.qkv, nullptr, nullptr, nullptr, b.st, 1, kQkv,
                                          s)) != cudaSuccess)
        return e;
    if ((e = launch_pdl(k_attn_step, kAttnCtas, 256, sizeof(AttnSmem), s, b.qkv, L.qn, L.kn, layer_k(b, layer),
                        layer_v(b, layer), b.part, b.cnt, b.att_hi, (const State*)b.st)) != cudaSuccess)
        return e;
    if ((e = gemv<kQDim, kGemvResid, false>(L.w_o, b.att_hi, nullptr, b.hidden, nullptr, nullptr, nullptr, b.st, 1,
                                            kDim, s)) != cudaSuccess)
        return e;
    if ((e = gemv<kDim, kGemvSwiGLU, true>(L.w_gu, b.hidden, L.ln2, b.gu_hi, nullptr, nullptr, nullptr, b.st, 1,
                                           2 * kFfn, s)) != cudaSuccess)
        return e;
    return gemv<kFfn, kGemvResid, false>(L.w_down, b.gu_hi, nullptr, b.hidden, nullptr, nullptr, nullptr, b.st, 1,
                                         kDim, s);
}

// Final RMSNorm of `last_row` fused into the tied head; its last CTA takes the
// argmax and sets the State (a decode step also moves its position on; after
// a prefill the host has set the position to the prompt's length).
cudaError_t launch_head(const Weights& w, const Buffers& b, const float* last_row, bool decode, cudaStream_t s) {
    return gemv<kDim, kGemvHead, true>(w.embed, last_row, w.norm, b.logits, b.best, b.cnt + kKvHeads, b.out, b.st,
                                       decode ? 1 : 0, kVocab, s);
}

cudaError_t launch_interleave_rows(const float* a, const float* b, float* out, int rows, int cols, cudaStream_t s) {
    k_interleave_rows<<<1184, 256, 0, s>>>(a, b, out, rows, cols);
    return cudaGetLastError();
}

}  // namespace qwen
}  // namespace itts
