// Batch-1 decode step of the IndexTTS 2.5 GPT on B200 (sm_100a).
//
// One decode step (src/gpt.cpp:88-125 with initial=false) is five phases per
// layer plus the head:
//   A  LN1 (+ token embedding at layer 0) fused into the QKV GEMV   [3840 x 1280]
//   B  split-K attention over the KV cache with the K/V append     (20 heads)
//   C  c_proj GEMV + bias + residual                              [1280 x 1280]
//   D  LN2 fused into the c_fc GEMV + bias + tanh-GELU             [5120 x 1280]
//   E  mlp.c_proj GEMV + bias + residual                          [1280 x 5120]
//   F  ln_f, final_norm and the mel_head GEMV                      [8194 x 1280]
// Every phase is a function of (cta, ncta) over the whole grid.  Two drivers
// run them:
//   * k_decode_persistent: one cooperative launch of one 512-thread CTA per SM
//     for a whole token loop; phases are separated by a grid barrier (bounded
//     spin on an L2 counter), the sampler runs redundantly in every CTA so the
//     next token needs no extra barrier, and the next step's embedding is
//     computed locally.
//   * the layered path: one launch per phase (same device code), used for
//     diagnosis and as the non-cooperative fallback.
// The decode is HBM-bound: every GEMV streams its weight rows once per step
// with 128-bit evict-first loads, ~80 KB in flight per SM; activations
// (<= 32 KB) stay in L2 and are read with L2-only loads because other SMs
// wrote them in the previous phase.
#include <cooperative_groups.h>

#include "common.cuh"
#include "model.hpp"
#include "sampler.cuh"

namespace itts {

struct PhaseSmem {
    float red[32];
    float red2[64];
    float q[kHeadDim];
    float p[kThreads];
    float pv[8][kHeadDim];
    int flag;
    int abort;
};

struct DecodeSmem {
    PhaseSmem ph;
    SamplerSmem sa;
};

// Rotating owner of row r in phase `phase` of `layer`: spreads the remainder
// rows of R % ncta over different CTAs from phase to phase.
__device__ __forceinline__ int row_rot(int layer, int phase, int ncta) { return (layer * 6 + phase) * 29 % ncta; }

// x (length C) -> registers: thread (group-local index tig) holds float4 slots
// tig + j * GW * 32, j < NJ.  Activations come from L2 (written by other SMs).
template <int C, int GW>
__device__ __forceinline__ void load_x(const float* x, float4 (&xr)[C / (GW * 128)]) {
    constexpr int NJ = C / (GW * 128), GT = GW * 32;
    const int tig = threadIdx.x % GT;
    const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll
    for (int j = 0; j < NJ; ++j) xr[j] = __ldcg(x4 + tig + j * GT);
}

// LayerNorm of the 1280-vector held by the first 64 threads (GEMV layout
// <1280, 2>); every thread normalises its own 20 values.  Two-pass mean and
// centred variance as mit2_layernorm_f32_rows (kernels.metal:618-669).
__device__ __forceinline__ void layernorm_x(float4 (&xr)[5], const float* __restrict__ g,
                                            const float* __restrict__ b, float* red) {
    const bool owner = threadIdx.x < 64;
    float s = 0.f;
    if (owner) {
#pragma unroll
        for (int j = 0; j < 5; ++j) s += (xr[j].x + xr[j].y) + (xr[j].z + xr[j].w);
    }
    const float mean = block_sum(s, red) * (1.0f / kWidth);
    float v = 0.f;
    if (owner) {
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const float a = xr[j].x - mean, bb = xr[j].y - mean, c = xr[j].z - mean, d = xr[j].w - mean;
            v = fmaf(a, a, v);
            v = fmaf(bb, bb, v);
            v = fmaf(c, c, v);
            v = fmaf(d, d, v);
        }
    }
    const float var = block_sum(v, red) * (1.0f / kWidth);
    const float inv = 1.0f / sqrtf(var + kLnEps);
    const int tig = threadIdx.x & 63;
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        const float4 gg = __ldg(g4 + tig + 64 * j), bb = __ldg(b4 + tig + 64 * j);
        xr[j].x = (xr[j].x - mean) * inv * gg.x + bb.x;
        xr[j].y = (xr[j].y - mean) * inv * gg.y + bb.y;
        xr[j].z = (xr[j].z - mean) * inv * gg.z + bb.z;
        xr[j].w = (xr[j].w - mean) * inv * gg.w + bb.w;
    }
}

// y[r] = W[r, :] . x for the rows this CTA owns (r with (r + rot) % ncta == cta).
// GW warps share one row (GW = 2 for 1280 columns, 8 for 5120), each lane
// holding NJ = 5 float4 of x; two rows per group are in flight per iteration.
template <int C, int GW, class Epi>
__device__ __forceinline__ void gemv_rows(const float* __restrict__ Wm, int R, const float4 (&xr)[C / (GW * 128)],
                                          int cta, int ncta, int rot, float* red, Epi epi) {
    constexpr int NJ = C / (GW * 128), GROUPS = kWarps / GW, GT = GW * 32, U = 2;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = warp / GW, tig = threadIdx.x % GT;
    int first = (cta - rot) % ncta;
    if (first < 0) first += ncta;
    const int nr = first < R ? (R - 1 - first) / ncta + 1 : 0;
    for (int base = 0; base < nr; base += GROUPS * U) {
        float4 w[U][NJ];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int li = base + u * GROUPS + g;
            if (li < nr) {
                const float4* wr = reinterpret_cast<const float4*>(Wm + (size_t)(first + li * ncta) * C) + tig;
#pragma unroll
                for (int j = 0; j < NJ; ++j) w[u][j] = ld_stream(wr + j * GT);
            } else {
#pragma unroll
                for (int j = 0; j < NJ; ++j) w[u][j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        float acc[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            acc[u] = 0.f;
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[u] = dot4(w[u][j], xr[j], acc[u]);
            acc[u] = warp_sum(acc[u]);
        }
        if (lane == 0) {
#pragma unroll
            for (int u = 0; u < U; ++u) red[warp * U + u] = acc[u];
        }
        __syncthreads();
        if ((warp % GW) == 0 && lane < U) {
            const int li = base + lane * GROUPS + g;
            if (li < nr) {
                float s = 0.f;
#pragma unroll
                for (int k = 0; k < GW; ++k) s += red[(warp + k) * U + lane];
                epi(first + li * ncta, s);
            }
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- phases
__device__ void phase_qkv(const DecodeArgs& a, const LayerW& L, int layer, uint32_t token, uint32_t pos, int cta,
                          int ncta, PhaseSmem& sm) {
    float4 xr[5];
    if (layer == 0) {
        // gpt_build_current: x = mel_embedding[code] + mel_pos_embedding[pos]
        const int tig = threadIdx.x & 63;
        const float4* me = reinterpret_cast<const float4*>(a.w->mel_emb + (size_t)token * kWidth);
        const float4* mp = reinterpret_cast<const float4*>(a.w->mel_pos + (size_t)pos * kWidth);
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const float4 e = __ldg(me + tig + 64 * j), p = __ldg(mp + tig + 64 * j);
            xr[j] = make_float4(e.x + p.x, e.y + p.y, e.z + p.z, e.w + p.w);
        }
        if (cta == 0 && threadIdx.x < 64) {
            float4* h4 = reinterpret_cast<float4*>(a.b.h);
#pragma unroll
            for (int j = 0; j < 5; ++j) h4[tig + 64 * j] = xr[j];
        }
    } else {
        load_x<kWidth, 2>(a.b.h, xr);
    }
    layernorm_x(xr, L.ln1_g, L.ln1_b, sm.red);
    float* out = a.b.qkv;
    const float* bias = L.b_qkv;
    gemv_rows<kWidth, 2>(L.w_qkv, kQkv, xr, cta, ncta, row_rot(layer, 0, ncta), sm.red2,
                         [&](int r, float acc) { out[r] = acc + __ldg(bias + r); });
}

// Split-K attention for one query over keys [0, S] (S cached + the current
// key from qkv), restating mit2_gpt_cached_attention_resident_f32
// (kernels.metal:2064-2145).  Work unit = (head, chunk of ch keys); one CTA
// per unit, one thread per key for the scores; the chunk partials (max, sum,
// 64 outputs) are merged by the last CTA to finish the head.  The unit that
// holds key S appends this token's K/V to the cache.
__device__ void phase_attn(const DecodeArgs& a, int layer, uint32_t S, int cta, int ncta, PhaseSmem& sm) {
    const uint32_t keys = S + 1;
    uint32_t ch = (keys * kHeads + ncta - 1) / ncta;
    ch = (ch + 31u) & ~31u;
    ch = min(max(ch, 32u), (uint32_t)kThreads);
    const uint32_t nch = (keys + ch - 1) / ch, units = kHeads * nch;
    const int t = threadIdx.x;
    for (uint32_t u = cta; u < units; u += ncta) {
        const uint32_t h = u / nch, c = u % nch, k0 = c * ch, k1 = min(k0 + ch, keys);
        float* Kc = a.b.kv + (((size_t)layer * 2 + 0) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
        float* Vc = a.b.kv + (((size_t)layer * 2 + 1) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
        const float* kcur = a.b.qkv + kWidth + h * kHeadDim;
        const float* vcur = a.b.qkv + 2 * kWidth + h * kHeadDim;
        if (t < kHeadDim) sm.q[t] = __ldcg(a.b.qkv + h * kHeadDim + t);
        __syncthreads();
        const uint32_t key = k0 + t;
        float s = -INFINITY;
        if (key < k1) {
            const float4* kr = reinterpret_cast<const float4*>(key < S ? Kc + (size_t)key * kHeadDim : kcur);
            const float4* q4 = reinterpret_cast<const float4*>(sm.q);
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < kHeadDim / 4; ++i) acc = dot4(__ldcg(kr + i), q4[i], acc);
            s = acc * 0.125f;  // rsqrt(64)
        }
        const float m = block_max(s, sm.red);
        const float p = key < k1 ? expf(s - m) : 0.f;
        sm.p[t] = p;
        const float l = block_sum(p, sm.red);
        const int d = t & 63, grp = t >> 6;
        float o = 0.f;
        const uint32_t n = k1 - k0;
#pragma unroll 4
        for (uint32_t j = grp; j < n; j += 8) {
            const uint32_t kk = k0 + j;
            const float v = kk < S ? __ldcg(Vc + (size_t)kk * kHeadDim + d) : __ldcg(vcur + d);
            o = fmaf(sm.p[j], v, o);
        }
        sm.pv[grp][d] = o;
        __syncthreads();
        float tot = 0.f;
        if (t < kHeadDim) {
#pragma unroll
            for (int g2 = 0; g2 < 8; ++g2) tot += sm.pv[g2][t];
        }
        if (nch == 1) {
            if (t < kHeadDim) a.b.attn[h * kHeadDim + t] = tot / l;
        } else {
            float* pp = a.b.part + ((size_t)h * nch + c) * 66;
            if (t < kHeadDim) pp[2 + t] = tot;
            if (t == 0) {
                pp[0] = m;
                pp[1] = l;
            }
            __threadfence();
            __syncthreads();
            if (t == 0) sm.flag = atomicAdd(&a.b.ctl->head_cnt[h], 1u) == nch - 1;
            __syncthreads();
            if (sm.flag) {
                __threadfence();
                if (t < kHeadDim) {
                    const float* ph = a.b.part + (size_t)h * nch * 66;
                    float M = -INFINITY;
                    for (uint32_t cc = 0; cc < nch; ++cc) M = fmaxf(M, __ldcg(ph + cc * 66));
                    float Ls = 0.f, O = 0.f;
                    for (uint32_t cc = 0; cc < nch; ++cc) {
                        const float w = expf(__ldcg(ph + cc * 66) - M);
                        Ls = fmaf(w, __ldcg(ph + cc * 66 + 1), Ls);
                        O = fmaf(w, __ldcg(ph + cc * 66 + 2 + t), O);
                    }
                    a.b.attn[h * kHeadDim + t] = O / Ls;
                }
                if (t == 0) atomicExch(&a.b.ctl->head_cnt[h], 0u);
            }
        }
        if (c == nch - 1) {
            if (t < kHeadDim)
                Kc[(size_t)S * kHeadDim + t] = __ldcg(kcur + t);
            else if (t < 2 * kHeadDim)
                Vc[(size_t)S * kHeadDim + t - kHeadDim] = __ldcg(vcur + t - kHeadDim);
        }
        __syncthreads();
    }
}

__device__ void phase_oproj(const DecodeArgs& a, const LayerW& L, int layer, int cta, int ncta, PhaseSmem& sm) {
    float4 xr[5];
    load_x<kWidth, 2>(a.b.attn, xr);
    float* out = a.b.r;
    const float* res = a.b.h;
    const float* bias = L.b_o;
    gemv_rows<kWidth, 2>(L.w_o, kWidth, xr, cta, ncta, row_rot(layer, 2, ncta), sm.red2,
                         [&](int r, float acc) { out[r] = __ldcg(res + r) + (acc + __ldg(bias + r)); });
}

__device__ void phase_fc(const DecodeArgs& a, const LayerW& L, int layer, int cta, int ncta, PhaseSmem& sm) {
    float4 xr[5];
    load_x<kWidth, 2>(a.b.r, xr);
    layernorm_x(xr, L.ln2_g, L.ln2_b, sm.red);
    float* out = a.b.ff;
    const float* bias = L.b_fc;
    gemv_rows<kWidth, 2>(L.w_fc, kFfn, xr, cta, ncta, row_rot(layer, 3, ncta), sm.red2,
                         [&](int r, float acc) { out[r] = gelu_ref(acc + __ldg(bias + r)); });
}

__device__ void phase_mproj(const DecodeArgs& a, const LayerW& L, int layer, int cta, int ncta, PhaseSmem& sm) {
    float4 xr[5];
    load_x<kFfn, 8>(a.b.ff, xr);
    float* out = a.b.h;
    const float* res = a.b.r;
    const float* bias = L.b_mp;
    gemv_rows<kFfn, 8>(L.w_mp, kWidth, xr, cta, ncta, row_rot(layer, 4, ncta), sm.red2,
                       [&](int r, float acc) { out[r] = __ldcg(res + r) + (acc + __ldg(bias + r)); });
}

// gpt.cpp:120-122: last hidden row -> ln_f -> final_norm -> mel_head.
__device__ void phase_head(const DecodeArgs& a, int cta, int ncta, PhaseSmem& sm) {
    float4 xr[5];
    load_x<kWidth, 2>(a.b.h, xr);
    layernorm_x(xr, a.w->lnf_g, a.w->lnf_b, sm.red);
    layernorm_x(xr, a.w->fn_g, a.w->fn_b, sm.red);
    float* out = a.b.logits;
    const float* bias = a.w->b_head;
    gemv_rows<kWidth, 2>(a.w->w_head, kVocab, xr, cta, ncta, row_rot(0, 5, ncta), sm.red2,
                         [&](int r, float acc) { out[r] = acc + __ldg(bias + r); });
}

// Grid barrier for the persistent kernel (all CTAs co-resident by the
// cooperative launch).  Monotonic arrival counter, bounded spin; returns true
// when the kernel must abort (a CTA reported an error or the wait timed out).
__device__ __forceinline__ bool grid_barrier(const DecodeArgs& a, unsigned& target, int where, PhaseSmem& sm) {
    target += gridDim.x;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* bar = &a.b.ctl->bar;
        int* status = a.b.ctl->status;
        __threadfence();
        atomicAdd(bar, 1u);
        const unsigned long long t0 = globaltimer_ns();
        unsigned spins = 0;
        while (ld_acquire_gpu(bar) < target) {
            if ((++spins & 31u) == 0) {
                if (ld_volatile(status) != 0) break;
                if (globaltimer_ns() - t0 > kWaitLimitNs) {
                    set_status(status, kStatusBarrierTimeout, where, (int)target);
                    break;
                }
            }
        }
        __threadfence();
        sm.abort = ld_volatile(status) != 0;
    }
    __syncthreads();
    return sm.abort != 0;
}

__device__ bool forward_step(const DecodeArgs& a, uint32_t token, uint32_t pos, uint32_t S, int cta, int ncta,
                             PhaseSmem& sm, unsigned& target) {
    const int layers = a.w->layers;
    for (int l = 0; l < layers; ++l) {
        const LayerW& L = a.w->layer[l];
        phase_qkv(a, L, l, token, pos, cta, ncta, sm);
        if (grid_barrier(a, target, l * 8 + 0, sm)) return true;
        phase_attn(a, l, S, cta, ncta, sm);
        if (grid_barrier(a, target, l * 8 + 1, sm)) return true;
        phase_oproj(a, L, l, cta, ncta, sm);
        if (grid_barrier(a, target, l * 8 + 2, sm)) return true;
        phase_fc(a, L, l, cta, ncta, sm);
        if (grid_barrier(a, target, l * 8 + 3, sm)) return true;
        phase_mproj(a, L, l, cta, ncta, sm);
        if (grid_barrier(a, target, l * 8 + 4, sm)) return true;
    }
    phase_head(a, cta, ncta, sm);
    return grid_barrier(a, target, 1000, sm);
}

__global__ void __launch_bounds__(kThreads, 1) k_decode_persistent(DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
    const int cta = blockIdx.x, ncta = gridDim.x;
    unsigned target = 0;
    if (threadIdx.x == 0) sm.ph.abort = 0;
    sampler_init_seen(sm.sa, a.history, a.history_n);
    uint32_t token = a.first_code, n_codes = 0, stopped = 0, fwd = 0;
    for (uint32_t i = 0; i < a.n_iter; ++i) {
        if (a.mode == kModeGenerate) {
            token = run_sampler(a.b.logits, a.opts, i, a.opts.do_sample == 0, sm.sa, nullptr, a.b.ctl->status);
            if (token == (uint32_t)kStopCode) {
                stopped = 1;
                break;
            }
            if (token >= (uint32_t)kStartCode) {
                if (token != 0xffffffffu && threadIdx.x == 0)
                    set_status(a.b.ctl->status, kStatusInvalidCode, 200, (int)token);
                break;
            }
            if (cta == 0 && threadIdx.x == 0) a.codes[i] = token;
            ++n_codes;
            sampler_mark_seen(sm.sa, token);
            if (i + 1 == a.n_iter) break;
        }
        if (forward_step(a, token, a.pos0 + i, a.s0 + i, cta, ncta, sm.ph, target)) break;
        ++fwd;
    }
    if (cta == 0 && threadIdx.x == 0) {
        DecodeCtl* ctl = a.b.ctl;
        ctl->info[0] = n_codes;
        ctl->info[1] = stopped;
        ctl->info[2] = (uint32_t)ld_volatile(ctl->status);
        ctl->info[3] = fwd;
        if (a.info_out) {
            for (int i = 0; i < 4; ++i) a.info_out[i] = ctl->info[i];
        }
    }
}

// ------------------------------------------------------------ layered path
enum LayerPhase : int { kPhQkv = 0, kPhAttn, kPhOproj, kPhFc, kPhMproj, kPhHead };

__global__ void __launch_bounds__(kThreads, 1) k_phase(DecodeArgs a, int phase, int layer, uint32_t pos, uint32_t S) {
    __shared__ PhaseSmem sm;
    if (ld_volatile(&a.b.ctl->done)) return;
    const int cta = blockIdx.x, ncta = gridDim.x;
    const uint32_t token = *reinterpret_cast<volatile uint32_t*>(&a.b.ctl->token);
    switch (phase) {
        case kPhQkv: phase_qkv(a, a.w->layer[layer], layer, token, pos, cta, ncta, sm); break;
        case kPhAttn: phase_attn(a, layer, S, cta, ncta, sm); break;
        case kPhOproj: phase_oproj(a, a.w->layer[layer], layer, cta, ncta, sm); break;
        case kPhFc: phase_fc(a, a.w->layer[layer], layer, cta, ncta, sm); break;
        case kPhMproj: phase_mproj(a, a.w->layer[layer], layer, cta, ncta, sm); break;
        default: phase_head(a, cta, ncta, sm); break;
    }
}

// One CTA: selects code i of the layered generate loop (or installs the input
// code for a single step) and updates ctl->{token, done, info}.
__global__ void __launch_bounds__(kThreads, 1) k_layer_sample(DecodeArgs a, uint32_t i) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    DecodeCtl* ctl = a.b.ctl;
    if (ld_volatile(&ctl->done)) return;
    if (a.mode != kModeGenerate) {
        if (threadIdx.x == 0) ctl->token = a.first_code;
        return;
    }
    sampler_init_seen(sm, a.history, a.history_n);
    for (uint32_t k = threadIdx.x; k < i; k += blockDim.x) {
        const uint32_t t = a.codes[k];
        atomicOr(&sm.seen[t >> 5], 1u << (t & 31));
    }
    __syncthreads();
    const uint32_t token = run_sampler(a.b.logits, a.opts, i, a.opts.do_sample == 0, sm, nullptr, ctl->status);
    if (threadIdx.x != 0) return;
    bool finish = false;
    if (token == (uint32_t)kStopCode) {
        ctl->info[1] = 1;
        finish = true;
    } else if (token >= (uint32_t)kStartCode) {
        if (token != 0xffffffffu) set_status(ctl->status, kStatusInvalidCode, 200, (int)token);
        finish = true;
    } else {
        a.codes[i] = token;
        ctl->info[0] = i + 1;
        ctl->token = token;
        if (i + 1 == a.n_iter)
            finish = true;
        else
            ctl->info[3] = ctl->info[3] + 1;
    }
    if (finish) {
        ctl->done = 1;
        ctl->info[2] = (uint32_t)ctl->status[0];
        if (a.info_out)
            for (int k = 0; k < 4; ++k) a.info_out[k] = ctl->info[k];
    }
}

__global__ void k_layer_finish(DecodeArgs a) {
    DecodeCtl* ctl = a.b.ctl;
    if (a.mode != kModeGenerate) {
        ctl->info[3] = 1;
        ctl->info[2] = (uint32_t)ctl->status[0];
    }
    if (a.info_out)
        for (int k = 0; k < 4; ++k) a.info_out[k] = ctl->info[k];
}

__global__ void __launch_bounds__(kThreads, 1) k_processors(const float* logits, SampleOpts o, const uint32_t* hist,
                                                            uint32_t hist_n, float* out, int* status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    sampler_init_seen(sm, hist, hist_n);
    run_sampler(logits, o, 0, false, sm, out, status);
}

// Beam search, one parent (gpt_sampling.cpp:206-214): float log-softmax of
// the parent's logits, the processors with num_beams > 1 semantics, plus the
// parent's cumulative score.  One CTA.
__global__ void __launch_bounds__(kThreads, 1) k_beam_scores(const float* logits, SampleOpts o, const uint32_t* hist,
                                                             uint32_t hist_n, float beam_score, float* tmp, float* out,
                                                             int* status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    sampler_init_seen(sm, hist, hist_n);
    const int base = threadIdx.x * kPer, cnt = max(0, min(kPer, kVocab - base));
    float v[kPer];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
        v[k] = k < cnt ? __ldcg(logits + base + k) : -INFINITY;
        mx = fmaxf(mx, v[k]);
    }
    const float peak = block_max(mx, sm.redf);
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt) s += expf(v[k] - peak);
    const float sum = block_sum(s, sm.redf);
    const float log_sum = peak + logf(sum);
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt) tmp[base + k] = v[k] - log_sum;
    __threadfence();
    __syncthreads();
    run_sampler(tmp, o, 0, false, sm, out, status);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt) out[base + k] = out[base + k] + beam_score;
}

// ------------------------------------------------------------ host side
size_t decode_smem_bytes() { return sizeof(DecodeSmem); }

cudaError_t decode_configure(int* blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(k_decode_persistent, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(DecodeSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_layer_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SamplerSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_processors, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SamplerSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_beam_scores, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SamplerSmem));
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k_decode_persistent, kThreads,
                                                         sizeof(DecodeSmem));
}

cudaError_t launch_decode_persistent(const DecodeArgs& a, int ncta, cudaStream_t s) {
    DecodeArgs copy = a;
    void* args[] = {&copy};
    return cudaLaunchCooperativeKernel((const void*)k_decode_persistent, dim3(ncta), dim3(kThreads), args,
                                       sizeof(DecodeSmem), s);
}

cudaError_t launch_decode_layered(const DecodeArgs& a, int layers, int ncta, cudaStream_t s, uint64_t* launches) {
    for (uint32_t i = 0; i < a.n_iter; ++i) {
        k_layer_sample<<<1, kThreads, sizeof(SamplerSmem), s>>>(a, i);
        ++*launches;
        if (a.mode == kModeGenerate && i + 1 == a.n_iter) break;
        const uint32_t pos = a.pos0 + i, S = a.s0 + i;
        for (int l = 0; l < layers; ++l)
            for (int ph = kPhQkv; ph <= kPhMproj; ++ph) {
                k_phase<<<ncta, kThreads, 0, s>>>(a, ph, l, pos, S);
                ++*launches;
            }
        k_phase<<<ncta, kThreads, 0, s>>>(a, kPhHead, 0, pos, S);
        ++*launches;
    }
    k_layer_finish<<<1, 1, 0, s>>>(a);
    ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_head(const DecodeArgs& a, int ncta, cudaStream_t s) {
    k_phase<<<ncta, kThreads, 0, s>>>(a, kPhHead, 0, 0, 0);
    return cudaGetLastError();
}

cudaError_t launch_processors(const float* logits, const SampleOpts& o, const uint32_t* hist, uint32_t hist_n,
                              float* out, int* status, cudaStream_t s) {
    k_processors<<<1, kThreads, sizeof(SamplerSmem), s>>>(logits, o, hist, hist_n, out, status);
    return cudaGetLastError();
}

cudaError_t launch_beam_scores(const float* logits, const SampleOpts& o, const uint32_t* hist, uint32_t hist_n,
                               float beam_score, float* tmp, float* out, int* status, cudaStream_t s) {
    k_beam_scores<<<1, kThreads, sizeof(SamplerSmem), s>>>(logits, o, hist, hist_n, beam_score, tmp, out, status);
    return cudaGetLastError();
}

}  // namespace itts
