// Batch-1 decode of the IndexTTS 2.5 GPT on B200 (sm_100a).
//
// One decode step (src/gpt.cpp:88-125 with initial=false) is four phases per
// layer plus the head, each a function of (cta, ncta) over the whole grid:
//   A    h -> LN1 -> QKV GEMV (rows of [3840 x 1280])
//   B    split-K attention over the KV cache + K/V append (kernels.metal:2064-2145)
//   C    merge of the attention partials -> c_proj GEMV + bias + residual -> r
//   MLP  r -> LN2 -> c_fc GEMV + GELU (this CTA's 5120/ncta rows) -> their share
//        of mlp.c_proj as a split-K product over those rows (mlp.c_proj kept
//        in its [in, out] layout), summed across CTAs with 64-bit fixed-point
//        atomics (order independent, hence deterministic)
//   head ln_f -> final_norm -> mel_head GEMV
// The next layer's h = r + (mlp + bias) is rebuilt from r and the fixed-point
// sums by every CTA that needs it, so the step has 4 grid-wide dependencies per
// layer instead of 6.
//
// Weight streaming: every CTA owns a contiguous block of rows per matrix.  Its
// rows (and the LayerNorm vectors) are fetched into a 10-slot x 20 KB shared-
// memory ring with cp.async.bulk (1-D TMA, completion on a "full" mbarrier;
// no multicast) by a dedicated producer warp that runs up to ten slots ahead of
// the 16 consumer warps (a consumed slot is handed back on an "empty"
// mbarrier) and issues cp.async.bulk.prefetch.L2 ten slots further ahead.  The
// stream therefore runs through grid barriers, the attention phase and the
// sampler, which are the latency-bound parts of the step; the consumers read
// weights from shared memory and synchronise on a named barrier the producer
// never joins.  Attention reads K/V directly (L2-coherent loads): one warp per key
// subset with an online softmax, K and V fetched together.
//
// Drivers:
//   * k_decode: one cooperative launch (one 512-thread CTA per SM) for a whole
//     token loop; grid barriers (bounded spin on an L2 counter) between phases;
//     the sampler runs redundantly in every CTA so the next token needs no
//     extra barrier.
//   * k_phase: one launch per phase with the same device code (layered mode,
//     for diagnosis and as the non-cooperative path); its ring covers only that
//     phase.
#include "common.cuh"
#include "model.hpp"
#include "sampler.cuh"

namespace itts {

// ------------------------------------------------------------ weight ring
constexpr int kRowBytes = kWidth * 4;              // every streamed row has 1280 fp32
constexpr int kRowsPerSlot = 4;
constexpr int kSlotBytes = kRowsPerSlot * kRowBytes;  // 20 KB
constexpr int kSlots = 10;
constexpr int kPfSlots = 12;

enum Seg : int { kSegLn1 = 0, kSegQkv, kSegO, kSegLn2, kSegFc, kSegMp, kSegFinalLn, kSegHead };

struct Cursor {
    int step, layer, seg;
    uint32_t off, budget;
};

struct SlotDesc {
    const char* src[4];
    uint32_t bytes[4];
    int n;
    uint32_t total;
};

struct Ring {
    __align__(128) unsigned char data[kSlots][kSlotBytes];
    unsigned long long full[kSlots];
    unsigned long long empty[kSlots];
    volatile uint32_t issued;  // slots issued by the producer
    volatile int stop;         // consumers are done: the producer must quit
    volatile int producer_done;
};

// This CTA's contiguous row block of each streamed matrix.
struct Rows {
    int q0, q1, o0, o1, f0, f1, h0, h1;
};

__device__ __forceinline__ Rows cta_rows(int cta, int ncta) {
    Rows r;
    r.q0 = int((long long)kQkv * cta / ncta);
    r.q1 = int((long long)kQkv * (cta + 1) / ncta);
    r.o0 = int((long long)kWidth * cta / ncta);
    r.o1 = int((long long)kWidth * (cta + 1) / ncta);
    r.f0 = int((long long)kFfn * cta / ncta);
    r.f1 = int((long long)kFfn * (cta + 1) / ncta);
    r.h0 = int((long long)kVocab * cta / ncta);
    r.h1 = int((long long)kVocab * (cta + 1) / ncta);
    return r;
}

struct PhaseSmem {
    float red[32];
    float red2[2][32];
    float bias[64];
    float res[64];
    float f[64];
    __align__(16) float attn[kWidth];
    float wm[kWarps], wl[kWarps];
    float wo[kWarps][kHeadDim];
    int abort;
};

struct DecodeSmem {
    Ring ring;
    PhaseSmem ph;
    SamplerSmem sa;
    ModelW w;  // the weight pointer table, read at every slot and phase start
};

// All threads: copy the weight pointer table into shared memory.
__device__ __forceinline__ void load_table(ModelW& dst, const ModelW* src) {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    uint32_t* d = reinterpret_cast<uint32_t*>(&dst);
    for (uint32_t i = threadIdx.x; i < sizeof(ModelW) / 4; i += blockDim.x) d[i] = __ldg(s + i);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Bounded wait for a ring slot; every thread waits.  The spin touches no
// global memory for the first kStatusPollNs (a global load costs a full L2
// round trip and would delay noticing the slot); after that it also watches
// the status word so that an error elsewhere ends the wait.  False on timeout
// or error.
constexpr unsigned long long kStatusPollNs = 200000ull;

__device__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity, int* status, int where) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            const unsigned long long dt = globaltimer_ns() - t0;
            if (dt > kStatusPollNs && ld_volatile(status) != 0) return false;
            if (dt > kWaitLimitNs) {
                set_status(status, kStatusRingTimeout, where, (int)i);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void advance_seg(Cursor& c, int layers) {
    if (c.seg == kSegMp) {
        ++c.layer;
        c.seg = c.layer == layers ? kSegFinalLn : kSegLn1;
    } else {
        ++c.seg;
    }
}

// The weight schedule of one CTA: per forward step, per layer: LN1 vectors,
// its QKV rows, its c_proj rows, LN2 vectors, its c_fc rows, its mlp.c_proj
// [in, out] rows; then the final LN vectors and its mel_head rows.  Row blocks
// are cut into 4-row slots.
__device__ bool next_slot(const ModelW& w, const Rows& rows, int n_steps, Cursor& c, SlotDesc& d) {
    while (c.budget > 0 && c.step < n_steps) {
        d.n = 0;
        if (c.seg == kSegLn1 || c.seg == kSegLn2) {
            const LayerW& lw = w.layer[c.layer];
            d.src[0] = reinterpret_cast<const char*>(c.seg == kSegLn1 ? lw.ln1_g : lw.ln2_g);
            d.src[1] = reinterpret_cast<const char*>(c.seg == kSegLn1 ? lw.ln1_b : lw.ln2_b);
            d.bytes[0] = d.bytes[1] = kRowBytes;
            d.n = 2;
            d.total = 2 * kRowBytes;
            advance_seg(c, w.layers);
            --c.budget;
            return true;
        }
        if (c.seg == kSegFinalLn) {
            const float* v[4] = {w.lnf_g, w.lnf_b, w.fn_g, w.fn_b};
            for (int i = 0; i < 4; ++i) {
                d.src[i] = reinterpret_cast<const char*>(v[i]);
                d.bytes[i] = kRowBytes;
            }
            d.n = 4;
            d.total = 4 * kRowBytes;
            c.seg = kSegHead;
            --c.budget;
            return true;
        }
        const float* base;
        int r0, r1;
        if (c.seg == kSegHead) {
            base = w.w_head;
            r0 = rows.h0;
            r1 = rows.h1;
        } else {
            const LayerW& lw = w.layer[c.layer];
            if (c.seg == kSegQkv) {
                base = lw.w_qkv;
                r0 = rows.q0;
                r1 = rows.q1;
            } else if (c.seg == kSegO) {
                base = lw.w_o;
                r0 = rows.o0;
                r1 = rows.o1;
            } else {
                base = c.seg == kSegFc ? lw.w_fc : lw.w_mpT;
                r0 = rows.f0;
                r1 = rows.f1;
            }
        }
        const uint32_t total = uint32_t(r1 - r0) * kRowBytes;
        if (c.off < total) {
            const uint32_t chunk = min(total - c.off, (uint32_t)kSlotBytes);
            d.src[0] = reinterpret_cast<const char*>(base + (size_t)r0 * kWidth) + c.off;
            d.bytes[0] = chunk;
            d.n = 1;
            d.total = chunk;
            c.off += chunk;
            if (c.off >= total) {
                c.off = 0;
                if (c.seg == kSegHead) {
                    ++c.step;
                    c.layer = 0;
                    c.seg = kSegLn1;
                } else {
                    advance_seg(c, w.layers);
                }
            }
            --c.budget;
            return true;
        }
        c.off = 0;
        if (c.seg == kSegHead) {
            ++c.step;
            c.layer = 0;
            c.seg = kSegLn1;
        } else {
            advance_seg(c, w.layers);
        }
    }
    return false;
}

// Producer warp (lane 0): walks the schedule, waits for a slot's previous use
// to be handed back, and issues its bulk copies.  While it waits on a full
// ring (the consumers are in a grid barrier, the attention phase or the
// sampler) it prefetches up to kPfSlots further slots into L2, so HBM keeps
// streaming; continuous prefetching slows the steady stream, so it is not done
// otherwise.  Every wait is bounded and also ends when the consumers raise
// `stop`.
__device__ void producer(const DecodeArgs& a, const ModelW& w, Ring& R, const Rows& rows, Cursor start, int n_steps) {
    int* status = a.b.ctl->status;
    Cursor tma = start, pf = start;
    SlotDesc d, dp;
    uint32_t j = 0, pfn = 0;  // slots issued; slots the prefetch cursor has passed
    while (!R.stop && next_slot(w, rows, n_steps, tma, d)) {
        const int s = j % kSlots;
        if (j >= kSlots) {
            const uint32_t parity = ((j / kSlots) - 1) & 1u;
            const unsigned long long t0 = globaltimer_ns();
            bool ok = true;
            for (uint32_t i = 0; !mbar_try_wait(&R.empty[s], parity); ++i) {
                if (pfn < j + 1 + kPfSlots && next_slot(w, rows, n_steps, pf, dp)) {
                    if (pfn > j)  // slots up to j are already issued or being issued
                        for (int q = 0; q < dp.n; ++q) bulk_prefetch_l2(dp.src[q], dp.bytes[q]);
                    ++pfn;
                    continue;
                }
                if ((i & 63u) == 63u) {
                    if (R.stop) { ok = false; break; }
                    const unsigned long long dt = globaltimer_ns() - t0;
                    if (dt > kStatusPollNs && ld_volatile(status) != 0) { ok = false; break; }
                    if (dt > kWaitLimitNs) {
                        set_status(status, kStatusRingTimeout, 900, (int)j);
                        ok = false;
                        break;
                    }
                }
            }
            if (!ok) break;
        }
        mbar_expect_tx(&R.full[s], d.total);
        unsigned char* dst = R.data[s];
        for (int i = 0; i < d.n; ++i) {
            bulk_g2s(dst, d.src[i], d.bytes[i], &R.full[s]);
            dst += d.bytes[i];
        }
        ++j;
        R.issued = j;
        while (pfn < j && next_slot(w, rows, n_steps, pf, dp)) ++pfn;  // keep the prefetch cursor ahead
    }
    __threadfence_block();
    R.producer_done = 1;
}

// Thread 0 of the consumers at exit: stop the producer, then wait for every
// issued slot that was not consumed (a copy must not land in shared memory of a
// CTA that has exited).
__device__ void ring_finish(Ring& R, uint32_t consumed) {
    R.stop = 1;
    __threadfence_block();
    const unsigned long long t0 = globaltimer_ns();
    while (!R.producer_done)
        if (globaltimer_ns() - t0 > kWaitLimitNs) break;
    for (uint32_t k = consumed; k < R.issued; ++k) {
        const unsigned long long t1 = globaltimer_ns();
        while (!mbar_try_wait(&R.full[k % kSlots], (k / kSlots) & 1u))
            if (globaltimer_ns() - t1 > kWaitLimitNs) return;
    }
}

// Thread 0, before the producer starts: the mbarriers.
__device__ void ring_init(Ring& R) {
    for (int i = 0; i < kSlots; ++i) {
        mbar_init(&R.full[i], 1);
        mbar_init(&R.empty[i], 1);
    }
    R.issued = 0;
    R.stop = 0;
    R.producer_done = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

struct Ctx {
    const DecodeArgs& a;
    const ModelW& w;  // shared-memory copy of *a.w
    Ring& R;
    PhaseSmem& sm;
    Rows rows;
    int cta, ncta;
    uint32_t k;  // slots consumed so far (uniform across the consumers)
};

// Every consumer thread waits for the next slot.  The caller folds `ok` into
// its next csync_or so that an abort is taken uniformly.
__device__ __forceinline__ const float* slot_wait(Ctx& cx, bool& ok, int where) {
    const int s = cx.k % kSlots;
    ok = mbar_wait_bounded(&cx.R.full[s], (cx.k / kSlots) & 1u, cx.a.b.ctl->status, where);
    return reinterpret_cast<const float*>(cx.R.data[s]);
}

// After a csync that follows the last read of the slot: hand it back.
__device__ __forceinline__ void slot_release(Ctx& cx) {
    if (threadIdx.x == 0) mbar_arrive(&cx.R.empty[cx.k % kSlots]);
    ++cx.k;
}

// Input-vector layout of the GEMVs: thread t owns columns 2*(t%128) + 256*j
// (+1), j < 5, so each 128-thread group holds the whole 1280-vector once and a
// 4-row slot keeps 4 groups busy.
__device__ __forceinline__ int col_of(int j) { return 2 * (threadIdx.x & 127) + 256 * j; }

// LayerNorm of the vector in `x` (statistics over group 0), gamma/beta at
// g/b (shared memory).  Two-pass mean and centred variance, eps inside the
// root (kernels.metal:618-669).
__device__ void layernorm2(float2 (&x)[5], const float* g, const float* b, float* red) {
    const bool owner = threadIdx.x < 128;
    float s = 0.f;
    if (owner) {
#pragma unroll
        for (int j = 0; j < 5; ++j) s += x[j].x + x[j].y;
    }
    const float mean = cblock_sum(s, red) * (1.0f / kWidth);
    float v = 0.f;
    if (owner) {
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const float a = x[j].x - mean, c = x[j].y - mean;
            v = fmaf(a, a, v);
            v = fmaf(c, c, v);
        }
    }
    const float var = cblock_sum(v, red) * (1.0f / kWidth);
    const float inv = 1.0f / sqrtf(var + kLnEps);
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        const int c = col_of(j);
        x[j].x = (x[j].x - mean) * inv * g[c] + b[c];
        x[j].y = (x[j].y - mean) * inv * g[c + 1] + b[c + 1];
    }
}

// Consumes the slot holding LayerNorm vectors and normalises x with the first
// (and, for the head, the second) pair.
__device__ bool ln_slot(Ctx& cx, float2 (&x)[5], int pairs, int where) {
    bool ok;
    const float* slot = slot_wait(cx, ok, where);
    if (csync_or(!ok)) return false;
    layernorm2(x, slot, slot + kWidth, cx.sm.red);
    if (pairs == 2) layernorm2(x, slot + 2 * kWidth, slot + 3 * kWidth, cx.sm.red);
    csync();
    slot_release(cx);
    return true;
}

// y[row] = W[row, :] . x for `nrows` streamed rows (4 per slot); epi(row, y)
// runs on consumer thread `row` after the slot's reduction.
template <class Epi>
__device__ bool gemv_slots(Ctx& cx, int nrows, const float2 (&x)[5], int where, Epi epi) {
    const int t = threadIdx.x, rr = t >> 7, tig = t & 127, warp = t >> 5, lane = t & 31;
    for (int r0 = 0; r0 < nrows; r0 += kRowsPerSlot) {
        bool ok;
        const float* slot = slot_wait(cx, ok, where);
        float acc = 0.f;
        if (ok && r0 + rr < nrows) {
            const float2* w = reinterpret_cast<const float2*>(slot + rr * kWidth) + tig;
#pragma unroll
            for (int j = 0; j < 5; ++j) {
                const float2 wv = w[j * 128];
                acc = fmaf(wv.x, x[j].x, acc);
                acc = fmaf(wv.y, x[j].y, acc);
            }
        }
        acc = warp_sum(acc);
        float* rb = cx.sm.red2[cx.k & 1];
        if (lane == 0) rb[warp] = acc;
        if (csync_or(!ok)) return false;
        slot_release(cx);
        if (t < kRowsPerSlot && r0 + t < nrows) epi(r0 + t, (rb[4 * t] + rb[4 * t + 1]) + (rb[4 * t + 2] + rb[4 * t + 3]));
    }
    return true;
}

constexpr float kFixScale = 4294967296.0f;  // 2^32
constexpr double kFixInv = 1.0 / 4294967296.0;

// Row r of the residual stream entering in-step layer `li` (li = layers: the
// input of the head).  li = 0: the token embedding (gpt_build_current,
// kernels.metal:1310-1325); otherwise r + (mlp.c_proj output + bias) of the
// previous layer, the output being the fixed-point sum of the CTAs' shares.
__device__ __forceinline__ float resid_in(const DecodeArgs& a, const ModelW& w, int li, int g, uint32_t token,
                                         uint32_t pos, int r) {
    if (li == 0)
        return __ldg(w.mel_emb + (size_t)token * kWidth + r) + __ldg(w.mel_pos + (size_t)pos * kWidth + r);
    const int gp = (g - 1) & 1;
    const float mp = float(double(__ldcg(a.b.acc + gp * kWidth + r)) * kFixInv);
    return __ldcg(a.b.r + gp * kWidth + r) + (mp + __ldg(w.layer[li - 1].b_mp + r));
}

__device__ __forceinline__ void load_resid(const DecodeArgs& a, const ModelW& w, int li, int g, uint32_t token,
                                           uint32_t pos, float2 (&x)[5]) {
    if (a.head_src && li == w.layers) {  // prefill: the last hidden row
#pragma unroll
        for (int j = 0; j < 5; ++j) x[j] = __ldcg(reinterpret_cast<const float2*>(a.head_src + col_of(j)));
        return;
    }
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        const int c = col_of(j);
        x[j] = make_float2(resid_in(a, w, li, g, token, pos, c), resid_in(a, w, li, g, token, pos, c + 1));
    }
}

// ---------------------------------------------------------------- phases
__device__ bool phase_qkv(Ctx& cx, int li, int g, uint32_t token, uint32_t pos) {
    const DecodeArgs& a = cx.a;
    const LayerW& L = cx.w.layer[li];
    const int r0 = cx.rows.q0, r1 = cx.rows.q1;
    if ((int)threadIdx.x < r1 - r0) cx.sm.bias[threadIdx.x] = __ldg(L.b_qkv + r0 + threadIdx.x);
    float2 x[5];
    load_resid(a, cx.w, li, g, token, pos, x);
    if (!ln_slot(cx, x, 1, 10 + li)) return false;
    float* out = a.b.qkv + r0;
    const float* bias = cx.sm.bias;
    return gemv_slots(cx, r1 - r0, x, 40 + li, [&](int row, float v) { out[row] = v + bias[row]; });
}

__device__ __forceinline__ uint32_t attn_chunk(uint32_t keys, int ncta) {
    uint32_t ch = (keys * kHeads + ncta - 1) / ncta;
    return max((ch + 15u) & ~15u, 16u);
}

// Split-K attention for the current query over keys [0, S] (S cached + the
// current key from qkv).  Unit = (head, chunk of ch keys); warp w takes keys
// w, w+16, ... of the chunk with an online softmax (K and V fetched together);
// the 16 warp states are merged in shared memory into one partial
// (max, sum, 64 outputs) per unit, merged across chunks in phase C.  The unit
// holding key S appends this token's K/V to the cache.
__device__ void phase_attn(Ctx& cx, int li, uint32_t S) {
    const DecodeArgs& a = cx.a;
    const uint32_t keys = S + 1;
    const uint32_t ch = attn_chunk(keys, cx.ncta);
    const uint32_t nch = (keys + ch - 1) / ch, units = kHeads * nch;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    for (uint32_t u = cx.cta; u < units; u += cx.ncta) {
        const uint32_t h = u / nch, c = u % nch, k0 = c * ch, k1 = min(k0 + ch, keys);
        float* Kc = a.b.kv + (((size_t)li * 2 + 0) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
        float* Vc = a.b.kv + (((size_t)li * 2 + 1) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
        const float* kcur = a.b.qkv + kWidth + h * kHeadDim;
        const float* vcur = a.b.qkv + 2 * kWidth + h * kHeadDim;
        const float2 q = __ldcg(reinterpret_cast<const float2*>(a.b.qkv + h * kHeadDim) + lane);
        float m = -INFINITY, l = 0.f;
        float2 o = make_float2(0.f, 0.f);
        for (uint32_t kb = k0 + warp; kb < k1; kb += 4 * kWarps) {
            float2 kv[4], vv[4];
            float s[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t kk = kb + i * kWarps;
                if (kk < k1) {
                    const float* kr = kk < S ? Kc + (size_t)kk * kHeadDim : kcur;
                    const float* vr = kk < S ? Vc + (size_t)kk * kHeadDim : vcur;
                    kv[i] = __ldcg(reinterpret_cast<const float2*>(kr) + lane);
                    vv[i] = __ldcg(reinterpret_cast<const float2*>(vr) + lane);
                } else {
                    kv[i] = vv[i] = make_float2(0.f, 0.f);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) s[i] = fmaf(q.x, kv[i].x, q.y * kv[i].y);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int i = 0; i < 4; ++i) s[i] += __shfl_xor_sync(0xffffffffu, s[i], off);
            float mn = m;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                s[i] = kb + i * kWarps < k1 ? s[i] * 0.125f : -INFINITY;  // rsqrt(64)
                mn = fmaxf(mn, s[i]);
            }
            const float corr = expf(m - mn);
            l *= corr;
            o.x *= corr;
            o.y *= corr;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float p = expf(s[i] - mn);
                l += p;
                o.x = fmaf(p, vv[i].x, o.x);
                o.y = fmaf(p, vv[i].y, o.y);
            }
            m = mn;
        }
        if (lane == 0) {
            cx.sm.wm[warp] = m;
            cx.sm.wl[warp] = l;
        }
        cx.sm.wo[warp][2 * lane] = o.x;
        cx.sm.wo[warp][2 * lane + 1] = o.y;
        csync();
        if (t < kHeadDim) {
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, cx.sm.wm[w]);
            float Ls = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float e = cx.sm.wl[w] > 0.f ? expf(cx.sm.wm[w] - M) : 0.f;
                Ls = fmaf(e, cx.sm.wl[w], Ls);
                O = fmaf(e, cx.sm.wo[w][t], O);
            }
            float* pp = a.b.part + ((size_t)h * nch + c) * 66;
            pp[2 + t] = O;
            if (t == 0) {
                pp[0] = M;
                pp[1] = Ls;
            }
        }
        if (c == nch - 1) {
            if (t >= 64 && t < 128)
                Kc[(size_t)S * kHeadDim + t - 64] = __ldcg(kcur + t - 64);
            else if (t >= 128 && t < 192)
                Vc[(size_t)S * kHeadDim + t - 128] = __ldcg(vcur + t - 128);
        }
        csync();
    }
}

__device__ bool phase_oproj(Ctx& cx, int li, int g, uint32_t token, uint32_t pos, uint32_t S) {
    const DecodeArgs& a = cx.a;
    const LayerW& L = cx.w.layer[li];
    const int r0 = cx.rows.o0, r1 = cx.rows.o1;
    const int t = threadIdx.x;
    if (t < r1 - r0) {
        cx.sm.bias[t] = __ldg(L.b_o + r0 + t);
        cx.sm.res[t] = resid_in(a, cx.w, li, g, token, pos, r0 + t);
    }
    // merge the split-K attention partials of every head (same chunking as B)
    const uint32_t keys = S + 1;
    const uint32_t ch = attn_chunk(keys, cx.ncta);
    const uint32_t nch = (keys + ch - 1) / ch;
    if (t < kWidth / 4) {
        const int h = (4 * t) / kHeadDim, d = (4 * t) % kHeadDim;
        const float* ph = a.b.part + (size_t)h * nch * 66;
        float M = -INFINITY;
        for (uint32_t c = 0; c < nch; ++c) M = fmaxf(M, __ldcg(ph + c * 66));
        float Ls = 0.f, o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
        for (uint32_t c = 0; c < nch; ++c) {
            const float* pc = ph + c * 66;
            const float e = expf(__ldcg(pc) - M);
            Ls = fmaf(e, __ldcg(pc + 1), Ls);
            o0 = fmaf(e, __ldcg(pc + 2 + d), o0);
            o1 = fmaf(e, __ldcg(pc + 3 + d), o1);
            o2 = fmaf(e, __ldcg(pc + 4 + d), o2);
            o3 = fmaf(e, __ldcg(pc + 5 + d), o3);
        }
        *reinterpret_cast<float4*>(&cx.sm.attn[4 * t]) = make_float4(o0 / Ls, o1 / Ls, o2 / Ls, o3 / Ls);
    }
    csync();
    float2 x[5];
#pragma unroll
    for (int j = 0; j < 5; ++j) x[j] = *reinterpret_cast<const float2*>(&cx.sm.attn[col_of(j)]);
    float* out = a.b.r + (g & 1) * kWidth + r0;
    const float* bias = cx.sm.bias;
    const float* res = cx.sm.res;
    return gemv_slots(cx, r1 - r0, x, 70 + li, [&](int row, float v) { out[row] = res[row] + (v + bias[row]); });
}

__device__ bool phase_mlp(Ctx& cx, int li, int g) {
    const DecodeArgs& a = cx.a;
    const LayerW& L = cx.w.layer[li];
    const int f0 = cx.rows.f0, f1 = cx.rows.f1;
    const int nf = f1 - f0, t = threadIdx.x;
    if (t < nf) cx.sm.bias[t] = __ldg(L.b_fc + f0 + t);
    // clear this CTA's share of the accumulator the next layer will use
    if (t < cx.rows.o1 - cx.rows.o0) a.b.acc[((g + 1) & 1) * kWidth + cx.rows.o0 + t] = 0ll;
    float2 x[5];
#pragma unroll
    for (int j = 0; j < 5; ++j) x[j] = __ldcg(reinterpret_cast<const float2*>(a.b.r + (g & 1) * kWidth + col_of(j)));
    if (!ln_slot(cx, x, 1, 100 + li)) return false;
    float* f = cx.sm.f;
    const float* bias = cx.sm.bias;
    if (!gemv_slots(cx, nf, x, 130 + li, [&](int row, float v) { f[row] = gelu_ref(v + bias[row]); })) return false;
    csync();
    // split-K share of mlp.c_proj: out[j] += sum_{i in rows} WT[i, j] * f[i]
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < nf; r0 += kRowsPerSlot) {
        bool ok;
        const float* slot = slot_wait(cx, ok, 160 + li);
        if (ok && t < kWidth / 4) {
            const int n = min(kRowsPerSlot, nf - r0);
            for (int rr = 0; rr < n; ++rr) {
                const float4 w = reinterpret_cast<const float4*>(slot + rr * kWidth)[t];
                const float fv = f[r0 + rr];
                acc.x = fmaf(w.x, fv, acc.x);
                acc.y = fmaf(w.y, fv, acc.y);
                acc.z = fmaf(w.z, fv, acc.z);
                acc.w = fmaf(w.w, fv, acc.w);
            }
        }
        if (csync_or(!ok)) return false;
        slot_release(cx);
    }
    if (t < kWidth / 4) {
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(a.b.acc + (g & 1) * kWidth) + 4 * t;
        atomicAdd(dst + 0, (unsigned long long)__float2ll_rn(acc.x * kFixScale));
        atomicAdd(dst + 1, (unsigned long long)__float2ll_rn(acc.y * kFixScale));
        atomicAdd(dst + 2, (unsigned long long)__float2ll_rn(acc.z * kFixScale));
        atomicAdd(dst + 3, (unsigned long long)__float2ll_rn(acc.w * kFixScale));
    }
    return true;
}

// gpt.cpp:120-122: last hidden row -> ln_f -> final_norm -> mel_head.
__device__ bool phase_head(Ctx& cx, int g, uint32_t token, uint32_t pos) {
    const DecodeArgs& a = cx.a;
    const int r0 = cx.rows.h0, r1 = cx.rows.h1;
    if ((int)threadIdx.x < r1 - r0) cx.sm.bias[threadIdx.x] = __ldg(cx.w.b_head + r0 + threadIdx.x);
    float2 x[5];
    load_resid(a, cx.w, cx.w.layers, g, token, pos, x);
    if (!ln_slot(cx, x, 2, 200)) return false;
    float* out = a.b.logits + r0;
    const float* bias = cx.sm.bias;
    return gemv_slots(cx, r1 - r0, x, 201, [&](int row, float v) { out[row] = v + bias[row]; });
}

// Grid barrier of the persistent kernel (all CTAs co-resident by the
// cooperative launch): monotonic arrival counter, bounded spin; true when the
// kernel must abort (error status or timeout).
__device__ bool grid_barrier(Ctx& cx, unsigned& target, int where) {
    target += gridDim.x;
    csync();
    if (threadIdx.x == 0) {
        unsigned* bar = &cx.a.b.ctl->bar;
        int* status = cx.a.b.ctl->status;
        __threadfence();
        atomicAdd(bar, 1u);
        const unsigned long long t0 = globaltimer_ns();
        unsigned spins = 0;
        while (ld_acquire_gpu(bar) < target) {
            if ((++spins & 31u) == 0) {
                const unsigned long long dt = globaltimer_ns() - t0;
                if (dt > kStatusPollNs && ld_volatile(status) != 0) break;
                if (dt > kWaitLimitNs) {
                    set_status(status, kStatusBarrierTimeout, where, (int)target);
                    break;
                }
            }
        }
        __threadfence();
        cx.sm.abort = ld_volatile(status) != 0;
    }
    csync();
    return cx.sm.abort != 0;
}

// One forward step; true when aborted.
__device__ bool forward_step(Ctx& cx, int step, uint32_t token, uint32_t pos, uint32_t S, unsigned& target) {
    const int L = cx.w.layers;
    for (int li = 0; li < L; ++li) {
        const int g = step * L + li;
        if (!phase_qkv(cx, li, g, token, pos) || grid_barrier(cx, target, li * 8 + 0)) return true;
        phase_attn(cx, li, S);
        if (grid_barrier(cx, target, li * 8 + 1)) return true;
        if (!phase_oproj(cx, li, g, token, pos, S) || grid_barrier(cx, target, li * 8 + 2)) return true;
        if (!phase_mlp(cx, li, g) || grid_barrier(cx, target, li * 8 + 3)) return true;
    }
    return !phase_head(cx, step * L + L, token, pos) || grid_barrier(cx, target, 1000);
}

constexpr int kCtaThreads = kThreads + 32;  // 16 consumer warps + the producer warp

__global__ void __launch_bounds__(kCtaThreads, 1) k_decode(DecodeArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
    const int cta = blockIdx.x, ncta = gridDim.x;
    const int n_fwd = a.mode == kModeGenerate ? int(a.n_iter) - 1 : 1;
    const Rows rows = cta_rows(cta, ncta);
    load_table(sm.w, a.w);
    if (threadIdx.x == 0) {
        sm.ph.abort = 0;
        ring_init(sm.ring);
    }
    __syncthreads();
    if (threadIdx.x >= kThreads) {  // producer warp
        if (threadIdx.x == kThreads) {
            if (n_fwd > 0) producer(a, sm.w, sm.ring, rows, Cursor{0, 0, kSegLn1, 0, 0xffffffffu}, n_fwd);
            else sm.ring.producer_done = 1;
        }
        return;
    }
    sampler_init_seen(sm.sa, a.history, a.history_n);
    Ctx cx{a, sm.w, sm.ring, sm.ph, rows, cta, ncta, 0};
    SamplerBig* big = a.b.sampler_big + cta;
    unsigned target = 0;
    uint32_t token = a.first_code, n_codes = 0, stopped = 0, fwd = 0;
    for (uint32_t i = 0; i < a.n_iter; ++i) {
        if (a.mode == kModeGenerate) {
            token = run_sampler(a.b.logits, a.opts, i, a.opts.do_sample == 0, sm.sa, big, nullptr, a.b.ctl->status);
            if (token == (uint32_t)kStopCode) {
                stopped = 1;
                break;
            }
            if (token >= (uint32_t)kStartCode) {
                if (token != 0xffffffffu && threadIdx.x == 0)
                    set_status(a.b.ctl->status, kStatusInvalidCode, 300, (int)token);
                break;
            }
            if (cta == 0 && threadIdx.x == 0) a.codes[i] = token;
            ++n_codes;
            sampler_mark_seen(sm.sa, token);
            if (i + 1 == a.n_iter) break;
        }
        if (forward_step(cx, int(i), token, a.pos0 + i, a.s0 + i, target)) break;
        ++fwd;
    }
    if (threadIdx.x == 0) ring_finish(sm.ring, cx.k);
    if (cta == 0 && threadIdx.x == 0) {
        DecodeCtl* ctl = a.b.ctl;
        ctl->info[0] = n_codes;
        ctl->info[1] = stopped;
        ctl->info[2] = (uint32_t)ld_volatile(ctl->status);
        ctl->info[3] = fwd;
        if (a.info_out)
            for (int i = 0; i < 4; ++i) a.info_out[i] = ctl->info[i];
    }
}

// ------------------------------------------------------------ layered path
enum LayerPhase : int { kPhQkv = 0, kPhAttn, kPhOproj, kPhMlp, kPhHead };

__global__ void __launch_bounds__(kCtaThreads, 1) k_phase(DecodeArgs a, int phase, int li, int g, uint32_t pos,
                                                          uint32_t S) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(smem_raw);
    if (ld_volatile(&a.b.ctl->done)) return;
    const int cta = blockIdx.x, ncta = gridDim.x;
    const Rows rows = cta_rows(cta, ncta);
    load_table(sm.w, a.w);
    if (threadIdx.x == 0) ring_init(sm.ring);
    __syncthreads();
    if (threadIdx.x >= kThreads) {  // producer warp: exactly this phase's slots
        if (threadIdx.x == kThreads) {
            Cursor c{0, li, kSegLn1, 0, 0};
            const int nq = rows.q1 - rows.q0, no = rows.o1 - rows.o0, nf = rows.f1 - rows.f0, nh = rows.h1 - rows.h0;
            if (phase == kPhQkv) {
                c.budget = 1 + (nq + kRowsPerSlot - 1) / kRowsPerSlot;
            } else if (phase == kPhOproj) {
                c.seg = kSegO;
                c.budget = (no + kRowsPerSlot - 1) / kRowsPerSlot;
            } else if (phase == kPhMlp) {
                c.seg = kSegLn2;
                c.budget = 1 + 2 * ((nf + kRowsPerSlot - 1) / kRowsPerSlot);
            } else if (phase == kPhHead) {
                c.layer = sm.w.layers;
                c.seg = kSegFinalLn;
                c.budget = 1 + (nh + kRowsPerSlot - 1) / kRowsPerSlot;
            }
            if (c.budget) producer(a, sm.w, sm.ring, rows, c, 1);
            else sm.ring.producer_done = 1;
        }
        return;
    }
    const uint32_t token = *reinterpret_cast<volatile uint32_t*>(&a.b.ctl->token);
    Ctx cx{a, sm.w, sm.ring, sm.ph, rows, cta, ncta, 0};
    switch (phase) {
        case kPhQkv: phase_qkv(cx, li, g, token, pos); break;
        case kPhAttn: phase_attn(cx, li, S); break;
        case kPhOproj: phase_oproj(cx, li, g, token, pos, S); break;
        case kPhMlp: phase_mlp(cx, li, g); break;
        default: phase_head(cx, g, token, pos); break;
    }
    if (threadIdx.x == 0) ring_finish(sm.ring, cx.k);
}

constexpr size_t kSamplerSmallBytes = (sizeof(SamplerSmem) + 15) & ~size_t(15);
constexpr size_t kSamplerDynSmem = kSamplerSmallBytes + sizeof(SamplerBig);

// One CTA: selects code i of the layered generate loop (or installs the input
// code for a single step) and updates ctl->{token, done, info}.
__global__ void __launch_bounds__(kThreads, 1) k_layer_sample(DecodeArgs a, uint32_t i) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    SamplerBig* big = reinterpret_cast<SamplerBig*>(smem_raw + kSamplerSmallBytes);
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
    const uint32_t token = run_sampler(a.b.logits, a.opts, i, a.opts.do_sample == 0, sm, big, nullptr, ctl->status);
    if (threadIdx.x != 0) return;
    bool finish = false;
    if (token == (uint32_t)kStopCode) {
        ctl->info[1] = 1;
        finish = true;
    } else if (token >= (uint32_t)kStartCode) {
        if (token != 0xffffffffu) set_status(ctl->status, kStatusInvalidCode, 300, (int)token);
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
    SamplerBig* big = reinterpret_cast<SamplerBig*>(smem_raw + kSamplerSmallBytes);
    sampler_init_seen(sm, hist, hist_n);
    run_sampler(logits, o, 0, false, sm, big, out, status);
}

// Beam search, one parent (gpt_sampling.cpp:206-214): float log-softmax of
// the parent's logits, the processors with num_beams > 1 semantics, plus the
// parent's cumulative score.  One CTA.
__global__ void __launch_bounds__(kThreads, 1) k_beam_scores(const float* logits, SampleOpts o, const uint32_t* hist,
                                                             uint32_t hist_n, float beam_score, float* tmp, float* out,
                                                             int* status) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    SamplerBig* big = reinterpret_cast<SamplerBig*>(smem_raw + kSamplerSmallBytes);
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
    run_sampler(tmp, o, 0, false, sm, big, out, status);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt) out[base + k] = out[base + k] + beam_score;
}

// ------------------------------------------------------------ host side
size_t decode_smem_bytes() { return sizeof(DecodeSmem); }
size_t sampler_big_bytes() { return sizeof(SamplerBig); }
size_t sampler_dyn_smem_bytes() { return kSamplerDynSmem; }

cudaError_t decode_configure(int* blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DecodeSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_phase, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DecodeSmem));
    if (e != cudaSuccess) return e;
    for (const void* f : {(const void*)k_layer_sample, (const void*)k_processors, (const void*)k_beam_scores}) {
        e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSamplerDynSmem);
        if (e != cudaSuccess) return e;
    }
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, k_decode, kCtaThreads, sizeof(DecodeSmem));
}

cudaError_t launch_decode_persistent(const DecodeArgs& a, int ncta, cudaStream_t s) {
    DecodeArgs copy = a;
    void* args[] = {&copy};
    return cudaLaunchCooperativeKernel((const void*)k_decode, dim3(ncta), dim3(kCtaThreads), args, sizeof(DecodeSmem),
                                       s);
}

cudaError_t launch_decode_layered(const DecodeArgs& a, int layers, int ncta, cudaStream_t s, uint64_t* launches) {
    for (uint32_t i = 0; i < a.n_iter; ++i) {
        k_layer_sample<<<1, kThreads, kSamplerDynSmem, s>>>(a, i);
        ++*launches;
        if (a.mode == kModeGenerate && i + 1 == a.n_iter) break;
        const uint32_t pos = a.pos0 + i, S = a.s0 + i;
        for (int l = 0; l < layers; ++l) {
            const int g = int(i) * layers + l;
            for (int ph = kPhQkv; ph <= kPhMlp; ++ph) {
                k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, ph, l, g, pos, S);
                ++*launches;
            }
        }
        k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, kPhHead, layers, int(i) * layers + layers, pos, S);
        ++*launches;
    }
    k_layer_finish<<<1, 1, 0, s>>>(a);
    ++*launches;
    return cudaGetLastError();
}

cudaError_t launch_head(const DecodeArgs& a, int ncta, cudaStream_t s) {
    k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, kPhHead, 0, 0, 0, 0);
    return cudaGetLastError();
}

cudaError_t launch_processors(const float* logits, const SampleOpts& o, const uint32_t* hist, uint32_t hist_n,
                              float* out, int* status, cudaStream_t s) {
    k_processors<<<1, kThreads, kSamplerDynSmem, s>>>(logits, o, hist, hist_n, out, status);
    return cudaGetLastError();
}

cudaError_t launch_beam_scores(const float* logits, const SampleOpts& o, const uint32_t* hist, uint32_t hist_n,
                               float beam_score, float* tmp, float* out, int* status, cudaStream_t s) {
    k_beam_scores<<<1, kThreads, kSamplerDynSmem, s>>>(logits, o, hist, hist_n, beam_score, tmp, out, status);
    return cudaGetLastError();
}

}  // namespace itts
