// Batch-1 decode of the IndexTTS 2.5 GPT on B200 (sm_100a): the device code
// and launchers, compiled once per weight type (decode.cu: fp32 matrices,
// decode_bf16.cu: bf16 matrices) into namespace itts::ITTS_WNS.
//
// One decode step (src/gpt.cpp:88-125 with initial=false) is five phases per
// layer plus the head, each a function of (cta, ncta) over the whole grid:
//   A    h -> LN1 -> this CTA's c_attn rows -> qkv
//   B    split-K attention over the KV cache + K/V append (kernels.metal:2064-
//        2145); the last unit of each head merges the head's partials -> attn
//   C    attn -> this CTA's attn.c_proj rows + bias + residual -> hm
//   D    hm -> LN2 -> this CTA's c_fc rows + GELU -> f
//   E    f -> this CTA's mlp.c_proj rows (5120 wide) + bias + residual -> h
//   head h -> ln_f -> final_norm -> mel_head rows -> logits (in the generate
//        loop already carrying the repetition penalty and the temperature)
// Activations pass between CTAs as epoch-tagged 64-bit words that the reader
// polls (the data is its own flag), f through a per-layer arrival counter; the
// only grid barrier of a step follows the head.
//
// Weight streaming: every CTA owns a contiguous block of rows per matrix.  Its
// rows are fetched into a 10-slot x 20 KB shared-memory ring with
// cp.async.bulk (1-D TMA, completion on a "full" mbarrier, L2 evict-first; no
// multicast) by a dedicated producer warp that walks the CTA's segment
// schedule, two copies in flight at a time; the 16 consumer warps hand a slot
// back on its "empty" mbarrier, and while the ring is full the producer
// prefetches further ahead into L2.  LayerNorm vectors are loaded into
// registers (each lane's columns) when a phase starts waiting for its input.  The stream therefore runs through the hand-off waits, the
// attention phase and the sampler, which are the latency-bound parts of the
// step.
//
// Drivers:
//   * k_decode: one cooperative launch (one CTA per SM) for a whole token
//     loop; the sampler runs redundantly in every CTA so the next token needs
//     no extra barrier.
//   * k_phase: one launch per phase with the same device code (layered mode,
//     for diagnosis and as the non-cooperative path); its ring covers only that
//     phase.
#pragma once
#include <cuda_bf16.h>

#include "common.cuh"
#include "model.hpp"
#include "sampler.cuh"

#ifndef ITTS_WNS
#error "define ITTS_WNS and ITTS_WBF16 before including decode_body.cuh"
#endif

namespace itts {
namespace ITTS_WNS {


// ------------------------------------------------------------ weight ring
#if ITTS_WBF16
using wtype = __nv_bfloat16;  // element of the streamed weight matrices
constexpr int kRowsPerSlot = 8;  // rows of 1280 per slot
#else
using wtype = float;
constexpr int kRowsPerSlot = 4;
#endif
constexpr int kWBytes = int(sizeof(wtype));
constexpr int kRowBytes = kWidth * kWBytes;            // one 1280-wide matrix row
constexpr int kSlotBytes = kRowsPerSlot * kRowBytes;  // 20 KB
constexpr int kSlots = 10;
// Bulk copies a CTA keeps in flight.  Two 20 KB copies (148 x 40 KB
// outstanding) cover the HBM latency at the rate the layers consume; more only
// lengthens the memory queues that every hand-off load and store also waits
// in: the ring refills after a phase in a paced trickle instead of a burst of
// copies from every CTA at once.
constexpr int kInFlight = 2;
// Consumer geometry: warp w works on row w / kWarpsPerRow of a slot and on
// column block w % kWarpsPerRow (kColsPerWarp wide); lane l reads 8 bytes per
// load (2 fp32 or 4 bf16 weights) and holds the matching kVec float2 of the
// input vector (col_of).  A 5120-wide row spans kWarpsPerLong warps with the
// same per-warp width.
constexpr int kWarpsPerRow = kWarps / kRowsPerSlot;
constexpr int kColsPerWarp = kWidth / kWarpsPerRow;
constexpr int kVec = kColsPerWarp / 64;
constexpr int kLongPerSlot = kSlotBytes / (kFfn * kWBytes);
constexpr int kWarpsPerLong = kWarps / kLongPerSlot;
static_assert(kWarpsPerRow * kRowsPerSlot == kWarps && kColsPerWarp % 64 == 0, "slot geometry");
static_assert(kWarpsPerLong * kColsPerWarp == kFfn, "5120-wide rows use the same per-warp width");

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

constexpr int kMaxRowsPerCta = 64;  // host check: ceil(8194 / grid) <= 64 (so ceil(1280 / grid) <= 16)
constexpr int kPartStride = 68;     // attention partial: max, sum, 2 pad, 64 outputs
constexpr int kMaxChunks = 8;       // key chunks per head (partials merged per head)

struct PhaseSmem {
    float red[32];
    float wstat[kWarps][2];  // LayerNorm: per-warp (mean, M2)
    union {
        float rowred[kMaxRowsPerCta][kWarpsPerRow];  // 1280-wide rows: block sums
        float longred[16][kWarpsPerLong];            // 5120-wide rows: block sums
    };
    float f[kMaxRowsPerCta];          // this CTA's GELU outputs
    __align__(16) float xin[kWidth];  // staged input vector (phase A: the layer input, kept for phase C)
    union {                           // phase B's warp states / phase C's merged heads
        float wo[kWarps][kHeadDim];
        __align__(16) float attn[kWidth];
    };
    float wm[kWarps], wl[kWarps];
    __align__(16) float qkvh[3 * kHeadDim];  // phase B: q, k, v of the unit's head
    int abort, last;
};

struct DecodeSmem {
    Ring ring;
    PhaseSmem ph;
    SamplerSmem sa;
    ModelW w;  // the weight pointer table, read at every slot and phase start
};
static_assert(kInFlight >= 1 && kInFlight < kSlots, "paced copies must stay inside the ring");
static_assert(sizeof(DecodeSmem) <= 227 * 1024, "decode kernel shared memory above the sm_100 per-CTA limit");

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
// try_wait with a suspend-time hint: a thread whose phase does not complete
// is woken after about `ns` nanoseconds instead of the hardware's default
// suspend limit (about a millisecond), so a loop around it notices a stop
// request promptly.
__device__ __forceinline__ bool mbar_try_wait_hint(unsigned long long* bar, uint32_t parity, uint32_t ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return done != 0;
}
// L2 policy of the streamed weights: evicted first, so that one step's 1.9 GB
// sweep does not push the KV cache, the activations and the kernel's own
// instructions out of L2.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Bounded wait for a ring slot; every thread waits.  The spin touches no
// global memory for the first kStatusPollNs (a global load costs a full L2
// round trip and would delay noticing the slot); after that it also watches
// the status word so that an error elsewhere ends the wait.  False on timeout
// or error.
constexpr unsigned long long kStatusPollNs = 200000ull;

// Time limit of the launch's waits: DecodeArgs::wait_ns, or kWaitLimitNs when 0.
__device__ __forceinline__ unsigned long long wait_limit(const DecodeArgs& a) {
    return a.wait_ns ? a.wait_ns : kWaitLimitNs;
}

__device__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity, const DecodeArgs& a, int where) {
    if (mbar_try_wait(bar, parity)) return true;
    int* status = a.b.ctl->status;
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            const unsigned long long dt = globaltimer_ns() - t0;
            if (dt > kStatusPollNs && ld_volatile(status) != 0) return false;
            if (dt > wait_limit(a)) {
                set_status(status, kStatusRingTimeout, where, (int)i);
                return false;
            }
        }
    }
}

// The weight schedule of one CTA, as segments of contiguous bytes; segment k
// of a forward step (4 per layer, then 1 for the head):
//   4l+0 its c_attn rows     4l+1 its attn.c_proj rows
//   4l+2 its c_fc rows       4l+3 its mlp.c_proj rows (5120 wide)
//   4L   its mel_head rows
// Segments are cut into kSlotBytes slots (kRowsPerSlot rows of 1280, or
// kRowsPerSlot / 4 rows of 5120).
constexpr int kSegsPerLayer = 4;
__device__ __forceinline__ void seg_of(const ModelW& w, const Rows& r, int k, const char*& p, uint32_t& bytes) {
    auto rows_of = [](const float* m, int r0, int r1, int width) {  // matrix rows [r0, r1) of `width` weights
        return reinterpret_cast<const char*>(m) + (size_t)r0 * width * kWBytes;
    };
    if (k < kSegsPerLayer * w.layers) {
        const LayerW& lw = w.layer[k / kSegsPerLayer];
        switch (k % kSegsPerLayer) {
            case 0: p = rows_of(lw.w_qkv, r.q0, r.q1, kWidth); bytes = uint32_t(r.q1 - r.q0) * kRowBytes; break;
            case 1: p = rows_of(lw.w_o, r.o0, r.o1, kWidth); bytes = uint32_t(r.o1 - r.o0) * kRowBytes; break;
            case 2: p = rows_of(lw.w_fc, r.f0, r.f1, kWidth); bytes = uint32_t(r.f1 - r.f0) * kRowBytes; break;
            default: p = rows_of(lw.w_mp, r.o0, r.o1, kFfn); bytes = uint32_t(r.o1 - r.o0) * kFfn * kWBytes; break;
        }
    } else {
        p = rows_of(w.w_head, r.h0, r.h1, kWidth);
        bytes = uint32_t(r.h1 - r.h0) * kRowBytes;
    }
}

__device__ __forceinline__ int segs_per_step(const ModelW& w) { return kSegsPerLayer * w.layers + 1; }

// Schedule position of the L2 prefetch that runs ahead of the ring.
struct PfCursor {
    int step, k;
    uint32_t off, seg_bytes;
    unsigned long long pos;  // schedule bytes passed so far
    const char* p;
    uint64_t policy;
};

constexpr uint32_t kPfChunk = 32768;
constexpr unsigned long long kPfAhead = 256ull * 1024;  // bytes of schedule kept in flight beyond the ring

// Moves the prefetch cursor by one chunk (issuing cp.async.bulk.prefetch.L2
// for it when `issue`); false at the end of the schedule.
__device__ __forceinline__ bool pf_advance(const ModelW& w, const Rows& rows, int k0, int k1, int n_steps,
                                           PfCursor& c, bool issue) {
    while (c.off >= c.seg_bytes) {  // next non-empty segment
        c.off = 0;
        if (++c.k >= k1) {
            c.k = k0;
            if (++c.step >= n_steps) return false;
        }
        seg_of(w, rows, c.k, c.p, c.seg_bytes);
    }
    const uint32_t n = min(c.seg_bytes - c.off, kPfChunk);
    if (issue)
        asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(c.p + c.off), "r"(n),
                     "l"(c.policy)
                     : "memory");
    c.off += n;
    c.pos += n;
    return true;
}

// Bounded wait of the producer for a slot's previous use to be handed back;
// while it waits it keeps the L2 prefetch kPfAhead bytes ahead of the ring.
// False when the consumers raised `stop`, on an error status or on timeout.
// The schedule can outlast the consumers (a loop that ends on the stop code),
// so `stop` is checked after every try, and each try sleeps at most ~1 us.
__device__ bool wait_empty(Ring& R, int s, uint32_t parity, const DecodeArgs& a, uint32_t j, const ModelW& w,
                           const Rows& rows, int k0, int k1, int n_steps, PfCursor& pf, unsigned long long issued) {
    if (mbar_try_wait_hint(&R.empty[s], parity, 1000)) return true;
    int* status = a.b.ctl->status;
    const unsigned long long t0 = globaltimer_ns();
    bool more = true;
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait_hint(&R.empty[s], parity, 1000)) return true;
        if (R.stop) return false;
        if (more && pf.pos < issued + kPfAhead) {
            more = pf_advance(w, rows, k0, k1, n_steps, pf, pf.pos >= issued);
            continue;
        }
        if ((i & 63u) == 0) {
            const unsigned long long dt = globaltimer_ns() - t0;
            if (dt > kStatusPollNs && ld_volatile(status) != 0) return false;
            if (dt > wait_limit(a)) {
                set_status(status, kStatusRingTimeout, 900, (int)j);
                return false;
            }
        }
    }
}

// Producer warp (lane 0): issues segments [k0, k1) of each of n_steps forward
// steps into the ring, one bulk copy per slot, waiting for a slot's previous
// use to be handed back before reusing it and for the copy kInFlight slots
// back to have landed before issuing the next.
__device__ void producer(const DecodeArgs& a, const ModelW& w, Ring& R, const Rows& rows, int k0, int k1, int n_steps) {
    uint32_t j = 0, parity = 0;
    int s = 0;
    unsigned long long issued = 0;  // schedule bytes issued into the ring
    const uint64_t policy = evict_first_policy();
    PfCursor pf{0, k0 - 1, 0, 0, 0, nullptr, policy};
    for (int step = 0; step < n_steps; ++step) {
        for (int k = k0; k < k1; ++k) {
            const char* p;
            uint32_t bytes;
            seg_of(w, rows, k, p, bytes);
            for (uint32_t off = 0; off < bytes; off += kSlotBytes) {
                const uint32_t n = min(bytes - off, (uint32_t)kSlotBytes);
                if (j >= kInFlight) {  // that slot is still in the ring (kInFlight < kSlots)
                    const uint32_t jp = j - kInFlight;
                    if (!mbar_wait_bounded(&R.full[jp % kSlots], (jp / kSlots) & 1u, a, 901)) goto done;
                }
                if (j >= kSlots &&
                    !wait_empty(R, s, parity ^ 1u, a, j, w, rows, k0, k1, n_steps, pf, issued))
                    goto done;
                mbar_expect_tx(&R.full[s], n);
                bulk_g2s(R.data[s], p + off, n, &R.full[s], policy);
                issued += n;
                ++j;
                R.issued = j;
                if (++s == kSlots) {
                    s = 0;
                    parity ^= 1u;
                }
            }
        }
    }
done:
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
        mbar_init(&R.empty[i], kWarps);
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
    uint32_t k;       // slots consumed so far (uniform across the consumers)
    bool resident;    // persistent kernel: sm.xin survives from phase A to phase C
    const uint32_t* seen;  // persistent generate loop: the sampler's history set (else null)
};

// Every consumer thread waits for the next slot; `ok` is warp-uniform.
__device__ __forceinline__ const float* slot_wait(Ctx& cx, bool& ok, int where) {
    const int s = cx.k % kSlots;
    ok = mbar_wait_bounded(&cx.R.full[s], (cx.k / kSlots) & 1u, cx.a, where);
    ok = __all_sync(0xffffffffu, ok);
    return reinterpret_cast<const float*>(cx.R.data[s]);
}

// After this warp's last read of the slot: lane 0 hands the warp's share back
// (the empty barrier completes when all 16 consumer warps have arrived, so
// warps run through the ring independently of one another).
__device__ __forceinline__ void slot_release(Ctx& cx) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&cx.R.empty[cx.k % kSlots]);
    ++cx.k;
}

// Input-vector layout of the 1280-wide GEMVs: the kWarpsPerRow warps of a
// row hold the whole vector once (kVec float2 per lane).
// Column of x[j].x in the warp's block: consecutive 8-byte weight loads of a
// warp cover 64 fp32 or 128 bf16 columns.
__device__ __forceinline__ int lane_col(int j) {
#if ITTS_WBF16
    return 4 * (threadIdx.x & 31) + 128 * (j >> 1) + 2 * (j & 1);
#else
    return 2 * (threadIdx.x & 31) + 64 * j;
#endif
}
__device__ __forceinline__ int col_of(int j) { return kColsPerWarp * ((threadIdx.x >> 5) % kWarpsPerRow) + lane_col(j); }

// Chan et al.'s pairwise update of (mean, M2) for two halves of equal size n.
__device__ __forceinline__ void chan_merge(float& m, float& M2, float mb, float M2b, float n) {
    const float d = mb - m;
    m = m + 0.5f * d;
    M2 = (M2 + M2b) + d * d * (0.5f * n);
}

// LayerNorm of the vector in `x`, gamma/beta at g/b (shared memory), eps
// inside the root (kernels.metal:618-669).  Every group of kWarpsPerRow warps
// holds the whole vector, so each group computes the statistics on its own:
// per-thread mean and centred sum of squares, merged pairwise across lanes
// and then across the group's warps (one group barrier), the same operations
// in the same order in every group.
__device__ void layernorm2(float2 (&x)[kVec], const float2 (&g)[kVec], const float2 (&b)[kVec], float (*wstat)[2]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < kVec; ++j) m += x[j].x + x[j].y;
    m *= 1.0f / (2 * kVec);
    float M2 = 0.f;
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        const float a = x[j].x - m, c = x[j].y - m;
        M2 = fmaf(a, a, M2);
        M2 = fmaf(c, c, M2);
    }
    float n = 2 * kVec;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {  // lanes: (l, l^o) with the lower lane first
        const float mo = __shfl_xor_sync(0xffffffffu, m, o), M2o = __shfl_xor_sync(0xffffffffu, M2, o);
        if (lane & o) {
            float mm = mo, MM = M2o;
            chan_merge(mm, MM, m, M2, n);
            m = mm;
            M2 = MM;
        } else {
            chan_merge(m, M2, mo, M2o, n);
        }
        n *= 2.f;
    }
    if (lane == 0) {
        wstat[warp][0] = m;
        wstat[warp][1] = M2;
    }
    const int grp = warp / kWarpsPerRow, w0 = grp * kWarpsPerRow;
    if (kWarpsPerRow > 1)
        asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "n"(32 * kWarpsPerRow) : "memory");
    else
        __syncwarp();
    float gm[kWarpsPerRow], gM[kWarpsPerRow];
#pragma unroll
    for (int i = 0; i < kWarpsPerRow; ++i) {
        gm[i] = wstat[w0 + i][0];
        gM[i] = wstat[w0 + i][1];
    }
#pragma unroll
    for (int k = 1; k < kWarpsPerRow; k <<= 1) {  // warps of the group, pairwise tree
#pragma unroll
        for (int q = 0; q < kWarpsPerRow; q += 2 * k) chan_merge(gm[q], gM[q], gm[q + k], gM[q + k], n);
        n *= 2.f;
    }
    const float mean = gm[0], var = gM[0] * (1.0f / kWidth);
    const float inv = 1.0f / sqrtf(var + kLnEps);
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        x[j].x = (x[j].x - mean) * inv * g[j].x + b[j].x;
        x[j].y = (x[j].y - mean) * inv * g[j].y + b[j].y;
    }
}

// A LayerNorm's gamma and beta at this lane's GEMV columns, loaded into
// registers when a phase starts waiting for its input (they do not depend on it).
__device__ __forceinline__ void ln_load(const float* g, const float* b, float2 (&gv)[kVec], float2 (&bv)[kVec]) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        const int c = col_of(j);
        gv[j] = __ldg(reinterpret_cast<const float2*>(g + c));
        bv[j] = __ldg(reinterpret_cast<const float2*>(b + c));
    }
}


// Slots per phase and CTA for grids of 129..148 CTAs (the host requires
// ceil(8194 / grid) <= 64): c_attn 30 rows, c_proj 10, c_fc 40, mlp.c_proj 10
// long rows, mel_head 64 rows.  The slot loop of each phase is unrolled to
// exactly its bound, which keeps the kernel's code (and its instruction-cache
// footprint per layer) small.
constexpr int kSlotsQkv = (30 + kRowsPerSlot - 1) / kRowsPerSlot;
constexpr int kSlotsO = (10 + kRowsPerSlot - 1) / kRowsPerSlot;
constexpr int kSlotsFc = (40 + kRowsPerSlot - 1) / kRowsPerSlot;
constexpr int kSlotsMp = (10 + kLongPerSlot - 1) / kLongPerSlot;
constexpr int kSlotsHead = (64 + kRowsPerSlot - 1) / kRowsPerSlot;

// Dot products of x with `nrows` streamed rows of kRowLen floats (kRowsPer
// per slot, kWPR warps per row).  Each warp keeps one partial per slot in a
// register and the butterflies of all slots run together after the last one,
// so a slot costs its wait, loads, FMAs and release; block sums go to
// red[row * kWPR + block].
template <int kRowLen, int kRowsPer, int kWPR, int kMaxSlots>
__device__ bool stream_dots(Ctx& cx, int nrows, const float2 (&x)[kVec], float* red, int where) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rr = warp / kWPR, q = warp % kWPR;
    float acc[kMaxSlots];
    bool ok = true;
#pragma unroll
    for (int si = 0; si < kMaxSlots; ++si) {
        acc[si] = 0.f;
        const int r0 = si * kRowsPer;
        if (r0 < nrows && ok) {
            const float* slot = slot_wait(cx, ok, where);
            if (ok) {
                if (r0 + rr < nrows) {
                    const wtype* row = reinterpret_cast<const wtype*>(slot) + rr * kRowLen + q * kColsPerWarp;
                    float a0 = 0.f, a1 = 0.f;
#if ITTS_WBF16
                    const uint2* w = reinterpret_cast<const uint2*>(row) + lane;
#pragma unroll
                    for (int j = 0; j < kVec; j += 2) {  // 4 bf16: widened by placing them in the high half
                        const uint2 raw = w[(j >> 1) * 32];
                        a0 = fmaf(__uint_as_float(raw.x << 16), x[j].x, a0);
                        a1 = fmaf(__uint_as_float(raw.x & 0xffff0000u), x[j].y, a1);
                        a0 = fmaf(__uint_as_float(raw.y << 16), x[j + 1].x, a0);
                        a1 = fmaf(__uint_as_float(raw.y & 0xffff0000u), x[j + 1].y, a1);
                    }
#else
                    const float2* w = reinterpret_cast<const float2*>(row) + lane;
#pragma unroll
                    for (int j = 0; j < kVec; ++j) {
                        const float2 wv = w[j * 32];
                        a0 = fmaf(wv.x, x[j].x, a0);
                        a1 = fmaf(wv.y, x[j].y, a1);
                    }
#endif
                    acc[si] = a0 + a1;
                }
                slot_release(cx);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int si = 0; si < kMaxSlots; ++si) acc[si] += __shfl_xor_sync(0xffffffffu, acc[si], o);
    if (lane == 0)
#pragma unroll
        for (int si = 0; si < kMaxSlots; ++si) {
            const int r = si * kRowsPer + rr;
            if (r < nrows) red[r * kWPR + q] = acc[si];
        }
    return ok;
}

// y[row] = W[row, :] . x for `nrows` streamed 1280-wide rows; epi(row, y)
// runs on consumer thread `row` once all slots are consumed.
template <int kMaxSlots, class Epi>
__device__ bool gemv_slots(Ctx& cx, int nrows, const float2 (&x)[kVec], int where, Epi epi) {
    const bool ok = stream_dots<kWidth, kRowsPerSlot, kWarpsPerRow, kMaxSlots>(cx, nrows, x, &cx.sm.rowred[0][0], where);
    if (csync_or(!ok)) return false;
    const int t = threadIdx.x;
    if (t < nrows) {
        const float* s = cx.sm.rowred[t];
        float v = s[0];
#pragma unroll
        for (int i = 1; i < kWarpsPerRow; ++i) v += s[i];
        epi(t, v);
    }
    return true;
}

// ------------------------------------------------------ tagged hand-offs
// A value handed to other CTAs is one 64-bit word (epoch << 32 | float bits)
// stored with a single-copy-atomic relaxed store; the reader polls the words
// it needs until all carry the epoch it wants, so the data is its own flag and
// no grid barrier separates the phases of a layer.  Epoch of in-step layer l
// of forward step i of a launch: i * layers + l + 1 (0: cleared memory).
__device__ __forceinline__ void put_tagged(unsigned long long* p, uint32_t epoch, float v) {
    const unsigned long long w = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_tagged2(const unsigned long long* p) {
    ulonglong2 v;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool has_tag(unsigned long long w, uint32_t epoch) { return uint32_t(w >> 32) == epoch; }
__device__ __forceinline__ float tagged_value(unsigned long long w) { return __uint_as_float(uint32_t(w)); }

// Polls words p[0..2n) (n 16-byte pairs from p, stride 2) until all carry
// `epoch`; bounded like every wait (false on timeout or an error status).
__device__ bool poll_tagged(const unsigned long long* p, int n, uint32_t epoch, float* out, const DecodeArgs& a,
                            int where) {
    int* status = a.b.ctl->status;
    ulonglong2 v[2];
    for (int i = 0; i < n; ++i) v[i] = ld_tagged2(p + 2 * i);
    unsigned long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
        bool ready = true;
        for (int i = 0; i < n; ++i) ready = ready && has_tag(v[i].x, epoch) && has_tag(v[i].y, epoch);
        if (ready) break;
        if (it == 0) t0 = globaltimer_ns();
        if ((it & 15u) == 15u) {
            const unsigned long long dt = globaltimer_ns() - t0;
            if (dt > kStatusPollNs && ld_volatile(status) != 0) return false;
            if (dt > wait_limit(a)) {
                set_status(status, kStatusBarrierTimeout, where, (int)epoch);
                return false;
            }
        }
        for (int i = 0; i < n; ++i)
            if (!(has_tag(v[i].x, epoch) && has_tag(v[i].y, epoch))) v[i] = ld_tagged2(p + 2 * i);
    }
    for (int i = 0; i < n; ++i) {
        out[2 * i] = tagged_value(v[i].x);
        out[2 * i + 1] = tagged_value(v[i].y);
    }
    return true;
}

// Stages a tagged 1280-vector in shared memory (threads < 320, four words
// each); the caller's next consumer barrier publishes it.  False on abort.
__device__ __forceinline__ bool stage_tagged(const unsigned long long* src, uint32_t epoch, float* dst,
                                             const DecodeArgs& a, int where) {
    const int t = threadIdx.x;
    if (t >= kWidth / 4) return true;
    float v[4];
    if (!poll_tagged(src + 4 * t, 2, epoch, v, a, where)) return false;
    *reinterpret_cast<float4*>(dst + 4 * t) = make_float4(v[0], v[1], v[2], v[3]);
    return true;
}

// The residual stream entering in-step layer `li` (li = layers: the input of
// the head), staged in shared memory: li = 0 the token embedding
// (gpt_build_current, kernels.metal:1310-1325), the prefill's last hidden row
// for the prefill head, otherwise the previous layer's output h.
__device__ __forceinline__ bool stage_resid(const DecodeArgs& a, const ModelW& w, int li, uint32_t epoch,
                                            uint32_t token, uint32_t pos, float* dst, int where) {
    const int t = threadIdx.x;
    if (t >= kWidth / 4) return true;
    if (a.head_src && li == w.layers) {
        reinterpret_cast<float4*>(dst)[t] = __ldcg(reinterpret_cast<const float4*>(a.head_src) + t);
    } else if (li == 0) {
        const float4 e = __ldg(reinterpret_cast<const float4*>(w.mel_emb + (size_t)token * kWidth) + t);
        const float4 p = __ldg(reinterpret_cast<const float4*>(w.mel_pos + (size_t)pos * kWidth) + t);
        reinterpret_cast<float4*>(dst)[t] = make_float4(e.x + p.x, e.y + p.y, e.z + p.z, e.w + p.w);
    } else {
        return stage_tagged(a.b.h, epoch - 1, dst, a, where);
    }
    return true;
}

// x in the GEMV layout from a staged vector.
__device__ __forceinline__ void gather_x(const float* v, float2 (&x)[kVec]) {
#pragma unroll
    for (int j = 0; j < kVec; ++j) x[j] = *reinterpret_cast<const float2*>(v + col_of(j));
}

// Input-vector layout of the 5120-wide GEMV (mlp.c_proj over f).
__device__ __forceinline__ int long_col_of(int j) {
    return kColsPerWarp * ((threadIdx.x >> 5) % kWarpsPerLong) + lane_col(j);
}

// y[row] = W[row, :] . f for `nrows` streamed 5120-wide rows (kLongPerSlot
// per slot); epi(row, y) runs on thread `row` once all slots are consumed.
template <class Epi>
__device__ bool gemv_long_slots(Ctx& cx, int nrows, const float2 (&x)[kVec], int where, Epi epi) {
    const bool ok = stream_dots<kFfn, kLongPerSlot, kWarpsPerLong, kSlotsMp>(cx, nrows, x, &cx.sm.longred[0][0], where);
    if (csync_or(!ok)) return false;
    const int t = threadIdx.x;
    if (t < nrows) {
        const float* s = cx.sm.longred[t];
        float v[kWarpsPerLong / 2];
#pragma unroll
        for (int i = 0; i < kWarpsPerLong / 2; ++i) v[i] = s[2 * i] + s[2 * i + 1];
#pragma unroll
        for (int w = kWarpsPerLong / 4; w >= 1; w >>= 1)
#pragma unroll
            for (int i = 0; i < w; ++i) v[i] = v[2 * i] + v[2 * i + 1];
        epi(t, v[0]);
    }
    return true;
}

// ---------------------------------------------------------------- phases
// Key chunk of one attention unit: a multiple of 16 keys, at most kMaxChunks
// chunks per head, about one unit per CTA.
__device__ __forceinline__ uint32_t attn_chunk(uint32_t keys, int ncta) {
    uint32_t ch = (keys * kHeads + ncta - 1) / ncta;
    ch = max(ch, (keys + kMaxChunks - 1) / kMaxChunks);
    return max((ch + 15u) & ~15u, 16u);
}

// Thread 0: starts fetching the cached K/V rows of this CTA's attention units
// (keys [k0, min(k1, S)) of phase B, written in earlier steps) into L2 while
// phase A runs, so phase B's loads hit L2.
__device__ __forceinline__ void prefetch_attn_kv(const Ctx& cx, int li, uint32_t S) {
    const uint32_t keys = S + 1;
    const uint32_t ch = attn_chunk(keys, cx.ncta);
    const uint32_t nch = (keys + ch - 1) / ch, units = kHeads * nch;
    for (uint32_t u = cx.cta; u < units; u += cx.ncta) {
        const uint32_t h = u / nch, k0 = (u % nch) * ch, k1 = min(k0 + ch, S);
        if (k1 <= k0) continue;
        const uint32_t bytes = (k1 - k0) * kHeadDim * 4;
        for (int kv = 0; kv < 2; ++kv) {
            const float* src = cx.a.b.kv + (((size_t)li * 2 + kv) * kHeads + h) * (size_t)kKvCapacity * kHeadDim +
                               (size_t)k0 * kHeadDim;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
        }
    }
}

__device__ bool phase_qkv(Ctx& cx, int li, uint32_t epoch, uint32_t token, uint32_t pos, uint32_t S) {
    if (threadIdx.x == 0) prefetch_attn_kv(cx, li, S);
    const DecodeArgs& a = cx.a;
    const int t = threadIdx.x, r0 = cx.rows.q0, nrows = cx.rows.q1 - r0;
    const float bias = t < nrows ? __ldg(cx.w.layer[li].b_qkv + r0 + t) : 0.f;  // used after the last slot
    const LayerW& lw = cx.w.layer[li];
    float2 gv[kVec], bv[kVec];
    ln_load(lw.ln1_g, lw.ln1_b, gv, bv);
    const bool staged = stage_resid(a, cx.w, li, epoch, token, pos, cx.sm.xin, 10 + li);  // kept for phase C
    if (csync_or(!staged)) return false;
    float2 x[kVec];
    gather_x(cx.sm.xin, x);
    layernorm2(x, gv, bv, cx.sm.wstat);
    unsigned long long* out = a.b.qkv + r0;
    return gemv_slots<kSlotsQkv>(cx, nrows, x, 40 + li, [&](int row, float v) { put_tagged(out + row, epoch, v + bias); });
}

// Split-K attention for the current query over keys [0, S] (S cached + the
// current key), kernels.metal:2064-2145.  Unit = (head, chunk of ch keys);
// warp w takes keys w, w+16, ... of the chunk with an online softmax over
// blocks of 8 keys (their K and V rows fetched together); the 16 warp states are merged into one partial (max,
// sum, 64 outputs).  The unit holding key S appends this token's K/V to the
// cache.  A per-head arrival counter (acq_rel) finds the last unit of a head,
// which merges the head's partials and hands the 64 outputs on as tagged
// words; the others go straight on to phase C.
__device__ bool phase_attn(Ctx& cx, int li, uint32_t epoch, uint32_t S) {
    const DecodeArgs& a = cx.a;
    const uint32_t keys = S + 1;
    const uint32_t ch = attn_chunk(keys, cx.ncta);
    const uint32_t nch = (keys + ch - 1) / ch, units = kHeads * nch;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    float* qkv = cx.sm.qkvh;
    for (uint32_t u = cx.cta; u < units; u += cx.ncta) {
        const uint32_t h = u / nch, c = u % nch, k0 = c * ch, k1 = min(k0 + ch, keys);
        float* Kc = a.b.kv + (((size_t)li * 2 + 0) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
        float* Vc = a.b.kv + (((size_t)li * 2 + 1) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
        bool ok = true;
        if (t < 48) {  // q, k, v of head h: 3 x 16 threads x 4 words
            const int part = t >> 4, q4 = t & 15;
            float v[4];
            ok = poll_tagged(a.b.qkv + part * kWidth + h * kHeadDim + 4 * q4, 2, epoch, v, a, 60 + li);
            *reinterpret_cast<float4*>(qkv + part * kHeadDim + 4 * q4) = make_float4(v[0], v[1], v[2], v[3]);
        }
        if (csync_or(!ok)) return false;
        const float* kcur = qkv + kHeadDim;
        const float* vcur = qkv + 2 * kHeadDim;
        const float2 q = *reinterpret_cast<const float2*>(qkv + 2 * lane);
        float m = -INFINITY, l = 0.f;
        float2 o = make_float2(0.f, 0.f);
        constexpr int kKB = 8;  // keys per warp per online-softmax block: all their K/V loads in flight at once
        for (uint32_t kb = k0 + warp; kb < k1; kb += kKB * kWarps) {
            float2 kv[kKB], vv[kKB];
            float sk[kKB];
#pragma unroll
            for (int i = 0; i < kKB; ++i) {
                const uint32_t kk = kb + i * kWarps;
                if (kk < k1) {
                    if (kk < S) {
                        kv[i] = __ldcg(reinterpret_cast<const float2*>(Kc + (size_t)kk * kHeadDim) + lane);
                        vv[i] = __ldcg(reinterpret_cast<const float2*>(Vc + (size_t)kk * kHeadDim) + lane);
                    } else {
                        kv[i] = *reinterpret_cast<const float2*>(kcur + 2 * lane);
                        vv[i] = *reinterpret_cast<const float2*>(vcur + 2 * lane);
                    }
                } else {
                    kv[i] = vv[i] = make_float2(0.f, 0.f);
                }
            }
#pragma unroll
            for (int i = 0; i < kKB; ++i) sk[i] = fmaf(q.x, kv[i].x, q.y * kv[i].y);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int i = 0; i < kKB; ++i) sk[i] += __shfl_xor_sync(0xffffffffu, sk[i], off);
            float mn = m;
#pragma unroll
            for (int i = 0; i < kKB; ++i) {
                sk[i] = kb + i * kWarps < k1 ? sk[i] * 0.125f : -INFINITY;  // rsqrt(64)
                mn = fmaxf(mn, sk[i]);
            }
            const float corr = expf(m - mn);
            l *= corr;
            o.x *= corr;
            o.y *= corr;
#pragma unroll
            for (int i = 0; i < kKB; ++i) {
                const float p = expf(sk[i] - mn);
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
            float* pp = a.b.part + ((size_t)h * nch + c) * kPartStride;
            pp[4 + t] = O;
            if (t == 0) {
                pp[0] = M;
                pp[1] = Ls;
            }
        }
        if (c == nch - 1) {
            if (t >= 64 && t < 128)
                Kc[(size_t)S * kHeadDim + t - 64] = kcur[t - 64];
            else if (t >= 128 && t < 192)
                Vc[(size_t)S * kHeadDim + t - 128] = vcur[t - 128];
        }
        csync();
        if (t == 0) {
            unsigned* cnt = &a.b.ctl->head_cnt[li][h];
            unsigned old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
            const bool last = old == nch - 1;
            // reused in the next step, after its grid barrier
            if (last) *reinterpret_cast<volatile unsigned*>(cnt) = 0;
            cx.sm.last = last;
        }
        csync();
        if (cx.sm.last) {  // last unit of head h: merge its partials
            if (t < kHeadDim) {
                const float* ph = a.b.part + (size_t)h * nch * kPartStride;
                float mv[kMaxChunks], lv[kMaxChunks], ov[kMaxChunks];
#pragma unroll
                for (int cc = 0; cc < kMaxChunks; ++cc)
                    if (cc < (int)nch) {
                        mv[cc] = __ldcg(ph + cc * kPartStride);
                        lv[cc] = __ldcg(ph + cc * kPartStride + 1);
                        ov[cc] = __ldcg(ph + cc * kPartStride + 4 + t);
                    }
                float M = -INFINITY;
#pragma unroll
                for (int cc = 0; cc < kMaxChunks; ++cc)
                    if (cc < (int)nch) M = fmaxf(M, mv[cc]);
                float Ls = 0.f, O = 0.f;
#pragma unroll
                for (int cc = 0; cc < kMaxChunks; ++cc)
                    if (cc < (int)nch) {
                        const float e = expf(mv[cc] - M);
                        Ls = fmaf(e, lv[cc], Ls);
                        O = fmaf(e, ov[cc], O);
                    }
                put_tagged(a.b.attn + h * kHeadDim + t, epoch, O / Ls);
            }
        }
        csync();
    }
    return true;
}

__device__ bool phase_oproj(Ctx& cx, int li, uint32_t epoch, uint32_t token, uint32_t pos) {
    const DecodeArgs& a = cx.a;
    const int r0 = cx.rows.o0, nrows = cx.rows.o1 - r0;
    const int t = threadIdx.x;
    float bias = 0.f, res = 0.f;  // used after the last slot
    bool ok = true;
    if (t < nrows) {
        const int r = r0 + t;
        bias = __ldg(cx.w.layer[li].b_o + r);
        if (cx.resident) {
            res = cx.sm.xin[r];
        } else if (li == 0) {  // layered path: the layer input from global memory
            res = __ldg(cx.w.mel_emb + (size_t)token * kWidth + r) + __ldg(cx.w.mel_pos + (size_t)pos * kWidth + r);
        } else {
            const unsigned long long* hp = a.b.h + (r & ~1);
            float v[2];
            ok = poll_tagged(hp, 1, epoch - 1, v, a, 70 + li);
            res = v[r & 1];
        }
    }
    ok = ok && stage_tagged(a.b.attn, epoch, cx.sm.attn, a, 70 + li);
    if (csync_or(!ok)) return false;
    float2 x[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) x[j] = *reinterpret_cast<const float2*>(&cx.sm.attn[col_of(j)]);
    unsigned long long* out = a.b.hm + r0;
    return gemv_slots<kSlotsO>(cx, nrows, x, 70 + li,
                               [&](int row, float v) { put_tagged(out + row, epoch, res + (v + bias)); });
}

// hm -> LN2 -> this CTA's c_fc rows -> GELU -> f.
__device__ bool phase_fc(Ctx& cx, int li, uint32_t epoch) {
    const DecodeArgs& a = cx.a;
    const int f0 = cx.rows.f0, nf = cx.rows.f1 - f0, t = threadIdx.x;
    const float bias = t < nf ? __ldg(cx.w.layer[li].b_fc + f0 + t) : 0.f;
    const LayerW& lw = cx.w.layer[li];
    float2 gv[kVec], bv[kVec];
    ln_load(lw.ln2_g, lw.ln2_b, gv, bv);
    const bool staged = stage_tagged(a.b.hm, epoch, cx.sm.xin, a, 100 + li);
    if (csync_or(!staged)) return false;
    float2 x[kVec];
    gather_x(cx.sm.xin, x);
    layernorm2(x, gv, bv, cx.sm.wstat);
    float* out = a.b.f + f0;
    if (!gemv_slots<kSlotsFc>(cx, nf, x, 130 + li, [&](int row, float v) { out[row] = gelu_ref(v + bias); }))
        return false;
    // f is read whole by every CTA: one arrival count per layer (monotonic over
    // the steps of a launch) instead of per-word tags, so readers load it once
    csync();
    if (t == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&a.b.ctl->f_cnt[li]) : "memory");
    return true;
}

// Thread 0: bounded wait until `*cnt` reaches `target` (acquire); false on
// timeout or an error status.
__device__ bool wait_count(const unsigned* cnt, unsigned target, const DecodeArgs& a, int where) {
    if (ld_acquire_gpu(cnt) >= target) return true;
    int* status = a.b.ctl->status;
    const unsigned long long t0 = globaltimer_ns();
    for (unsigned spins = 1;; ++spins) {
        if (ld_acquire_gpu(cnt) >= target) return true;
        if ((spins & 31u) == 0) {
            const unsigned long long dt = globaltimer_ns() - t0;
            if (dt > kStatusPollNs && ld_volatile(status) != 0) return false;
            if (dt > wait_limit(a)) {
                set_status(status, kStatusBarrierTimeout, where, (int)target);
                return false;
            }
        }
    }
}

// f -> this CTA's mlp.c_proj rows (the rows of its attn.c_proj block) -> h = hm + y + bias.
__device__ bool phase_mp(Ctx& cx, int li, uint32_t epoch) {
    const DecodeArgs& a = cx.a;
    const int r0 = cx.rows.o0, nrows = cx.rows.o1 - r0, t = threadIdx.x;
    float bias = 0.f, res = 0.f;
    bool ok = true;
    if (t < nrows) {
        bias = __ldg(cx.w.layer[li].b_mp + r0 + t);
        float v[2];
        ok = poll_tagged(a.b.hm + ((r0 + t) & ~1), 1, epoch, v, a, 160 + li);
        res = v[(r0 + t) & 1];
    }
    if (t == 0) {
        const unsigned step = (epoch - 1) / unsigned(cx.w.layers);
        ok = wait_count(&a.b.ctl->f_cnt[li], unsigned(cx.ncta) * (step + 1), a, 160 + li) && ok;
    }
    if (csync_or(!ok)) return false;
    float2 x[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) x[j] = __ldcg(reinterpret_cast<const float2*>(a.b.f + long_col_of(j)));
    unsigned long long* out = a.b.h + r0;
    return gemv_long_slots(cx, nrows, x, 160 + li,
                           [&](int row, float v) { put_tagged(out + row, epoch, res + (v + bias)); });
}

// gpt.cpp:120-122: last hidden row -> ln_f -> final_norm -> mel_head.
// `epoch` is that of the last layer (whose output h is the input).
__device__ bool phase_head(Ctx& cx, uint32_t epoch, uint32_t token, uint32_t pos) {
    const DecodeArgs& a = cx.a;
    const int t = threadIdx.x, r0 = cx.rows.h0, nrows = cx.rows.h1 - r0;
    const float bias = t < nrows ? __ldg(cx.w.b_head + r0 + t) : 0.f;
    float2 gv[kVec], bv[kVec];
    ln_load(cx.w.lnf_g, cx.w.lnf_b, gv, bv);
    const bool staged = stage_resid(a, cx.w, cx.w.layers, epoch + 1, token, pos, cx.sm.xin, 200);
    if (csync_or(!staged)) return false;
    float2 x[kVec];
    gather_x(cx.sm.xin, x);
    layernorm2(x, gv, bv, cx.sm.wstat);
    ln_load(cx.w.fn_g, cx.w.fn_b, gv, bv);
    csync();  // the next LayerNorm reuses wstat
    layernorm2(x, gv, bv, cx.sm.wstat);
    float* out = a.b.logits + r0;
    // in the persistent generate loop the logits feed only the next draw: the
    // repetition penalty and temperature are applied here, one logit per thread,
    // instead of serially per thread of the sampler (sample_next passes scaled)
    const uint32_t* seen = cx.seen;
    return gemv_slots<kSlotsHead>(cx, nrows, x, 201, [&](int row, float v) {
        const float s = v + bias;
        out[row] = seen ? score_scale(s, uint32_t(r0 + row), seen, a.opts) : s;
    });
}

// Grid barrier of the persistent kernel (all CTAs co-resident by the
// cooperative launch): thread 0 adds its CTA's arrival with a release
// reduction and polls the monotonic counter with acquire loads.  The status
// word is read only when the wait is slow, so an error raised elsewhere ends
// the wait after kStatusPollNs; true when the kernel must abort.
__device__ bool grid_barrier(Ctx& cx, unsigned& target, int where) {
    target += gridDim.x;
    csync();
    if (threadIdx.x == 0) {
        unsigned* bar = &cx.a.b.ctl->bar;
        int* status = cx.a.b.ctl->status;
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
        int abort = 0;
        if (ld_acquire_gpu(bar) < target) {
            const unsigned long long t0 = globaltimer_ns();
            for (unsigned spins = 1; ld_acquire_gpu(bar) < target; ++spins) {
                if ((spins & 31u) == 0) {
                    const unsigned long long dt = globaltimer_ns() - t0;
                    if (dt > kStatusPollNs && ld_volatile(status) != 0) {
                        abort = 1;
                        break;
                    }
                    if (dt > wait_limit(cx.a)) {
                        set_status(status, kStatusBarrierTimeout, where, (int)target);
                        abort = 1;
                        break;
                    }
                }
            }
        }
        cx.sm.abort = abort;
    }
    csync();
    return cx.sm.abort != 0;
}

// One forward step (number `step` of the launch); true when aborted.  The
// layers hand their activations on as tagged words; the step's one grid
// barrier follows the head (the sampler needs every CTA's logits, and the
// barrier also publishes this step's K/V appends to the next step).
__device__ bool forward_step(Ctx& cx, int step, uint32_t token, uint32_t pos, uint32_t S, unsigned& target) {
    const int L = cx.w.layers;
    const uint32_t e0 = uint32_t(step) * uint32_t(L);
    for (int li = 0; li < L; ++li) {
        const uint32_t e = e0 + li + 1;
        if (!phase_qkv(cx, li, e, token, pos, S) || !phase_attn(cx, li, e, S) || !phase_oproj(cx, li, e, token, pos) ||
            !phase_fc(cx, li, e) || !phase_mp(cx, li, e))
            return true;
    }
    return !phase_head(cx, e0 + L, token, pos) || grid_barrier(cx, target, 1000);
}

// The sampler in its own frame, so its registers do not constrain the phases.
__device__ __noinline__ uint32_t sample_next(const float* logits, SampleOpts o, uint32_t i, SamplerSmem& sa,
                                             SamplerBig* big, int* status) {
    // draw 0 reads the prefill's raw logits; later draws read the head's scaled scores
    return run_sampler(logits, o, i, o.do_sample == 0, sa, big, nullptr, status, i > 0);
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
            if (n_fwd > 0) producer(a, sm.w, sm.ring, rows, 0, segs_per_step(sm.w), n_fwd);
            else sm.ring.producer_done = 1;
        }
        return;
    }
    sampler_init_seen(sm.sa, a.history, a.history_n);
    Ctx cx{a, sm.w, sm.ring, sm.ph, rows, cta, ncta, 0, true, a.mode == kModeGenerate ? sm.sa.seen : nullptr};
    SamplerBig* big = a.b.sampler_big + cta;
    unsigned target = 0;
    uint32_t token = a.first_code, n_codes = 0, stopped = 0, fwd = 0;
    for (uint32_t i = 0; i < a.n_iter; ++i) {
        if (a.mode == kModeGenerate) {
            token = sample_next(a.b.logits, a.opts, i, sm.sa, big, a.b.ctl->status);
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
enum LayerPhase : int { kPhQkv = 0, kPhAttn, kPhOproj, kPhFc, kPhMp, kPhHead };

__global__ void __launch_bounds__(kCtaThreads, 1) k_phase(DecodeArgs a, int phase, int li, uint32_t epoch,
                                                          uint32_t pos, uint32_t S) {
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
            // segments of this phase (see seg_of)
            int k0 = kSegsPerLayer * li, k1 = k0;
            if (phase == kPhQkv) k1 = k0 + 1;
            else if (phase == kPhOproj) k0 += 1, k1 = k0 + 1;
            else if (phase == kPhFc) k0 += 2, k1 = k0 + 1;
            else if (phase == kPhMp) k0 += 3, k1 = k0 + 1;
            else if (phase == kPhHead) k0 = kSegsPerLayer * sm.w.layers, k1 = k0 + 1;
            if (k1 > k0) producer(a, sm.w, sm.ring, rows, k0, k1, 1);
            else sm.ring.producer_done = 1;
        }
        return;
    }
    const uint32_t token = *reinterpret_cast<volatile uint32_t*>(&a.b.ctl->token);
    Ctx cx{a, sm.w, sm.ring, sm.ph, rows, cta, ncta, 0, false, nullptr};
    switch (phase) {
        case kPhQkv: phase_qkv(cx, li, epoch, token, pos, S); break;
        case kPhAttn: phase_attn(cx, li, epoch, S); break;
        case kPhOproj: phase_oproj(cx, li, epoch, token, pos); break;
        case kPhFc: phase_fc(cx, li, epoch); break;
        case kPhMp: phase_mp(cx, li, epoch); break;
        default: phase_head(cx, epoch, token, pos); break;
    }
    if (threadIdx.x == 0) ring_finish(sm.ring, cx.k);
}

// ------------------------------------------------------------ host side
size_t decode_smem_bytes() { return sizeof(DecodeSmem); }

cudaError_t decode_configure(int* blocks_per_sm) {
    cudaError_t e = cudaFuncSetAttribute(k_decode, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DecodeSmem));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_phase, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DecodeSmem));
    if (e != cudaSuccess) return e;
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
        cudaError_t e = launch_layer_sample(a, i, s);
        if (e != cudaSuccess) return e;
        ++*launches;
        if (a.mode == kModeGenerate && i + 1 == a.n_iter) break;
        const uint32_t pos = a.pos0 + i, S = a.s0 + i;
        for (int l = 0; l < layers; ++l) {
            const uint32_t epoch = i * uint32_t(layers) + uint32_t(l) + 1;
            for (int ph = kPhQkv; ph <= kPhMp; ++ph) {
                k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, ph, l, epoch, pos, S);
                ++*launches;
            }
        }
        k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, kPhHead, layers, i * uint32_t(layers) + uint32_t(layers),
                                                              pos, S);
        ++*launches;
    }
    cudaError_t e = launch_layer_finish(a, s);
    ++*launches;
    return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_head(const DecodeArgs& a, int ncta, cudaStream_t s) {
    k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, kPhHead, 0, 0, 0, 0);
    return cudaGetLastError();
}

// Layer 0's attn.c_proj phase for an epoch that no phase publishes: every CTA
// polls the attention hand-off until the launch's wait limit, records a
// timeout in the status word and returns (its ring drained).  Exercises the
// device-timeout path with a wait nothing ends, without a fault or a hang.
cudaError_t launch_wait_probe(const DecodeArgs& a, int ncta, cudaStream_t s) {
    k_phase<<<ncta, kCtaThreads, sizeof(DecodeSmem), s>>>(a, kPhOproj, 0, 0x7fffffffu, 0, 0);
    return cudaGetLastError();
}

}  // namespace ITTS_WNS
}  // namespace itts
