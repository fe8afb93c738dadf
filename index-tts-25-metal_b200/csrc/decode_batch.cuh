// Batched decode of the IndexTTS 2.5 GPT on B200 (sm_100a): M <= kMaxBatch
// independent rows (requests of generate_batch, or the hypotheses of a beam
// search) advance one token per step together, and every weight byte is read
// from HBM once per step for all rows.  Included after decode_body.cuh, so it
// is compiled once per weight type like the batch-1 kernels and shares their
// weight ring, producer warp, segment schedule and LayerNorm merge.
//
// One forward step (src/gpt.cpp:88-125, initial=false, for M rows) is five
// phases per layer plus the head, each followed by a grid-wide hand-off:
//   k_bgemv<QKV>   LN1 + c_attn rows            x    -> qkv  (and the L2
//                                                             prefetch of the K/V)
//   k_battn        split-K attention + K/V append qkv -> attn (kernels.metal:2064-2145)
//   k_bgemv<OPROJ> attn.c_proj rows + residual  attn -> hm
//   k_bgemv<FC>    LN2 + c_fc rows + GELU       hm   -> f
//   k_bgemv<MP>    mlp.c_proj rows + residual   f    -> x
// x 24 layers, then the head (ln_f -> final_norm -> mel_head) and one
// sampler per row.  Two drivers run the same phase code:
//   * k_bdecode: one cooperative launch (one CTA per SM) for many steps; the
//     producer warp streams the weights of step after step through the ring
//     while the phases meet at grid barriers, and CTA m samples row m.
//   * the layered kernels (one launch per phase, k_batch_sample for the
//     draws): diagnostic and non-cooperative path.
// Rows join and leave independently (continuous batching): a row's draw i
// happens at global step base[m] + i and feeds forward step i (mel position
// 2 + i, s0 + i cached tokens); rows that are not active are skipped by the
// attention units and the epilogues.  Per-step values live in device memory
// (BatchState).
//
// Same numbers as batch 1.  Every output of a row is computed with the
// operations, operands and order of the batch-1 kernels:
//   * GEMV: lane l of the warp on (row, column block q) accumulates the same
//     10 (fp32) or 20 (bf16) columns in the same two fma chains; the 32 lane
//     partials meet in the xor-butterfly pairing (l, l^16), (l, l^8), ...;
//     the block sums are added in q order.  The batched kernel holds the
//     inputs of kMPG rows in registers (warps split into G groups of rows),
//     so one weight load feeds kMPG rows, and the butterflies of the kMPG
//     rows run as one transposed reduction (each of the first exchanges
//     halves the values a lane carries) with the identical pairing per output.
//   * LayerNorm: the batch-1 statistics (per-thread two-pass, Chan merges in
//     the same pairing) for each row.
//   * Attention: the chunking of batch 1 (attn_chunk over the same grid); the
//     16 per-warp online softmaxes of a unit run as "virtual warps" (real
//     warp w runs virtual warp w of every unit the CTA holds) and merge in
//     warp order; the last unit of a (row, head) merges the partials in chunk
//     order.
#pragma once

namespace itts {
namespace ITTS_WNS {

// Rows whose input vectors one warp keeps in registers: kMPG x kVec float2
// (40 floats per lane for either weight type).
#if ITTS_WBF16
constexpr int kMPG = 2;
#else
constexpr int kMPG = 4;
#endif
constexpr int kLongRowsMax = kSlots * kLongPerSlot;  // 5120-wide rows a CTA can hold in its ring

// Warp split of a 1280-wide GEMV for G row groups: group g (warps
// g*WPG .. g*WPG+WPG-1) multiplies rows g*kMPG .. g*kMPG+kMPG-1; within the
// group warp (rs, q) takes column block q of slot rows rs, rs + RS, ...
template <int G>
struct BGeo {
    static constexpr int WPG = kWarps / G;
    static constexpr int RS = WPG / kWarpsPerRow;
    static constexpr int RPW = kRowsPerSlot / RS;
    static_assert(RS >= 1 && RS * kWarpsPerRow == WPG && RPW * RS == kRowsPerSlot, "batch GEMV geometry");
};

// Split-K attention units of every active row (batch-1 chunking per row),
// enumerated row-major.
struct BUnits {
    uint32_t start[kMaxBatch + 1];  // first unit of each row
    uint32_t nch[kMaxBatch], ch[kMaxBatch], S[kMaxBatch];
    uint32_t arena[kMaxBatch];      // KV arena of each row
};

// Attention scratch for P units at a time: the 16 virtual-warp states of
// each unit, its q/k/v, its (row, head, chunk).
template <int P>
struct BAttnSmem {
    float vm[P][kWarps], vl[P][kWarps];
    float vo[P][kWarps][kHeadDim];
    __align__(16) float qkvh[P][3 * kHeadDim];
    uint32_t um[2][P], uh[2][P], uc[2][P];  // (row, head, chunk) of the pass's units; two passes' worth
    int last[P];
    BUnits units;
};
constexpr int kUnitsPersistent = 4;  // per pass in k_bdecode (shares shared memory with the ring)
constexpr int kUnitsLayered = 8;     // per pass in k_battn

struct BatchSmem {
    Ring ring;
    ModelW w;
    union {
        float red[kMaxRowsPerCta][kWarpsPerRow][kMaxBatch];  // 1280-wide rows: block sums (row, q, m)
        float longred[kLongRowsMax][kWarpsPerLong][kMaxBatch];
        BAttnSmem<kUnitsPersistent> at;
        SamplerSmem sa;
    };
    float wstat[kMPG][kWarps][2];
    int abort;
};
static_assert(sizeof(BatchSmem) <= 227 * 1024, "batched decode shared memory above the sm_100 per-CTA limit");


struct BCtx {
    const BatchArgs& a;
    const ModelW& w;
    Ring& R;
    BatchSmem& sm;
    Rows rows;
    int cta, ncta;
    uint32_t k;  // slots consumed so far
};

__device__ __forceinline__ const wtype* bslot_wait(BCtx& cx, uint32_t k, bool& ok, int where) {
    const int s = k % kSlots;
    ok = mbar_wait_bounded(&cx.R.full[s], (k / kSlots) & 1u, cx.a.d, where);
    ok = __all_sync(0xffffffffu, ok);
    return reinterpret_cast<const wtype*>(cx.R.data[s]);
}
__device__ __forceinline__ void bslot_release(BCtx& cx, uint32_t k) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&cx.R.empty[k % kSlots]);
}

// Dot products of kMPG rows' inputs with one weight row: the two fma chains
// of the batch-1 GEMV for each row (fp32: float2 loads; bf16: 4 weights per
// 8-byte load, widened into the high half of an fp32 word).
__device__ __forceinline__ void row_dots(const wtype* wrow, const float2 (&x)[kMPG][kVec], float (&acc)[kMPG]) {
    const int lane = threadIdx.x & 31;
#if ITTS_WBF16
    uint2 raw[kVec / 2];
    const uint2* w = reinterpret_cast<const uint2*>(wrow) + lane;
#pragma unroll
    for (int j = 0; j < kVec; j += 2) raw[j >> 1] = w[(j >> 1) * 32];
#pragma unroll
    for (int mm = 0; mm < kMPG; ++mm) {
        float2 a = make_float2(0.f, 0.f);  // the two chains (a0, a1), one paired fma per step
#pragma unroll
        for (int j = 0; j < kVec; j += 2) {
            const uint2 r = raw[j >> 1];
            a = fma2(make_float2(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xffff0000u)), x[mm][j], a);
            a = fma2(make_float2(__uint_as_float(r.y << 16), __uint_as_float(r.y & 0xffff0000u)), x[mm][j + 1], a);
        }
        acc[mm] = a.x + a.y;
    }
#else
    float2 wv[kVec];
    const float2* w = reinterpret_cast<const float2*>(wrow) + lane;
#pragma unroll
    for (int j = 0; j < kVec; ++j) wv[j] = w[j * 32];
#pragma unroll
    for (int mm = 0; mm < kMPG; ++mm) {
        float2 a = make_float2(0.f, 0.f);  // the two chains (a0, a1), one paired fma per step
#pragma unroll
        for (int j = 0; j < kVec; ++j) a = fma2(wv[j], x[mm][j], a);
        acc[mm] = a.x + a.y;
    }
#endif
}

// The warp sums of kMPG lane partials with the pairing of the batch-1
// butterfly (l, l^16), (l, l^8), ..., (l, l^1): the first log2(kMPG)
// exchanges halve the values a lane carries (a lane keeps the rows of its
// half and adds its partner's copies of them), the rest are plain
// butterflies.  Returns the sum of row warp_sums_row() of the group.
__device__ __forceinline__ float warp_sums(const float (&v)[kMPG]) {
    const int lane = threadIdx.x & 31;
    const bool hi = lane & 16;
#if ITTS_WBF16
    float k = hi ? v[1] : v[0];
    k += __shfl_xor_sync(0xffffffffu, hi ? v[0] : v[1], 16);
    k += __shfl_xor_sync(0xffffffffu, k, 8);
#else
    float k0 = hi ? v[2] : v[0], k1 = hi ? v[3] : v[1];
    const float s0 = hi ? v[0] : v[2], s1 = hi ? v[1] : v[3];
    k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
    k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
    const bool hi8 = lane & 8;
    float k = hi8 ? k1 : k0;
    k += __shfl_xor_sync(0xffffffffu, hi8 ? k0 : k1, 8);
#endif
    k += __shfl_xor_sync(0xffffffffu, k, 4);
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}
__device__ __forceinline__ int warp_sums_row() { return (threadIdx.x & 31) >> (kMPG == 4 ? 3 : 4); }
__device__ __forceinline__ bool warp_sums_writer() { return ((threadIdx.x & 31) & (kMPG == 4 ? 7 : 15)) == 0; }

// LayerNorm of the kMPG row vectors in x (GEMV layout) with the batch-1
// statistics of layernorm2 for each: per-thread mean and centred sum of
// squares, Chan merges across lanes, then across the kWarpsPerRow warps of
// the group (one group barrier for all rows).
__device__ void layernorm_rows(float2 (&x)[kMPG][kVec], const float2 (&g)[kVec], const float2 (&b)[kVec],
                               float (*wstat)[kWarps][2]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int mm = 0; mm < kMPG; ++mm) {
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < kVec; ++j) m += x[mm][j].x + x[mm][j].y;
        m *= 1.0f / (2 * kVec);
        float M2 = 0.f;
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
            const float a = x[mm][j].x - m, c = x[mm][j].y - m;
            M2 = fmaf(a, a, M2);
            M2 = fmaf(c, c, M2);
        }
        float n = 2 * kVec;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float mo = __shfl_xor_sync(0xffffffffu, m, o), M2o = __shfl_xor_sync(0xffffffffu, M2, o);
            if (lane & o) {
                float mb = mo, Mb = M2o;
                chan_merge(mb, Mb, m, M2, n);
                m = mb;
                M2 = Mb;
            } else {
                chan_merge(m, M2, mo, M2o, n);
            }
            n *= 2.f;
        }
        if (lane == 0) {
            wstat[mm][warp][0] = m;
            wstat[mm][warp][1] = M2;
        }
    }
    const int grp = warp / kWarpsPerRow, w0 = grp * kWarpsPerRow;
    if (kWarpsPerRow > 1)
        asm volatile("bar.sync %0, %1;" ::"r"(2 + grp), "n"(32 * kWarpsPerRow) : "memory");
    else
        __syncwarp();
    float mean[kMPG], inv[kMPG];
#pragma unroll
    for (int mm = 0; mm < kMPG; ++mm) {
        float gm[kWarpsPerRow], gM[kWarpsPerRow];
#pragma unroll
        for (int i = 0; i < kWarpsPerRow; ++i) {
            gm[i] = wstat[mm][w0 + i][0];
            gM[i] = wstat[mm][w0 + i][1];
        }
        float n = 2 * kVec * 32;
#pragma unroll
        for (int k = 1; k < kWarpsPerRow; k <<= 1) {
#pragma unroll
            for (int q = 0; q < kWarpsPerRow; q += 2 * k) chan_merge(gm[q], gM[q], gm[q + k], gM[q + k], n);
            n *= 2.f;
        }
        mean[mm] = gm[0];
        const float var = gM[0] * (1.0f / kWidth);
        inv[mm] = 1.0f / sqrtf(var + kLnEps);
    }
#pragma unroll
    for (int mm = 0; mm < kMPG; ++mm)
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
            x[mm][j].x = (x[mm][j].x - mean[mm]) * inv[mm] * g[j].x + b[j].x;
            x[mm][j].y = (x[mm][j].y - mean[mm]) * inv[mm] * g[j].y + b[j].y;
        }
}

// ------------------------------------------------------------- rows
__device__ __forceinline__ uint32_t rows_active(const BatchArgs& a) {
    return (uint32_t)ld_volatile((const int*)&a.st->active);
}
// Forward step of row m whose input is the code drawn at global step gstep.
__device__ __forceinline__ uint32_t row_fwd(const BatchArgs& a, uint32_t m, uint32_t gstep) {
    return gstep - a.st->base[m];
}

// Batch row of this warp's input registers slot mm (its group's rows).
template <int G>
__device__ __forceinline__ int group_row(int mm) {
    return ((threadIdx.x >> 5) / BGeo<G>::WPG) * kMPG + mm;
}

// Input vectors of this warp's rows at its GEMV columns: src + m * stride
// (inactive rows and rows >= M read as zero).  At layer 0 the residual stream
// is the token embedding (gpt_build_current, kernels.metal:1310-1325).
template <int G>
__device__ __forceinline__ void load_rows(const BCtx& cx, const float* src, size_t stride, bool embed, uint32_t act,
                                          uint32_t gstep, float2 (&x)[kMPG][kVec]) {
#pragma unroll
    for (int mm = 0; mm < kMPG; ++mm) {
        const int m = group_row<G>(mm);
        const bool on = m < (int)cx.a.M && ((act >> m) & 1u);
        uint32_t tok = 0, pos = 0;
        if (on && embed) {
            tok = __ldcg(&cx.a.st->token[m]);
            pos = 2 + row_fwd(cx.a, m, gstep);
        }
#pragma unroll
        for (int j = 0; j < kVec; ++j) {
            const int c = col_of(j);
            if (!on) {
                x[mm][j] = make_float2(0.f, 0.f);
            } else if (embed) {
                const float2 e = __ldg(reinterpret_cast<const float2*>(cx.w.mel_emb + (size_t)tok * kWidth + c));
                const float2 p = __ldg(reinterpret_cast<const float2*>(cx.w.mel_pos + (size_t)pos * kWidth + c));
                x[mm][j] = make_float2(e.x + p.x, e.y + p.y);
            } else {
                x[mm][j] = __ldcg(reinterpret_cast<const float2*>(src + (size_t)m * stride + c));
            }
        }
    }
}

// y[row][m] = W[row, :] . x_m for `nrows` streamed 1280-wide rows and the
// active rows of the batch; epi(row, m, y) runs once all slots are consumed.
template <int G, class Epi>
__device__ bool bgemv_1280(BCtx& cx, int nrows, const float2 (&x)[kMPG][kVec], uint32_t act, int where, Epi epi) {
    using Geo = BGeo<G>;
    const int warp = threadIdx.x >> 5;
    const int wg = warp % Geo::WPG, rs = wg / kWarpsPerRow, q = wg % kWarpsPerRow;
    const int M = (int)cx.a.M;
    bool ok = true;
    const int nslots = (nrows + kRowsPerSlot - 1) / kRowsPerSlot;
#pragma unroll 1
    for (int si = 0; si < nslots && ok; ++si) {
        const wtype* slot = bslot_wait(cx, cx.k, ok, where);
        if (!ok) break;
        float acc[Geo::RPW][kMPG];
#pragma unroll
        for (int k = 0; k < Geo::RPW; ++k) {
            const int sr = rs + k * Geo::RS;
            if (si * kRowsPerSlot + sr < nrows) {
                row_dots(slot + sr * kWidth + q * kColsPerWarp, x, acc[k]);
            } else {
#pragma unroll
                for (int mm = 0; mm < kMPG; ++mm) acc[k][mm] = 0.f;
            }
        }
        bslot_release(cx, cx.k);
        ++cx.k;
#pragma unroll
        for (int k = 0; k < Geo::RPW; ++k) {
            const float v = warp_sums(acc[k]);
            const int row = si * kRowsPerSlot + rs + k * Geo::RS, m = group_row<G>(warp_sums_row());
            if (warp_sums_writer() && row < nrows && m < M) cx.sm.red[row][q][m] = v;
        }
    }
    if (csync_or(!ok)) return false;
    for (int t = threadIdx.x; t < nrows * M; t += kThreads) {
        const int row = t / M, m = t % M;
        if (!((act >> m) & 1u)) continue;
        float v = cx.sm.red[row][0][m];
#pragma unroll
        for (int i = 1; i < kWarpsPerRow; ++i) v += cx.sm.red[row][i][m];
        epi(row, m, v);
    }
    csync();  // red is reused (and shares memory with the attention and sampler scratch)
    return true;
}

// y[row][m] = W[row, :] . f_m for the CTA's `nrows` 5120-wide rows, all held
// in the ring at once: one pass over the held slots per group of kMPG rows
// (their inputs in registers, batch-1 column layout); the slots go back to
// the producer after the last pass.
template <int G, class Epi>
__device__ bool bgemv_long(BCtx& cx, int nrows, uint32_t act, int where, Epi epi) {
    const int warp = threadIdx.x >> 5;
    const int rr = warp / kWarpsPerLong, q = warp % kWarpsPerLong;
    const int M = (int)cx.a.M;
    const int nslots = (nrows + kLongPerSlot - 1) / kLongPerSlot;
    bool ok = true;
#pragma unroll 1
    for (int g = 0; g < G && ok; ++g) {
        if (g > 0 && ((act >> (g * kMPG)) & ((1u << kMPG) - 1u)) == 0) continue;  // no active row in the group
        float2 x[kMPG][kVec];
#pragma unroll
        for (int mm = 0; mm < kMPG; ++mm) {
            const int m = g * kMPG + mm;
            const bool on = m < M && ((act >> m) & 1u);
#pragma unroll
            for (int j = 0; j < kVec; ++j)
                x[mm][j] = on ? __ldcg(reinterpret_cast<const float2*>(cx.a.f + (size_t)m * kFfn + long_col_of(j)))
                              : make_float2(0.f, 0.f);
        }
#pragma unroll 1
        for (int si = 0; si < nslots; ++si) {
            const wtype* slot;
            if (g == 0) {
                slot = bslot_wait(cx, cx.k + si, ok, where);
                if (!ok) break;
            } else {
                slot = reinterpret_cast<const wtype*>(cx.R.data[(cx.k + si) % kSlots]);
            }
            const int row = si * kLongPerSlot + rr;
            float acc[kMPG];
            if (row < nrows) {
                row_dots(slot + rr * kFfn + q * kColsPerWarp, x, acc);
            } else {
#pragma unroll
                for (int mm = 0; mm < kMPG; ++mm) acc[mm] = 0.f;
            }
            const float v = warp_sums(acc);
            const int m = g * kMPG + warp_sums_row();
            if (warp_sums_writer() && row < nrows && m < M) cx.sm.longred[row][q][m] = v;
        }
    }
    // hand every held slot back (after a failed wait ring_finish drains the copies)
    if (ok) {
        for (int si = 0; si < nslots; ++si) bslot_release(cx, cx.k + si);
        cx.k += nslots;
    }
    if (csync_or(!ok)) return false;
    for (int t = threadIdx.x; t < nrows * M; t += kThreads) {
        const int row = t / M, m = t % M;
        if (!((act >> m) & 1u)) continue;
        float v[kWarpsPerLong / 2];
#pragma unroll
        for (int i = 0; i < kWarpsPerLong / 2; ++i) v[i] = cx.sm.longred[row][2 * i][m] + cx.sm.longred[row][2 * i + 1][m];
#pragma unroll
        for (int w = kWarpsPerLong / 4; w >= 1; w >>= 1)
#pragma unroll
            for (int i = 0; i < w; ++i) v[i] = v[2 * i] + v[2 * i + 1];
        epi(row, m, v[0]);
    }
    csync();
    return true;
}

// --------------------------------------------------------------- attention
__device__ __forceinline__ float* arena_kv(const BatchArgs& a, const BUnits& u, uint32_t m, int li, int kv,
                                           uint32_t h) {
    return a.kv + (size_t)u.arena[m] * a.arena_floats +
           (((size_t)li * 2 + kv) * kHeads + h) * (size_t)kKvCapacity * kHeadDim;
}

// Called by warp 0: lane m reads row m's state (one round trip for all rows),
// then lane 0 accumulates the unit offsets.
__device__ __forceinline__ void batch_units(const BatchArgs& a, int ncta, uint32_t act, uint32_t gstep, BUnits& u) {
    const uint32_t m = threadIdx.x;
    if (m < a.M) {
        u.nch[m] = u.ch[m] = u.S[m] = 0;
        u.arena[m] = a.st->arena[m];
        if ((act >> m) & 1u) {
            const uint32_t S = a.st->s0[m] + row_fwd(a, m, gstep), keys = S + 1;
            const uint32_t ch = attn_chunk(keys, ncta);
            u.S[m] = S;
            u.ch[m] = ch;
            u.nch[m] = (keys + ch - 1) / ch;
        }
    }
    __syncwarp();
    if (m == 0) {
        uint32_t acc = 0;
        for (uint32_t r = 0; r < a.M; ++r) {
            u.start[r] = acc;
            acc += kHeads * u.nch[r];
        }
        u.start[a.M] = acc;
    }
}

// Virtual warp `warp` of R units of a pass at once, when every unit's chunk
// has at most 128 / R keys (so each virtual warp meets at most 8 / R keys of a
// unit, one batch-1 block): the K/V loads of the R units share one round
// trip, kept in the same eight load registers, unit r in slots
// [r * 8 / R, (r + 1) * 8 / R).  Each unit's block is then computed exactly as
// the batch-1 loop computes it: its keys in its slots, the block's other
// slots (keys past the chunk) as zero vectors with -inf scores.
template <int R, int P>
__device__ __forceinline__ void battn_vw_packed(const BatchArgs& a, int li, BAttnSmem<P>& sm, const uint32_t* um,
                                                const uint32_t* uh, const uint32_t* uc, int i0, int np, int warp,
                                                int lane) {
    constexpr int kKB = 8, W = kKB / R;
    float2 kv[kKB], vv[kKB];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = i0 + r;
        uint32_t m = 0, h = 0, S = 0, k0 = 0, k1 = 0;
        if (i < np) {
            m = um[i];
            h = uh[i];
            const uint32_t ch = sm.units.ch[m];
            S = sm.units.S[m];
            k0 = uc[i] * ch;
            k1 = min(k0 + ch, S + 1);
        }
        const float* Kc = arena_kv(a, sm.units, m, li, 0, h);
        const float* Vc = arena_kv(a, sm.units, m, li, 1, h);
#pragma unroll
        for (int ii = 0; ii < W; ++ii) {
            const uint32_t kk = k0 + warp + ii * kWarps;
            float2 kx = make_float2(0.f, 0.f), vx = kx;
            if (i < np && kk < k1) {
                if (kk < S) {
                    kx = __ldcg(reinterpret_cast<const float2*>(Kc + (size_t)kk * kHeadDim) + lane);
                    vx = __ldcg(reinterpret_cast<const float2*>(Vc + (size_t)kk * kHeadDim) + lane);
                } else {
                    kx = *reinterpret_cast<const float2*>(sm.qkvh[i] + kHeadDim + 2 * lane);
                    vx = *reinterpret_cast<const float2*>(sm.qkvh[i] + 2 * kHeadDim + 2 * lane);
                }
            }
            kv[r * W + ii] = kx;
            vv[r * W + ii] = vx;
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int i = i0 + r;
        if (i >= np) break;
        const uint32_t m = um[i], ch = sm.units.ch[m];
        const uint32_t k0 = uc[i] * ch, k1 = min(k0 + ch, sm.units.S[m] + 1), kb = k0 + warp;
        float mx = -INFINITY, l = 0.f;
        float2 o = make_float2(0.f, 0.f);
        if (kb < k1) {  // the batch-1 loop runs once for this virtual warp
            const float2 q = *reinterpret_cast<const float2*>(sm.qkvh[i] + 2 * lane);
            float sk[kKB];
#pragma unroll
            for (int ii = 0; ii < W; ++ii) sk[ii] = fmaf(q.x, kv[r * W + ii].x, q.y * kv[r * W + ii].y);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int ii = 0; ii < W; ++ii) sk[ii] += __shfl_xor_sync(0xffffffffu, sk[ii], off);
            float mn = mx;
#pragma unroll
            for (int ii = 0; ii < kKB; ++ii) {
                sk[ii] = ii < W && kb + ii * kWarps < k1 ? sk[ii] * 0.125f : -INFINITY;
                mn = fmaxf(mn, sk[ii]);
            }
            const float corr = expf(mx - mn);
            l *= corr;
            o.x *= corr;
            o.y *= corr;
#pragma unroll
            for (int ii = 0; ii < kKB; ++ii) {
                const float p = expf(sk[ii] - mn);
                const float2 v = ii < W ? vv[r * W + ii] : make_float2(0.f, 0.f);
                l += p;
                o = fma2(make_float2(p, p), v, o);
            }
            mx = mn;
        }
        if (lane == 0) {
            sm.vm[i][warp] = mx;
            sm.vl[i][warp] = l;
        }
        sm.vo[i][warp][2 * lane] = o.x;
        sm.vo[i][warp][2 * lane + 1] = o.y;
    }
}


// Split-K attention of layer li for every active row, P units of this CTA at
// a time (kernels.metal:2064-2145; batch-1 phase_attn per unit).  Called by
// the kThreads consumer threads.
template <int P>
__device__ void battn_phase(const BatchArgs& a, int li, uint32_t act, uint32_t gstep, int cta, int ncta,
                            BAttnSmem<P>& sm) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    // Lane t < P of warp 0 finds unit t of the pass starting at unit `base`.
    auto assign = [&](uint32_t base, int b) {
        const uint32_t u = base + (uint32_t)t * ncta, total = sm.units.start[a.M];
        if (u < total) {
            uint32_t m = 0;
            while (u >= sm.units.start[m + 1]) ++m;
            const uint32_t r = u - sm.units.start[m];
            sm.um[b][t] = m;
            sm.uh[b][t] = r / sm.units.nch[m];
            sm.uc[b][t] = r % sm.units.nch[m];
        } else {
            sm.um[b][t] = 0xffffffffu;
        }
    };
    if (warp == 0) {
        batch_units(a, ncta, act, gstep, sm.units);
        __syncwarp();
        if (t < P) assign((uint32_t)cta, 0);
    }
    csync();
    const uint32_t total = sm.units.start[a.M];
    int pass = 0;
#pragma unroll 1
    for (uint32_t base = cta; base < total; base += (uint32_t)ncta * P, ++pass) {
        const int b = pass & 1;
        const uint32_t *um = sm.um[b], *uh = sm.uh[b], *uc = sm.uc[b];
        int np = 0;
        for (int i = 0; i < P; ++i) np += um[i] != 0xffffffffu;
        // q, k, v of each unit's head: 3 x 16 threads x 4 floats per unit
        if (t < np * 48) {
            const int i = t / 48, part = (t % 48) >> 4, q4 = t & 15;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.qkv + (size_t)um[i] * kQkv + part * kWidth +
                                                                    uh[i] * kHeadDim) + q4);
            *reinterpret_cast<float4*>(&sm.qkvh[i][part * kHeadDim + 4 * q4]) = v;
        }
        csync();
        // virtual warp `warp` of every unit: the batch-1 per-warp online softmax
        uint32_t chmax = 0;
        for (int i = 0; i < np; ++i) chmax = max(chmax, sm.units.ch[um[i]]);
        if (chmax <= 32) {
#pragma unroll 1
            for (int i0 = 0; i0 < np; i0 += 4) battn_vw_packed<4>(a, li, sm, um, uh, uc, i0, np, warp, lane);
        } else if (chmax <= 64) {
#pragma unroll 1
            for (int i0 = 0; i0 < np; i0 += 2) battn_vw_packed<2>(a, li, sm, um, uh, uc, i0, np, warp, lane);
        } else {
#pragma unroll 1
        for (int i = 0; i < np; ++i) {
            const uint32_t m = um[i], h = uh[i], c = uc[i];
            const uint32_t S = sm.units.S[m], ch = sm.units.ch[m], keys = S + 1;
            const uint32_t k0 = c * ch, k1 = min(k0 + ch, keys);
            const float* Kc = arena_kv(a, sm.units, m, li, 0, h);
            const float* Vc = arena_kv(a, sm.units, m, li, 1, h);
            const float* kcur = sm.qkvh[i] + kHeadDim;
            const float* vcur = sm.qkvh[i] + 2 * kHeadDim;
            const float2 q = *reinterpret_cast<const float2*>(sm.qkvh[i] + 2 * lane);
            float mx = -INFINITY, l = 0.f;
            float2 o = make_float2(0.f, 0.f);
            constexpr int kKB = 8;
            for (uint32_t kb = k0 + warp; kb < k1; kb += kKB * kWarps) {
                float2 kv[kKB], vv[kKB];
                float sk[kKB];
#pragma unroll
                for (int ii = 0; ii < kKB; ++ii) {
                    const uint32_t kk = kb + ii * kWarps;
                    if (kk < k1) {
                        if (kk < S) {
                            kv[ii] = __ldcg(reinterpret_cast<const float2*>(Kc + (size_t)kk * kHeadDim) + lane);
                            vv[ii] = __ldcg(reinterpret_cast<const float2*>(Vc + (size_t)kk * kHeadDim) + lane);
                        } else {
                            kv[ii] = *reinterpret_cast<const float2*>(kcur + 2 * lane);
                            vv[ii] = *reinterpret_cast<const float2*>(vcur + 2 * lane);
                        }
                    } else {
                        kv[ii] = vv[ii] = make_float2(0.f, 0.f);
                    }
                }
#pragma unroll
                for (int ii = 0; ii < kKB; ++ii) sk[ii] = fmaf(q.x, kv[ii].x, q.y * kv[ii].y);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int ii = 0; ii < kKB; ++ii) sk[ii] += __shfl_xor_sync(0xffffffffu, sk[ii], off);
                float mn = mx;
#pragma unroll
                for (int ii = 0; ii < kKB; ++ii) {
                    sk[ii] = kb + ii * kWarps < k1 ? sk[ii] * 0.125f : -INFINITY;
                    mn = fmaxf(mn, sk[ii]);
                }
                const float corr = expf(mx - mn);
                l *= corr;
                o.x *= corr;
                o.y *= corr;
#pragma unroll
                for (int ii = 0; ii < kKB; ++ii) {
                    const float p = expf(sk[ii] - mn);
                    l += p;
                    o = fma2(make_float2(p, p), vv[ii], o);
                }
                mx = mn;
            }
            if (lane == 0) {
                sm.vm[i][warp] = mx;
                sm.vl[i][warp] = l;
            }
            sm.vo[i][warp][2 * lane] = o.x;
            sm.vo[i][warp][2 * lane + 1] = o.y;
        }
        }
        csync();
        // merge the 16 states of each unit (warp order), write its partial, append K/V
        if (t < np * kHeadDim) {
            const int i = t / kHeadDim, d = t % kHeadDim;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm.vm[i][w]);
            float Ls = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const float e = sm.vl[i][w] > 0.f ? expf(sm.vm[i][w] - M) : 0.f;
                Ls = fmaf(e, sm.vl[i][w], Ls);
                O = fmaf(e, sm.vo[i][w][d], O);
            }
            const uint32_t m = um[i];
            float* pp = a.part + (((size_t)m * kHeads + uh[i]) * kMaxChunks + uc[i]) * kPartStride;
            pp[4 + d] = O;
            if (d == 0) {
                pp[0] = M;
                pp[1] = Ls;
            }
        }
        for (int tt = t; tt < np * 2 * kHeadDim; tt += kThreads) {
            const int i = tt / (2 * kHeadDim), r = tt % (2 * kHeadDim);
            const uint32_t m = um[i];
            if (uc[i] == sm.units.nch[m] - 1) {
                float* dst = arena_kv(a, sm.units, m, li, r / kHeadDim, uh[i]) + (size_t)sm.units.S[m] * kHeadDim;
                dst[r % kHeadDim] = sm.qkvh[i][kHeadDim + r];
            }
        }
        csync();
        if (t < np) {
            const uint32_t m = um[t];
            unsigned* cnt = a.head_cnt + ((size_t)li * kMaxBatch + m) * kHeads + uh[t];
            unsigned old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
            const bool last = old == sm.units.nch[m] - 1;
            if (last) *reinterpret_cast<volatile unsigned*>(cnt) = 0;  // next use: after a grid-wide hand-off
            sm.last[t] = last;
        }
        csync();
        if (t < np * kHeadDim) {  // last unit of (row, head): merge its partials in chunk order
            const int i = t / kHeadDim, d = t % kHeadDim;
            if (sm.last[i]) {
                const uint32_t m = um[i], h = uh[i], nch = sm.units.nch[m];
                const float* ph = a.part + ((size_t)m * kHeads + h) * kMaxChunks * kPartStride;
                float mv[kMaxChunks], lv[kMaxChunks], ov[kMaxChunks];
#pragma unroll
                for (int cc = 0; cc < kMaxChunks; ++cc)
                    if (cc < (int)nch) {
                        mv[cc] = __ldcg(ph + cc * kPartStride);
                        lv[cc] = __ldcg(ph + cc * kPartStride + 1);
                        ov[cc] = __ldcg(ph + cc * kPartStride + 4 + d);
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
                a.attn[(size_t)m * kWidth + h * kHeadDim + d] = O / Ls;
            }
        }
        if (t < P) assign(base + (uint32_t)ncta * P, b ^ 1);  // the next pass's units (the other buffer)
        csync();
    }
}

// L2 prefetch of the cached K/V rows of the attention units this CTA will run
// for layer li, issued by all consumer threads (one 128-byte line each, no
// bulk-copy queue involved) at the start of the c_attn phase, so the
// attention phase reads them from L2.
__device__ void bprefetch_kv(const BatchArgs& a, int cta, int ncta, int li, uint32_t act, uint32_t gstep,
                             BUnits& u) {
    if (threadIdx.x < 32) batch_units(a, ncta, act, gstep, u);
    csync();
    const uint32_t total = u.start[a.M];
    for (uint32_t x = cta; x < total; x += ncta) {
        uint32_t m = 0;
        while (x >= u.start[m + 1]) ++m;
        const uint32_t r = x - u.start[m], h = r / u.nch[m], c = r % u.nch[m];
        const uint32_t k0 = c * u.ch[m], k1 = min(k0 + u.ch[m], u.S[m]);
        if (k1 <= k0) continue;
        const uint32_t lines = 4 * (k1 - k0);  // K and V, two lines per 64-float row
        for (uint32_t l = threadIdx.x; l < lines; l += kThreads) {
            const uint32_t kv = l / (2 * (k1 - k0)), rem = l % (2 * (k1 - k0));
            const float* p = arena_kv(a, u, m, li, (int)kv, h) + (size_t)(k0 + (rem >> 1)) * kHeadDim + (rem & 1) * 32;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
        }
    }
}

// ------------------------------------------------------------ GEMV phases
enum BatchPhase : int { kBQkv = 0, kBOproj, kBFc, kBMp, kBHead };

// The repetition penalty and temperature of one logit (score_scale) with the
// row's history set read from global memory.
__device__ __forceinline__ float score_scale_global(float s, uint32_t i, const uint32_t* seen, const SampleOpts& o) {
    if (o.rp != 1.0f && ((__ldcg(seen + (i >> 5)) >> (i & 31)) & 1u)) s = s < 0.0f ? s * o.rp : s / o.rp;
    if (o.temperature != 1.0f) s = s / o.temperature;
    return s;
}

// One GEMV phase of layer li (li = layers: the head) for the active rows whose
// fed codes were drawn at global step gstep.  Consumer threads only.
template <int PH, int G>
__device__ bool bgemv_phase(BCtx& cx, int li, uint32_t act, uint32_t gstep) {
    const BatchArgs& a = cx.a;
    const Rows& rows = cx.rows;
    if (PH == kBQkv) {
        bprefetch_kv(a, cx.cta, cx.ncta, li, act, gstep, cx.sm.at.units);
        const LayerW& lw = cx.w.layer[li];
        float2 gv[kVec], bv[kVec], x[kMPG][kVec];
        ln_load(lw.ln1_g, lw.ln1_b, gv, bv);
        load_rows<G>(cx, a.x, kWidth, li == 0, act, gstep, x);
        layernorm_rows(x, gv, bv, cx.sm.wstat);
        const int r0 = rows.q0;
        return bgemv_1280<G>(cx, rows.q1 - r0, x, act, 40 + li, [&](int row, int m, float v) {
            a.qkv[(size_t)m * kQkv + r0 + row] = v + __ldg(lw.b_qkv + r0 + row);
        });
    } else if (PH == kBOproj) {
        const LayerW& lw = cx.w.layer[li];
        float2 x[kMPG][kVec];
        load_rows<G>(cx, a.attn, kWidth, false, act, gstep, x);
        const int r0 = rows.o0;
        return bgemv_1280<G>(cx, rows.o1 - r0, x, act, 70 + li, [&](int row, int m, float v) {
            const int r = r0 + row;
            float res;
            if (li == 0) {
                const uint32_t tok = __ldcg(&a.st->token[m]), pos = 2 + row_fwd(a, m, gstep);
                res = __ldg(cx.w.mel_emb + (size_t)tok * kWidth + r) + __ldg(cx.w.mel_pos + (size_t)pos * kWidth + r);
            } else {
                res = __ldcg(a.x + (size_t)m * kWidth + r);
            }
            a.hm[(size_t)m * kWidth + r] = res + (v + __ldg(lw.b_o + r));
        });
    } else if (PH == kBFc) {
        const LayerW& lw = cx.w.layer[li];
        float2 gv[kVec], bv[kVec], x[kMPG][kVec];
        ln_load(lw.ln2_g, lw.ln2_b, gv, bv);
        load_rows<G>(cx, a.hm, kWidth, false, act, gstep, x);
        layernorm_rows(x, gv, bv, cx.sm.wstat);
        const int f0 = rows.f0;
        return bgemv_1280<G>(cx, rows.f1 - f0, x, act, 130 + li, [&](int row, int m, float v) {
            a.f[(size_t)m * kFfn + f0 + row] = gelu_ref(v + __ldg(lw.b_fc + f0 + row));
        });
    } else if (PH == kBMp) {
        const LayerW& lw = cx.w.layer[li];
        const int r0 = rows.o0;
        return bgemv_long<G>(cx, rows.o1 - r0, act, 160 + li, [&](int row, int m, float v) {
            const int r = r0 + row;
            const float res = __ldcg(a.hm + (size_t)m * kWidth + r);
            a.x[(size_t)m * kWidth + r] = res + (v + __ldg(lw.b_mp + r));
        });
    } else {  // head: ln_f -> final_norm -> mel_head (gpt.cpp:120-122)
        float2 gv[kVec], bv[kVec], x[kMPG][kVec];
        ln_load(cx.w.lnf_g, cx.w.lnf_b, gv, bv);
        load_rows<G>(cx, a.x, kWidth, false, act, gstep, x);
        layernorm_rows(x, gv, bv, cx.sm.wstat);
        ln_load(cx.w.fn_g, cx.w.fn_b, gv, bv);
        csync();  // the next LayerNorm reuses wstat
        layernorm_rows(x, gv, bv, cx.sm.wstat);
        const int r0 = rows.h0;
        return bgemv_1280<G>(cx, rows.h1 - r0, x, act, 201, [&](int row, int m, float v) {
            const uint32_t r = r0 + row;
            const float s = v + __ldg(cx.w.b_head + r);
            a.logits[(size_t)m * kBatchLogitsStride + r] =
                a.scaled_head ? score_scale_global(s, r, a.seen + (size_t)m * kSeenWords, a.opts[m]) : s;
        });
    }
}

// ------------------------------------------------------------ layered path
// Codes fed by a layered forward step: drawn at global step st->step - 1 (the
// sampler kernel advanced st->step after its draw).
__device__ __forceinline__ uint32_t layered_gstep(const BatchArgs& a) {
    return (uint32_t)ld_volatile((const int*)&a.st->step) - 1u;
}

template <int PH, int G>
__global__ void __launch_bounds__(kCtaThreads, 1) k_bgemv(BatchArgs a, int li) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    BatchSmem& sm = *reinterpret_cast<BatchSmem*>(smem_raw);
    const uint32_t act = rows_active(a);
    if (act == 0) return;
    const int cta = blockIdx.x, ncta = gridDim.x;
    const Rows rows = cta_rows(cta, ncta);
    load_table(sm.w, a.d.w);
    if (threadIdx.x == 0) ring_init(sm.ring);
    __syncthreads();
    if (threadIdx.x >= kThreads) {  // producer warp: this phase's segment
        if (threadIdx.x == kThreads) {
            const int k0 = PH == kBHead ? kSegsPerLayer * sm.w.layers : kSegsPerLayer * li + PH;
            producer(a.d, sm.w, sm.ring, rows, k0, k0 + 1, 1);
        }
        return;
    }
    BCtx cx{a, sm.w, sm.ring, sm, rows, cta, ncta, 0};
    bgemv_phase<PH, G>(cx, li, act, layered_gstep(a));
    if (threadIdx.x == 0) ring_finish(sm.ring, cx.k);
}

__global__ void __launch_bounds__(kThreads, 1) k_battn(BatchArgs a, int li) {
    __shared__ BAttnSmem<kUnitsLayered> sm;
    const uint32_t act = rows_active(a);
    if (act == 0) return;
    battn_phase<kUnitsLayered>(a, li, act, layered_gstep(a), blockIdx.x, gridDim.x, sm);
}

// --------------------------------------------------------- persistent path
// Grid barrier of k_bdecode (all CTAs co-resident by the cooperative launch),
// as grid_barrier: release add, acquire poll by thread 0, bounded; true when
// the kernel must abort.
__device__ bool bgrid_barrier(BCtx& cx, unsigned& target, int where) {
    target += gridDim.x;
    csync();
    if (threadIdx.x == 0) {
        unsigned* bar = &cx.a.d.b.ctl->bar;
        int* status = cx.a.d.b.ctl->status;
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
                    if (dt > wait_limit(cx.a.d)) {
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

// Draw `gstep` of row m (one CTA): the processors and the token choice of the
// batch-1 loop (sample_next) on the row's logits, then the row's bookkeeping:
// code, count, stop (gpt_sampling.cpp:178-187), repetition-penalty set.  In
// its own frame so its registers do not constrain the phases.
__device__ __noinline__ void bsample_row(const BatchArgs& a, uint32_t m, uint32_t gstep, SamplerSmem& sa) {
    int* status = a.d.b.ctl->status;
    uint32_t* seen = a.seen + (size_t)m * kSeenWords;
    for (int k = threadIdx.x; k < kBits; k += kThreads) sa.seen[k] = __ldcg(seen + k);
    csync();
    const uint32_t i = gstep - a.st->base[m];
    const SampleOpts& o = a.opts[m];
    // draw 0 reads the prefill's raw logits; later draws read the head's scaled scores
    const uint32_t token = run_sampler(a.logits + (size_t)m * kBatchLogitsStride, o, i, o.do_sample == 0, sa,
                                       a.big + m, nullptr, status, a.scaled_head && i > 0);
    if (threadIdx.x == 0) {
        BatchState* st = a.st;
        const uint32_t bit = 1u << m;
        if (token == (uint32_t)kStopCode) {
            st->stopped[m] = 1;
            atomicAnd(&st->active, ~bit);
        } else if (token >= (uint32_t)kStartCode) {
            if (token != 0xffffffffu) set_status(status, kStatusInvalidCode, 300, (int)token);
            atomicAnd(&st->active, ~bit);
        } else {
            a.codes[(size_t)m * a.codes_stride + i] = token;
            st->n_codes[m] = i + 1;
            st->token[m] = token;
            atomicOr(&seen[token >> 5], 1u << (token & 31));
            if (i + 1 >= st->maxc[m]) atomicAnd(&st->active, ~bit);
        }
    }
    csync();
}

// `iters` batched steps in one cooperative launch.  With `sample`, step it
// draws the next code of every active row (CTA m samples row m) and feeds the
// codes to one forward step; it ends early once no row is active.  Without,
// one forward step feeds the codes already in the state (drawn at global step
// st->step - 1: beam search).  The producer warp streams the weights of the
// forward steps one after another through the ring.
template <int G>
__global__ void __launch_bounds__(kCtaThreads, 1) k_bdecode(BatchArgs a, uint32_t iters, int sample) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    BatchSmem& sm = *reinterpret_cast<BatchSmem*>(smem_raw);
    const int cta = blockIdx.x, ncta = gridDim.x;
    const Rows rows = cta_rows(cta, ncta);
    load_table(sm.w, a.d.w);
    if (threadIdx.x == 0) {
        sm.abort = 0;
        ring_init(sm.ring);
    }
    __syncthreads();
    if (threadIdx.x >= kThreads) {  // producer warp
        if (threadIdx.x == kThreads) producer(a.d, sm.w, sm.ring, rows, 0, segs_per_step(sm.w), (int)iters);
        return;
    }
    BCtx cx{a, sm.w, sm.ring, sm, rows, cta, ncta, 0};
    const int L = sm.w.layers;
    unsigned target = 0;
    const uint32_t step0 = (uint32_t)ld_volatile((const int*)&a.st->step);
    uint32_t draws = 0;
    for (uint32_t it = 0; it < iters; ++it) {
        uint32_t gstep = step0 - 1u;
        if (sample) {
            gstep = step0 + it;
            const uint32_t act0 = rows_active(a);
            if ((uint32_t)cta < a.M && ((act0 >> cta) & 1u)) bsample_row(a, cta, gstep, sm.sa);
            ++draws;
            if (bgrid_barrier(cx, target, 990)) break;
        }
        const uint32_t act = rows_active(a);
        if (act == 0) break;
        bool ok = true;
        for (int li = 0; li < L && ok; ++li) {
            ok = bgemv_phase<kBQkv, G>(cx, li, act, gstep) && !bgrid_barrier(cx, target, 1000 + li);
            if (!ok) break;
            battn_phase<kUnitsPersistent>(a, li, act, gstep, cta, ncta, sm.at);
            ok = !bgrid_barrier(cx, target, 1100 + li) && bgemv_phase<kBOproj, G>(cx, li, act, gstep) &&
                 !bgrid_barrier(cx, target, 1200 + li) && bgemv_phase<kBFc, G>(cx, li, act, gstep) &&
                 !bgrid_barrier(cx, target, 1300 + li) && bgemv_phase<kBMp, G>(cx, li, act, gstep) &&
                 !bgrid_barrier(cx, target, 1400 + li);
        }
        if (!ok || !bgemv_phase<kBHead, G>(cx, L, act, gstep) || bgrid_barrier(cx, target, 1500)) break;
    }
    if (threadIdx.x == 0) ring_finish(sm.ring, cx.k);
    if (sample && cta == 0 && threadIdx.x == 0) a.st->step = step0 + draws;
}

// ------------------------------------------------------------ host side
template <int PH, int G>
cudaError_t set_bgemv_smem() {
    return cudaFuncSetAttribute(k_bgemv<PH, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(BatchSmem));
}

// Row-group counts instantiated: G * kMPG >= kMaxBatch.
#if ITTS_WBF16
#define ITTS_BATCH_GROUPS(X) X(1) X(2) X(4) X(8)
#else
#define ITTS_BATCH_GROUPS(X) X(1) X(2) X(4)
#endif

cudaError_t batch_configure() {
    cudaError_t e = cudaSuccess;
#define ITTS_CFG(G)                                                                                             \
    if (e == cudaSuccess) e = set_bgemv_smem<kBQkv, G>();                                                      \
    if (e == cudaSuccess) e = set_bgemv_smem<kBOproj, G>();                                                    \
    if (e == cudaSuccess) e = set_bgemv_smem<kBFc, G>();                                                       \
    if (e == cudaSuccess) e = set_bgemv_smem<kBMp, G>();                                                       \
    if (e == cudaSuccess) e = set_bgemv_smem<kBHead, G>();                                                     \
    if (e == cudaSuccess)                                                                                      \
        e = cudaFuncSetAttribute(k_bdecode<G>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(BatchSmem));
    ITTS_BATCH_GROUPS(ITTS_CFG)
#undef ITTS_CFG
    return e;
}

template <int G>
void launch_batch_layers(const BatchArgs& a, int layers, int ncta, cudaStream_t s, uint64_t* launches) {
    const size_t smem = sizeof(BatchSmem);
    for (int l = 0; l < layers; ++l) {
        k_bgemv<kBQkv, G><<<ncta, kCtaThreads, smem, s>>>(a, l);
        k_battn<<<ncta, kThreads, 0, s>>>(a, l);
        k_bgemv<kBOproj, G><<<ncta, kCtaThreads, smem, s>>>(a, l);
        k_bgemv<kBFc, G><<<ncta, kCtaThreads, smem, s>>>(a, l);
        k_bgemv<kBMp, G><<<ncta, kCtaThreads, smem, s>>>(a, l);
        *launches += 5;
    }
    k_bgemv<kBHead, G><<<ncta, kCtaThreads, smem, s>>>(a, layers);
    *launches += 1;
}

__host__ __forceinline__ int batch_groups(uint32_t M) { return (int(M) + kMPG - 1) / kMPG; }

// Layered path: one forward step of the active rows (codes drawn at global
// step st->step - 1) through every layer and the head: 5 launches per layer + 1.
cudaError_t launch_batch_forward(const BatchArgs& a, int layers, int ncta, cudaStream_t s, uint64_t* launches) {
    if (a.M < 1 || a.M > (uint32_t)kMaxBatch) return cudaErrorInvalidValue;
    const int G = batch_groups(a.M);
    if (G <= 1) launch_batch_layers<1>(a, layers, ncta, s, launches);
    else if (G <= 2) launch_batch_layers<2>(a, layers, ncta, s, launches);
    else if (G <= 4) launch_batch_layers<4>(a, layers, ncta, s, launches);
#if ITTS_WBF16
    else launch_batch_layers<8>(a, layers, ncta, s, launches);
#endif
    return cudaGetLastError();
}

template <int G>
cudaError_t launch_bdecode(const BatchArgs& a, uint32_t iters, int sample, int ncta, cudaStream_t s) {
    BatchArgs copy = a;
    void* args[] = {&copy, &iters, &sample};
    return cudaLaunchCooperativeKernel((const void*)k_bdecode<G>, dim3(ncta), dim3(kCtaThreads), args,
                                       sizeof(BatchSmem), s);
}

// Persistent path: `iters` steps (sample = 1: draw + forward; sample = 0: one
// forward of the codes in the state) in one cooperative launch.
cudaError_t launch_batch_persistent(const BatchArgs& a, uint32_t iters, int sample, int ncta, cudaStream_t s) {
    if (a.M < 1 || a.M > (uint32_t)kMaxBatch) return cudaErrorInvalidValue;
    const int G = batch_groups(a.M);
    if (G <= 1) return launch_bdecode<1>(a, iters, sample, ncta, s);
    if (G <= 2) return launch_bdecode<2>(a, iters, sample, ncta, s);
    if (G <= 4) return launch_bdecode<4>(a, iters, sample, ncta, s);
#if ITTS_WBF16
    return launch_bdecode<8>(a, iters, sample, ncta, s);
#else
    return cudaErrorInvalidValue;
#endif
}

}  // namespace ITTS_WNS
}  // namespace itts
