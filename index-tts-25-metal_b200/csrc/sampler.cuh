// On-device logits processors and token selection for one CTA of kThreads.
//
// Restates src/gpt_sampling.cpp:
//   * apply_gpt_sampling_processors (:28-128): repetition penalty over the
//     unique history, temperature, top-k (keep every score >= the k-th largest,
//     k floored at 2 with beams), top-p (ascending (score, index) order,
//     double-precision cumulative mass, remove while <= 1 - p, keep the top 1
//     or 2);
//   * sample_gpt_token_from_logits (:130-165): double CDF scan in index order
//     over exp(score - max), first index whose cumulative mass exceeds u*total,
//     falling back to the last index with non-zero mass;
//   * greedy selection std::max_element (:180): first index of the maximum.
// Every CTA that calls this computes the same result from the same inputs
// (fixed thread mapping and reduction order), which lets the persistent
// decode kernel sample redundantly in all CTAs instead of adding a barrier.
//
// Layout: thread t owns the contiguous logits [16 t, 16 t + 16) (four float4
// loads), thread 511 also the start and stop codes 8192 and 8193, so index-
// ordered compaction is one block scan.  The k-th largest score is found by a
// 4-pass 8-bit radix select on order-preserving integer keys with warp-
// aggregated histogram updates; the top-p survivors are sorted with a bitonic
// sort of 64-bit (score key, index) words (within one warp for up to 32); the
// double-precision sums that fix the reference's rounding order run
// sequentially in thread 0 over values computed in parallel.
#pragma once

#include "common.cuh"
#include "model.hpp"

namespace itts {

constexpr int kPer = 18;  // registers per thread (16, or 18 for the last thread)
static_assert(16 * kThreads + 2 == kVocab, "sampler layout: 16 codes per thread + 2 in the last");
__device__ __forceinline__ int elem_base() { return 16 * threadIdx.x; }
__device__ __forceinline__ int elem_cnt() { return threadIdx.x == kThreads - 1 ? kVocab - 16 * (kThreads - 1) : 16; }
constexpr int kBits = (kVocab + 31) / 32;
constexpr int kSortCap = 16384;  // next power of two >= 8194
constexpr int kFast = 256;       // survivors handled entirely in shared memory

// Shared-memory part (~9.7 KB).  Up to kFast survivors are gathered, sorted and
// their exp() values cached here; larger survivor sets use SamplerBig.
struct SamplerSmem {
    uint32_t seen[kBits];
    uint32_t removed[kBits];
    uint32_t hist[256];
    uint32_t scan[32];
    float redf[32];
    uint32_t redu[32];
    uint32_t sel_bin, sel_rem, result;
    int err;
    double f_total;
    uint32_t f_idx[kFast];
    float f_s[kFast];
    unsigned long long f_key[kFast];
    double f_pr[kFast];
    double f_q[kFast];  // top-p: exp / total in ascending order
};

// Workspace for more than kFast survivors (top-p without top-k, or wide ties):
// shared memory in single-CTA kernels, a per-CTA global slice in the
// persistent decode kernel.
struct SamplerBig {
    uint32_t sv_idx[kVocab];
    float sv_s[kVocab];
    unsigned long long key[kSortCap];
};

__device__ __forceinline__ uint32_t ord_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// SplitMix64 draw number `draw` (0-based) of a stream seeded with `seed`
// (gpt_sampling.cpp:11-26: the state advances by the golden gamma per draw).
__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t draw) {
    uint64_t z = seed + (draw + 1ull) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Philox4x32-10 (Salmon et al., SC'11): counter (draw_lo, draw_hi, 0, 0),
// key (seed_lo, seed_hi); the first two output words form the draw.
__device__ __forceinline__ uint64_t philox_at(uint64_t seed, uint64_t draw) {
    uint32_t c0 = uint32_t(draw), c1 = uint32_t(draw >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = uint32_t(seed), k1 = uint32_t(seed >> 32);
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
        const uint32_t n0 = hi1 ^ c1 ^ k0, n1 = lo1, n2 = hi0 ^ c3 ^ k1, n3 = lo0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return (uint64_t(c0) << 32) | c1;
}

__device__ __forceinline__ double uniform_at(int rng, uint64_t seed, uint64_t draw) {
    const uint64_t u = rng == 1 ? philox_at(seed, draw) : splitmix64_at(seed, draw);
    return double(u >> 11) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ bool bit_get(const uint32_t* b, uint32_t i) { return (b[i >> 5] >> (i & 31)) & 1u; }

// The first two processors for one logit: repetition penalty (negative scores
// multiplied, others divided) when token i was seen, then the temperature, in
// the order and float arithmetic of run_sampler.
__device__ __forceinline__ float score_scale(float s, uint32_t i, const uint32_t* seen, const SampleOpts& o) {
    if (o.rp != 1.0f && bit_get(seen, i)) s = s < 0.0f ? s * o.rp : s / o.rp;
    if (o.temperature != 1.0f) s = s / o.temperature;
    return s;
}

// Seeds the repetition-penalty set with `hist` (tokens >= 8194 are ignored,
// gpt_sampling.cpp:38-40).
__device__ inline void sampler_init_seen(SamplerSmem& sm, const uint32_t* hist, uint32_t n) {
    for (int i = threadIdx.x; i < kBits; i += kThreads) sm.seen[i] = 0;
    csync();
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) {
        const uint32_t t = hist[i];
        if (t < (uint32_t)kVocab) atomicOr(&sm.seen[t >> 5], 1u << (t & 31));
    }
    csync();
}

__device__ inline void sampler_mark_seen(SamplerSmem& sm, uint32_t t) {
    if (threadIdx.x == 0 && t < (uint32_t)kVocab) sm.seen[t >> 5] |= 1u << (t & 31);
    csync();
}

// Exclusive block scan of v; *total receives the sum.  blockDim.x == kThreads.
__device__ inline uint32_t block_excl_scan(uint32_t v, SamplerSmem& sm, uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    csync();
    if (lane == 31) sm.scan[warp] = inc;
    csync();
    if (warp == 0) {
        uint32_t w = lane < kWarps ? sm.scan[lane] : 0, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t n = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += n;
        }
        if (lane < kWarps) sm.scan[lane] = wi - w;
        if (lane == kWarps - 1) sm.redu[0] = wi;
    }
    csync();
    *total = sm.redu[0];
    return sm.scan[warp] + inc - v;
}

// Value of the kk-th largest element (with multiplicity) over the CTA's
// scores, i.e. sorted-descending[kk-1] of std::nth_element.
__device__ inline float kth_largest(const float (&s)[kPer], int cnt, uint32_t kk, SamplerSmem& sm) {
    uint32_t prefix = 0, mask = 0, rem = kk;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = threadIdx.x; i < 256; i += kThreads) sm.hist[i] = 0;
        csync();
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const uint32_t key = ord_key(s[k]);
            const bool part = k < cnt && (key & mask) == prefix;
            const uint32_t bin = (key >> shift) & 255u;
            const unsigned act = __ballot_sync(0xffffffffu, part);
            if (act) {  // the lanes sharing the first participant's bin (most of them, as scores
                        // cluster in a few high-order bins) add with one atomic; the rest singly
                const int leader = __ffs(act) - 1;
                const uint32_t lb = __shfl_sync(0xffffffffu, bin, leader);
                const unsigned same = __ballot_sync(0xffffffffu, part && bin == lb);
                if (lane == leader) atomicAdd(&sm.hist[lb], (uint32_t)__popc(same));
                if (part && bin != lb) atomicAdd(&sm.hist[bin], 1u);
            }
        }
        csync();
        if (warp == 0) {
            uint32_t c[8], sum = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                c[e] = sm.hist[255 - 8 * lane - e];
                sum += c[e];
            }
            uint32_t inc = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t n = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += n;
            }
            const unsigned ball = __ballot_sync(0xffffffffu, inc >= rem);
            const int tl = __ffs(ball) - 1;
            if (lane == tl) {
                uint32_t acc = inc - sum;
                for (int e = 0; e < 8; ++e) {
                    if (acc + c[e] >= rem) {
                        sm.sel_bin = 255u - 8u * lane - e;
                        sm.sel_rem = rem - acc;
                        break;
                    }
                    acc += c[e];
                }
            }
        }
        csync();
        prefix |= sm.sel_bin << shift;
        mask |= 0xffu << shift;
        rem = sm.sel_rem;
        csync();
    }
    return key_float(prefix);
}

// Ascending sort of key[0..32) by warp 0 in registers; the caller publishes
// the result with a consumer barrier.
__device__ inline void warp_sort32_asc(unsigned long long* key) {
    if (threadIdx.x >= 32) return;
    const int lane = threadIdx.x;
    unsigned long long v = key[lane];
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1)
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, v, j);
            const bool keep_min = ((lane & j) == 0) == ((lane & k) == 0);
            v = keep_min ? (o < v ? o : v) : (o > v ? o : v);
        }
    key[lane] = v;
}

__device__ inline void bitonic_sort_asc(unsigned long long* key, int P) {
    for (int k = 2; k <= P; k <<= 1)
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += kThreads) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const bool asc = (i & k) == 0;
                    const unsigned long long a = key[i], b = key[ixj];
                    if ((a > b) == asc) {
                        key[i] = b;
                        key[ixj] = a;
                    }
                }
            }
            csync();
        }
}

// First index of the maximum over the scores (std::max_element semantics).
__device__ inline uint32_t block_argmax(const float (&s)[kPer], int base, int cnt, SamplerSmem& sm) {
    float bv = -INFINITY;
    uint32_t bi = 0xffffffffu;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt && (s[k] > bv || bi == 0xffffffffu)) {
            bv = s[k];
            bi = base + k;
        }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != 0xffffffffu && (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi))) {
            bv = ov;
            bi = oi;
        }
    }
    csync();
    if (lane == 0) {
        sm.redf[warp] = bv;
        sm.redu[warp] = bi;
    }
    csync();
    if (threadIdx.x == 0) {
        float v = sm.redf[0];
        uint32_t i = sm.redu[0];
        for (int w = 1; w < kWarps; ++w) {
            const uint32_t oi = sm.redu[w];
            const float ov = sm.redf[w];
            if (oi != 0xffffffffu && (i == 0xffffffffu || ov > v || (ov == v && oi < i))) {
                v = ov;
                i = oi;
            }
        }
        sm.result = i;
    }
    csync();
    return sm.result;
}

// Runs the processors on `logits` and, unless `out_scores` is given, selects a
// token.  Returns the token, or 0xffffffff after setting `status` when the
// reference would throw.  Must be called by all threads of the CTA.  With
// `scaled` the scores already carry the repetition penalty and the temperature
// (applied elementwise where they were produced, score_scale below).
__device__ inline uint32_t run_sampler(const float* logits, const SampleOpts& o, uint64_t draw, bool greedy,
                                       SamplerSmem& sm, SamplerBig* big, float* out_scores, int* status,
                                       bool scaled = false) {
    const int tid = threadIdx.x;
    const int base = elem_base(), cnt = elem_cnt();
    float s[kPer];
    if ((reinterpret_cast<uintptr_t>(logits) & 15u) == 0) {
        const float4* p4 = reinterpret_cast<const float4*>(logits + base);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = __ldcg(p4 + q);
            s[4 * q] = v.x;
            s[4 * q + 1] = v.y;
            s[4 * q + 2] = v.z;
            s[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int k = 16; k < kPer; ++k) s[k] = k < cnt ? __ldcg(logits + base + k) : -INFINITY;
    } else {
#pragma unroll
        for (int k = 0; k < kPer; ++k) s[k] = k < cnt ? __ldcg(logits + base + k) : -INFINITY;
    }

    // repetition penalty (unique history; negative scores are multiplied)
    if (!scaled && o.rp != 1.0f) {
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (k < cnt && bit_get(sm.seen, base + k)) s[k] = s[k] < 0.0f ? s[k] * o.rp : s[k] / o.rp;
    }
    if (!scaled && o.temperature != 1.0f) {
#pragma unroll
        for (int k = 0; k < kPer; ++k) s[k] = s[k] / o.temperature;
    }
    if (o.top_k > 0 && o.top_k < (uint32_t)kVocab) {
        const uint32_t kk = max(o.top_k, o.num_beams > 1 ? 2u : 1u);
        const float pivot = kth_largest(s, cnt, kk, sm);
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (s[k] < pivot) s[k] = -INFINITY;
    }
    const bool top_p = o.top_p < 1.0f;
    if (!top_p && out_scores) {
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (k < cnt) out_scores[base + k] = s[k];
        return 0;
    }
    if (!top_p && greedy) return block_argmax(s, base, cnt, sm);

    // finite survivors in index order
    uint32_t nf = 0;
    float lmax = -INFINITY;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt && isfinite(s[k])) {
            ++nf;
            lmax = fmaxf(lmax, s[k]);
        }
    const float mx = cblock_max(lmax, sm.redf);
    uint32_t n = 0;
    uint32_t off = block_excl_scan(nf, sm, &n);
    const bool fast = n <= (uint32_t)kFast;
    uint32_t* idx = fast ? sm.f_idx : big->sv_idx;
    float* sc = fast ? sm.f_s : big->sv_s;
    unsigned long long* key = fast ? sm.f_key : big->key;
    double* pr = fast ? sm.f_pr : nullptr;
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt && isfinite(s[k])) {
            idx[off] = base + k;
            sc[off] = s[k];
            ++off;
        }
    for (int i = tid; i < kBits; i += kThreads) sm.removed[i] = 0;
    csync();
    if (n == 0) {
        if (tid == 0) set_status(status, kStatusNoFiniteLogits, 100, 0);
        csync();
        return 0xffffffffu;
    }
    // exp(double(s - max)) of every survivor, in parallel (the values the
    // reference computes one by one; the sums below keep its order)
    if (pr) {
        for (uint32_t i = tid; i < n; i += kThreads) pr[i] = exp(double(sc[i] - mx));
        csync();
    }

    if (top_p) {
        int P = 1;
        while (P < (int)n) P <<= 1;
        // (score key, survivor position): position order is index order
        const int P_init = P <= 32 ? 32 : P;  // the warp sort reads 32 entries
        for (int i = tid; i < P_init; i += kThreads)
            key[i] = i < (int)n ? ((unsigned long long)ord_key(sc[i]) << 32) | (uint32_t)i : ~0ull;
        csync();
        if (P <= 32) {
            warp_sort32_asc(key);
            csync();
        } else {
            bitonic_sort_asc(key, P);
        }
        if (tid == 0) {
            double total = 0.0;
            if (pr) {
#pragma unroll 8
                for (uint32_t i = 0; i < n; ++i) total += pr[i];
            } else {
                for (uint32_t i = 0; i < n; ++i) total += exp(double(sc[i] - mx));
            }
            sm.err = total > 0.0 ? 0 : kStatusZeroMass;
            sm.f_total = total;
        }
        csync();
        if (pr && !sm.err) {
            // each survivor's share in ascending order (the reference's division),
            // then the cumulative mass by one thread in that order: the count of
            // leading survivors whose mass stays <= 1 - p, removed in parallel
            const double total = sm.f_total;
            for (uint32_t j = tid; j < n; j += kThreads) sm.f_q[j] = pr[uint32_t(key[j])] / total;
            csync();
            if (tid == 0) {
                const double low = 1.0 - double(o.top_p);
                double cum = 0.0;
                uint32_t nrem = 0;
#pragma unroll 8
                for (uint32_t j = 0; j < n; ++j) {
                    cum += sm.f_q[j];
                    if (!(cum <= low)) break;  // cumulative mass only grows: nothing later is removed
                    nrem = j + 1;
                }
                sm.sel_rem = nrem;
            }
            csync();
            for (uint32_t j = tid; j < sm.sel_rem; j += kThreads) {
                const uint32_t t = idx[uint32_t(key[j])];
                atomicOr(&sm.removed[t >> 5], 1u << (t & 31));
            }
            csync();
            if (tid == 0) {
                const uint32_t keep = (o.num_beams > 1 && n >= 2) ? 2u : 1u;
                for (uint32_t i = 0; i < keep; ++i) {
                    const uint32_t t = idx[uint32_t(key[n - 1 - i])];
                    sm.removed[t >> 5] &= ~(1u << (t & 31));
                }
            }
        } else if (tid == 0 && !sm.err) {
            const double total = sm.f_total;
            {
                const double low = 1.0 - double(o.top_p);
                double cum = 0.0;
                for (uint32_t j = 0; j < n; ++j) {
                    const uint32_t pos = uint32_t(key[j]);
                    cum += pr ? sm.f_q[j] : exp(double(sc[pos] - mx)) / total;
                    if (cum <= low) {
                        const uint32_t t = idx[pos];
                        sm.removed[t >> 5] |= 1u << (t & 31);
                    } else {
                        break;  // cumulative mass only grows: nothing later is removed
                    }
                }
                const uint32_t keep = (o.num_beams > 1 && n >= 2) ? 2u : 1u;
                for (uint32_t i = 0; i < keep; ++i) {
                    const uint32_t t = idx[uint32_t(key[n - 1 - i])];
                    sm.removed[t >> 5] &= ~(1u << (t & 31));
                }
            }
        }
        csync();
        if (sm.err) {
            if (tid == 0) set_status(status, sm.err, 101, 0);
            csync();
            return 0xffffffffu;
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (k < cnt && bit_get(sm.removed, base + k)) s[k] = -INFINITY;
    }
    if (out_scores) {
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (k < cnt) out_scores[base + k] = s[k];
        return 0;
    }
    if (greedy) return block_argmax(s, base, cnt, sm);

    // CDF sample in index order (double precision).  The maximum is unchanged
    // by top-p (the top score is always kept).  With the survivors' exp values
    // cached, the mass of each survivor (0 when removed) is gathered in
    // parallel and one thread folds it in index order as the reference does.
    if (pr) {
        csync();
        for (uint32_t i = tid; i < n; i += kThreads) sm.f_q[i] = bit_get(sm.removed, idx[i]) ? 0.0 : pr[i];
        csync();
        if (tid == 0) {
            double total = 0.0;
#pragma unroll 8
            for (uint32_t i = 0; i < n; ++i) total += sm.f_q[i];
            if (!(total > 0.0)) {
                set_status(status, kStatusZeroMass, 102, 0);
                sm.result = 0xffffffffu;
            } else {
                const double target = uniform_at(o.rng, o.seed, draw) * total;
                double cum = 0.0;
                uint32_t last = 0, pick = 0xffffffffu;
                for (uint32_t i = 0; i < n; ++i) {
                    const double p = sm.f_q[i];
                    if (p <= 0.0) continue;
                    last = i;
                    cum += p;
                    if (target < cum) {
                        pick = i;
                        break;
                    }
                }
                sm.result = idx[pick == 0xffffffffu ? last : pick];
            }
        }
        csync();
        return sm.result;
    }
    if (tid == 0) {
        double total = 0.0;
        for (uint32_t i = 0; i < n; ++i)
            if (!bit_get(sm.removed, idx[i])) total += pr ? pr[i] : exp(double(sc[i] - mx));
        if (!(total > 0.0)) {
            set_status(status, kStatusZeroMass, 102, 0);
            sm.result = 0xffffffffu;
        } else {
            const double target = uniform_at(o.rng, o.seed, draw) * total;
            double cum = 0.0;
            uint32_t last = 0, pick = 0xffffffffu;
            for (uint32_t i = 0; i < n; ++i) {
                const uint32_t t = idx[i];
                if (bit_get(sm.removed, t)) continue;
                const double p = pr ? pr[i] : exp(double(sc[i] - mx));
                if (p <= 0.0) continue;
                last = t;
                cum += p;
                if (target < cum) {
                    pick = t;
                    break;
                }
            }
            sm.result = pick == 0xffffffffu ? last : pick;
        }
    }
    csync();
    return sm.result;
}

}  // namespace itts
