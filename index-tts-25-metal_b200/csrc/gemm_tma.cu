// The fp32-accuracy GEMMs of the GPT prefill, the semantic codec's decode and
// the Qwen3 prompt pass on the 5th-generation tensor cores (tcgen05, sm_100a),
// fed by TMA:
//   C[m, n] = epi(sum_k A[m, k] * W[n, k] + bias[n]),   A [M, K], W [N, K]
// epilogues: bias; GELU (tanh form) or GELU (erf form), optionally split into
// hi / lo for the next GEMM; residual; layer scale + residual; SwiGLU.
//
// Accuracy.  Every operand x is held as two TF32-exact fp32 words,
// hi = rn_tf32(x) and lo = rn_tf32(x - hi) (x - hi is exact in fp32), so
// x = hi + lo to within 2^-24 |x|.  The products hi*hi + hi*lo + lo*hi drop
// only lo*lo (below 2^-22 |a w|), each product is exact in the tensor core,
// and the sum is accumulated in two tensor-memory accumulators: `main` takes
// the hi*hi products, `cross` the two small ones, so the accumulator's own
// rounding acts on cross at a scale 2^11 below main.  Every kChunk K blocks
// (128 K) both are drained into fp32 registers with round-to-nearest adds
// (acc += main + cross) and the next chunk starts afresh, so the tensor
// core's accumulation error is bounded per 128-term chunk, as a CUDA-core
// fp32 dot product of the same length.  The weights are split once when the
// context is created (k_split_tf32); the activations by the kernel that
// produces them (LayerNorm, attention, the GELU epilogue of c_fc).
//
// Tiling.  128 x 128 output tiles shared out stream-K: the (tile, 32-wide K
// block) units are split evenly over up to one CTA per SM, so a CTA may own
// part of a tile; when the tiles number between 3/4 of the SMs and all of
// them, one CTA per whole tile.  320 threads in three roles:
//   warp 0 (one lane)  TMA producer: per 32-wide K block, four 2-D tensor
//                      loads (A hi, A lo: 128 rows; W hi, W lo: 128 rows) of
//                      128-byte rows into a kStages-deep ring of 64 KB stages,
//                      128-byte swizzled, completing on the stage's mbarrier.
//   warp 1 (one lane)  MMA issuer: per 8-wide K step, A_hi x [W_hi; W_lo]
//                      (N = 256: main in columns 0..127, cross in 128..255)
//                      and A_lo x W_hi (N = 128, into cross); commits free the
//                      stage and, at a chunk's end, publish the accumulator.
//                      Warp 1 also owns the 512 tensor-memory columns: two
//                      256-column accumulator buffers, so the MMAs of chunk
//                      c + 1 run while chunk c is drained.
//   warps 2-9          drain + epilogue: warp w reads accumulator lanes
//                      32 (w % 4) .. +31 (thread = output row) and one half
//                      of the columns, adds each chunk into 64 fp32
//                      registers, then applies bias and
//                      GELU (split into hi / lo for the next GEMM) or the
//                      residual.  A tile split between CTAs: every CTA
//                      stores its partial tile; the last to arrive (per-tile
//                      counter) sums the partials in CTA order, so results do
//                      not depend on which CTA finishes last.
// Launched with programmatic stream serialization: the producer requests the
// first stages' weight tiles before waiting for the previous kernel.
// Every mbarrier wait is bounded by time; a CTA that gives up records a status,
// waits (bounded) for its own TMA loads and MMAs, frees its tensor memory and
// returns without writing its tile.
//
// The GEMMs and the weight split replace the fp32 MPS GEMMs of the
// reference's prefill (metal_context.mm:368-410 via gpt.cpp:88-125).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>

#include "common.cuh"
#include "model.hpp"

namespace itts {
namespace {

constexpr int GM = 128, GN = 128, GK = 32;
constexpr int kStages = 3;
constexpr int kChunk = 4;  // K blocks per tensor-memory accumulation chunk
constexpr int kDrainWarps = 8;  // two per accumulator lane quarter, 64 columns each
constexpr int kDrainCols = GN / 2;
constexpr int kGemmThreads = 64 + 32 * kDrainWarps;
constexpr uint32_t kStageBytes = (2 * GM * GK + 2 * GN * GK) * 4;  // 64 KB
constexpr uint32_t kTmemCols = 512;
constexpr int kStageLd = 68;  // row stride (floats) of the epilogue's 64 x 64 staging quarter
constexpr int kMaxCtas = 148;
constexpr int kCtasPerTile = 6;  // CTAs per output tile when the tiles are few (a tile then has <= 8 contributors)
constexpr int kMaxContrib = 8;
static_assert(TmaPrefill::kCounters >= (kMaxPrefix / GM) * (kFfn / GN), "a counter per c_fc tile at 1024 rows");
constexpr size_t kWsFloats = size_t(2 * kMaxCtas) * GM * GN;  // two partial-tile slots per CTA

struct alignas(1024) GemmSmem {
    float a[kStages][2][GM * GK];  // [stage][hi, lo]
    float w[kStages][2][GN * GK];  // [stage][hi, lo]: adjacent, read as one 256-row operand
    float stage[64 * kStageLd];  // epilogue: one 64 x 64 quarter of the output tile
    unsigned long long full[kStages], empty[kStages], tfull[2], tempty[2], done;
    uint32_t tmem_base;
    int abort;
    int last;
};
constexpr size_t kGemmSmemBytes = sizeof(GemmSmem) + 1024;

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart, descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) |
           (uint64_t(2) << 61);
}

// Instruction descriptor: D f32, A and B tf32, both K-major, M = 128, N = n.
constexpr uint32_t idesc(int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(GM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void mma_commit(unsigned long long* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(unsigned long long* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(su32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait on a phase of `bar`.  Gives up when the time limit passes (and
// raises the CTA's abort flag) or, if `abort` is given, when another role of
// the CTA has raised it.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity, int* abort) {
    if (mbar_try(bar, parity)) return true;  // the common case reads no timer
    const unsigned long long t0 = globaltimer_ns();
    for (uint32_t i = 0;; ++i) {
        if (mbar_try(bar, parity)) return true;
        if ((i & 15u) == 15u) {
            if (abort && *reinterpret_cast<volatile int*>(abort)) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                if (abort) *reinterpret_cast<volatile int*>(abort) = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load(void* dst, const CUtensorMap* map, int x, int y, unsigned long long* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(su32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(addr));
}

struct GemmArgs {
    const float* bias;
    const float* R;  // residual [M, N] (kEpiResid)
    float* C;        // output [M, N]; with a split output, the hi half
    float* C_lo;     // split output: lo half (kEpiGelu), else null
    int M, N, K;
    int kbt;         // K blocks per tile (K / 32)
    int ntn;         // output tiles along N (N / 128)
    int ctas;        // CTAs of the launch (gridDim.x)
    long long units; // tiles x kbt: the (tile, K block) pairs shared out among the CTAs
    float* ws;       // partial tiles: two 128 x 128 slots per CTA (its first and its last tile)
    int* counters;   // per output tile: contributors that have stored their partial (the last resets)
    int* status;
    const float* gamma;  // layer scale [N] (kEpiScaleResid)
};

enum GemmEpi : int {
    kEpiBias = TmaEpiBias,
    kEpiGelu = TmaEpiGelu,
    kEpiResid = TmaEpiResid,
    kEpiSwiGLU = TmaEpiSwiGLU,
    kEpiGeluErf = TmaEpiGeluErf,
    kEpiScaleResid = TmaEpiScaleResid
};

// CTA i owns units [i U / G, (i + 1) U / G) of the tile-major (tile, K block)
// sequence: every CTA gets the same number of K blocks (to one), whatever the
// tile count.  Its units form segments, one per tile they touch.
__device__ __forceinline__ long long unit0(const GemmArgs& g, int i) { return (long long)i * g.units / g.ctas; }

// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of(const GemmArgs& g, long long u) {
    int i = int(u * g.ctas / g.units);
    while (i > 0 && unit0(g, i) > u) --i;
    while (i + 1 < g.ctas && unit0(g, i + 1) <= u) ++i;
    return i;
}

// Workspace slot of CTA i's partial of tile t: slot 0 for the first tile of
// its range, 1 for the last (a range inside one tile has only slot 0).
__device__ __forceinline__ float* slot(const GemmArgs& g, int i, int t) {
    const int first = int(unit0(g, i) / g.kbt);
    return g.ws + (size_t(2 * i + (t == first ? 0 : 1)) * GM) * GN;
}

template <int EPI>
__device__ __forceinline__ void store_out(const GemmArgs& g, int m, int n, float4 v, float4 b) {
    float4 y = make_float4(v.x + b.x, v.y + b.y, v.z + b.z, v.w + b.w);
    if (EPI == kEpiSwiGLU) {
        // W rows interleave gate and up (row 2r = gate_r, 2r + 1 = up_r): the
        // four columns are (gate, up) of outputs n/2 and n/2 + 1 of C[M][N/2],
        // silu(gate) * up as mit2_silu_mul_f32 (kernels.metal:363-374), split
        // into hi / lo for the next GEMM.
        const float s0 = y.x / (1.0f + expf(-y.x)) * y.y, s1 = y.z / (1.0f + expf(-y.z)) * y.w;
        const size_t o = size_t(m) * (g.N / 2) + n / 2;
        const float h0 = rn_tf32(s0), h1 = rn_tf32(s1);
        *reinterpret_cast<float2*>(g.C + o) = make_float2(h0, h1);
        *reinterpret_cast<float2*>(g.C_lo + o) = make_float2(rn_tf32(s0 - h0), rn_tf32(s1 - h1));
        return;
    }
    const size_t o = size_t(m) * g.N + n;
    if (EPI == kEpiGelu || EPI == kEpiGeluErf) {
        if (EPI == kEpiGelu)
            y = make_float4(gelu_ref(y.x), gelu_ref(y.y), gelu_ref(y.z), gelu_ref(y.w));
        else
            y = make_float4(gelu_erf(y.x), gelu_erf(y.y), gelu_erf(y.z), gelu_erf(y.w));
        if (g.C_lo) {
            const float4 h = make_float4(rn_tf32(y.x), rn_tf32(y.y), rn_tf32(y.z), rn_tf32(y.w));
            *reinterpret_cast<float4*>(g.C + o) = h;
            *reinterpret_cast<float4*>(g.C_lo + o) =
                make_float4(rn_tf32(y.x - h.x), rn_tf32(y.y - h.y), rn_tf32(y.z - h.z), rn_tf32(y.w - h.w));
            return;
        }
    } else if (EPI == kEpiResid) {
        const float4 r = *reinterpret_cast<const float4*>(g.R + o);
        y = make_float4(r.x + y.x, r.y + y.y, r.z + y.z, r.w + y.w);
    } else if (EPI == kEpiScaleResid) {  // x + gamma * pwconv2(.) (codec.cpp:46); R may alias C
        const float4 r = *reinterpret_cast<const float4*>(g.R + o);
        const float4 s = __ldg(reinterpret_cast<const float4*>(g.gamma + n));
        y = make_float4(fmaf(y.x, s.x, r.x), fmaf(y.y, s.y, r.y), fmaf(y.z, s.z, r.z), fmaf(y.w, s.w, r.w));
    }
    *reinterpret_cast<float4*>(g.C + o) = y;
}

// Bias at columns n..n+3, or zeros without a bias.
__device__ __forceinline__ float4 bias4(const GemmArgs& g, int n) {
    return g.bias ? __ldg(reinterpret_cast<const float4*>(g.bias + n)) : make_float4(0.f, 0.f, 0.f, 0.f);
}

__device__ __forceinline__ void drain_sync() { asm volatile("bar.sync 2, %0;" ::"n"(32 * kDrainWarps) : "memory"); }

template <int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_gemm_tma(const __grid_constant__ CUtensorMap ma_hi, const __grid_constant__ CUtensorMap ma_lo,
               const __grid_constant__ CUtensorMap mw_hi, const __grid_constant__ CUtensorMap mw_lo, GemmArgs g) {
    extern __shared__ unsigned char smem_raw[];
    GemmSmem& sm = *reinterpret_cast<GemmSmem*>(smem_raw + ((1024 - (su32(smem_raw) & 1023)) & 1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const long long u0 = unit0(g, cta), u1 = unit0(g, cta + 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&sm.full[s])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&sm.empty[s])) : "memory");
        }
        for (int b = 0; b < 2; ++b) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&sm.tfull[b])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(&sm.tempty[b])), "n"(kDrainWarps) : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(su32(&sm.done)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sm.abort = 0;
        sm.last = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&sm.tmem_base)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = sm.tmem_base;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer: the CTA's units in order, one ring stage each
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&ma_hi)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&ma_lo)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mw_hi)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mw_lo)) : "memory");
            int issued = 0;
            const int n = int(u1 - u0);
            // The first stages' weight tiles do not depend on the previous
            // kernel (PDL launch): they are requested before the wait for it,
            // the activation tiles after.  The loop below breaks only at
            // i >= kStages, so every stage armed here gets its A tiles too.
            const int early = min(n, kStages);
            for (int i = 0; i < early; ++i) {
                const long long u = u0 + i;
                const int t = int(u / g.kbt), kx = int(u % g.kbt) * GK, n0 = (t % g.ntn) * GN;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&sm.full[i])),
                             "r"(kStageBytes)
                             : "memory");
                tma_load(sm.w[i][0], &mw_hi, kx, n0, &sm.full[i]);
                tma_load(sm.w[i][1], &mw_lo, kx, n0, &sm.full[i]);
            }
            pdl_wait();
            for (int i = 0; i < n; ++i) {
                const int s = i % kStages;
                if (i >= kStages && !mbar_wait(&sm.empty[s], uint32_t((i / kStages) + 1) & 1u, &sm.abort)) break;
                const long long u = u0 + i;
                const int t = int(u / g.kbt), kx = int(u % g.kbt) * GK;
                const int m0 = (t / g.ntn) * GM, n0 = (t % g.ntn) * GN;
                if (i >= early) {
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(&sm.full[s])),
                                 "r"(kStageBytes)
                                 : "memory");
                    tma_load(sm.w[s][0], &mw_hi, kx, n0, &sm.full[s]);
                    tma_load(sm.w[s][1], &mw_lo, kx, n0, &sm.full[s]);
                }
                tma_load(sm.a[s][0], &ma_hi, kx, m0, &sm.full[s]);
                tma_load(sm.a[s][1], &ma_lo, kx, m0, &sm.full[s]);
                issued = i + 1;
            }
            // Loads still in flight land before the CTA may exit (after an abort
            // the consumer may not have waited for them).
            for (int i = max(0, issued - kStages); i < issued; ++i)
                mbar_wait(&sm.full[i % kStages], uint32_t(i / kStages) & 1u, nullptr);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer: chunks of kChunk units that never cross a tile
            int c = -1;  // chunk counter over the CTA's segments
            bool stop = false;
            for (long long u = u0; u < u1 && !stop;) {
                const int kb0 = int(u % g.kbt);
                const int len = int(min((long long)(g.kbt - kb0), u1 - u));
                for (int j = 0; j < len; ++j) {
                    const int i = int(u - u0) + j, s = i % kStages;
                    const bool cstart = j % kChunk == 0;
                    if (cstart) ++c;
                    const int buf = c & 1;
                    if (cstart && c >= 2 && !mbar_wait(&sm.tempty[buf], uint32_t((c >> 1) + 1) & 1u, &sm.abort)) {
                        stop = true;
                        break;
                    }
                    if (!mbar_wait(&sm.full[s], uint32_t(i / kStages) & 1u, &sm.abort)) {
                        stop = true;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t d = tmem + uint32_t(buf * 256);
                    const uint32_t ah = su32(sm.a[s][0]), al = su32(sm.a[s][1]), wh = su32(sm.w[s][0]);
#pragma unroll
                    for (int ks = 0; ks < GK / 8; ++ks) {  // 8 TF32 = 32 bytes per K step
                        const uint32_t o = 32u * ks;
                        mma_tf32(d, smem_desc(ah + o), smem_desc(wh + o), idesc(2 * GN), !(cstart && ks == 0));
                        mma_tf32(d + GN, smem_desc(al + o), smem_desc(wh + o), idesc(GN), 1u);
                    }
                    mma_commit(&sm.empty[s]);
                    if (j % kChunk == kChunk - 1 || j == len - 1) mma_commit(&sm.tfull[buf]);
                }
                u += len;
            }
            mma_commit(&sm.done);  // every MMA issued above has completed once this phase flips
            mbar_wait(&sm.done, 0u, nullptr);
        }
    } else {  // warps 2-9: drain, then per segment the epilogue
        pdl_wait();  // the epilogue reads R and writes C, the previous kernel's buffers
        const int q = warp & 3, hcol = (warp - 2) >> 2, dw = warp - 2;
        const int c0 = kDrainCols * hcol;  // this warp's first accumulator column
        const uint32_t taddr = tmem + (uint32_t(32 * q) << 16) + uint32_t(c0);
        bool ok = true;
        int c = -1;
        for (long long u = u0; u < u1 && ok;) {
            const int t = int(u / g.kbt), kb0 = int(u % g.kbt);
            const int len = int(min((long long)(g.kbt - kb0), u1 - u));
            const int m0 = (t / g.ntn) * GM, n0 = (t % g.ntn) * GN;
            float acc[kDrainCols];
#pragma unroll
            for (int j = 0; j < kDrainCols; ++j) acc[j] = 0.f;
            for (int j = 0; j < len; j += kChunk) {
                ++c;
                const int buf = c & 1;
                if (!mbar_wait(&sm.tfull[buf], uint32_t(c >> 1) & 1u, &sm.abort)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int e = 0; e < kDrainCols; e += 16) {
                    uint32_t mv[16], cv[16];
                    tmem_ld16(taddr + uint32_t(buf * 256 + e), mv);
                    tmem_ld16(taddr + uint32_t(buf * 256 + GN + e), cv);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int x = 0; x < 16; ++x) acc[e + x] += __uint_as_float(mv[x]) + __uint_as_float(cv[x]);
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0)
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(&sm.tempty[buf])) : "memory");
            }
            // Every drain warp agrees before the segment's output is written.
            uint32_t bad;
            asm volatile(
                "{\n\t.reg .pred pi, po;\n\tsetp.ne.u32 pi, %1, 0;\n\tbar.red.or.pred po, 2, %2, pi;\n\t"
                "selp.u32 %0, 1, 0, po;\n\t}"
                : "=r"(bad)
                : "r"((uint32_t)!ok), "n"(32 * kDrainWarps)
                : "memory");
            if (bad) {
                ok = false;
                break;
            }
            const bool whole = kb0 == 0 && len == g.kbt;
            float* part = whole ? nullptr : slot(g, cta, t);
            // Rows leave through shared memory a 64 x 64 quarter at a time (two
            // warps stage it, all eight write it out as coalesced rows): the
            // tile itself (whole) or this CTA's partial of it.
            const int col = (lane & 15) * 4;
            float4 bias2[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
            if (!part) {
                bias2[0] = bias4(g, n0 + col);
                bias2[1] = bias4(g, n0 + kDrainCols + col);
            }
            for (int pass = 0; pass < 4; ++pass) {
                const int rh = pass >> 1, ch = pass & 1;
                if ((q >> 1) == rh && hcol == ch) {
                    float* st = sm.stage + ((q & 1) * 32 + lane) * kStageLd;
#pragma unroll
                    for (int j = 0; j < kDrainCols; j += 4)
                        *reinterpret_cast<float4*>(st + j) = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
                }
                drain_sync();
#pragma unroll
                for (int rr = 0; rr < 8; rr += 2) {
                    const int r = dw * 8 + rr + (lane >> 4);
                    const float4 v = *reinterpret_cast<const float4*>(sm.stage + r * kStageLd + col);
                    const int row = rh * 64 + r, n = ch * kDrainCols + col;
                    if (part)
                        *reinterpret_cast<float4*>(part + size_t(row) * GN + n) = v;
                    else if (m0 + row < g.M)
                        store_out<EPI>(g, m0 + row, n0 + n, v, bias2[ch]);
                }
                drain_sync();
            }
            if (part) {  // the last contributor of the tile sums the partials in K order
                const int first = cta_of(g, (long long)t * g.kbt), nc = cta_of(g, (long long)(t + 1) * g.kbt - 1) - first + 1;
                drain_sync();  // every partial store of this CTA is issued
                if (dw == 0 && lane == 0) {
                    // The acq_rel add releases the stores the barrier ordered
                    // before it and, for the last arriver, acquires the others'.
                    int prev;
                    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(prev) : "l"(g.counters + t) : "memory");
                    const int last = prev == nc - 1;
                    if (last) g.counters[t] = 0;
                    sm.last = last;
                }
                drain_sync();
                if (sm.last) {
                    const float4 b = bias4(g, n0 + 4 * lane);
                    const float* p0 = slot(g, first, t) + 4 * lane;
                    if (nc <= 3) {  // the common case: four rows' loads in flight at once
                        const float* p1 = slot(g, first + 1, t) + 4 * lane;
                        const float* p2 = nc == 3 ? slot(g, first + 2, t) + 4 * lane : p1;
#pragma unroll 1
                        for (int r0 = dw * 16; r0 < dw * 16 + 16; r0 += 4) {
                            float4 v[4][3];
#pragma unroll
                            for (int rr = 0; rr < 4; ++rr) {
                                const size_t o = size_t(r0 + rr) * GN;
                                v[rr][0] = __ldcg(reinterpret_cast<const float4*>(p0 + o));
                                v[rr][1] = __ldcg(reinterpret_cast<const float4*>(p1 + o));
                                v[rr][2] = __ldcg(reinterpret_cast<const float4*>(p2 + o));
                            }
#pragma unroll
                            for (int rr = 0; rr < 4; ++rr) {
                                float4 a = make_float4(v[rr][0].x + v[rr][1].x, v[rr][0].y + v[rr][1].y,
                                                       v[rr][0].z + v[rr][1].z, v[rr][0].w + v[rr][1].w);
                                if (nc == 3)
                                    a = make_float4(a.x + v[rr][2].x, a.y + v[rr][2].y, a.z + v[rr][2].z, a.w + v[rr][2].w);
                                if (m0 + r0 + rr < g.M) store_out<EPI>(g, m0 + r0 + rr, n0 + 4 * lane, a, b);
                            }
                        }
                    } else {
                        const float* sp[kMaxContrib];
#pragma unroll
                        for (int i = 0; i < kMaxContrib; ++i) sp[i] = i < nc ? slot(g, first + i, t) + 4 * lane : p0;
#pragma unroll 1
                        for (int r = dw * 16; r < dw * 16 + 16; ++r) {
                            float4 v[kMaxContrib];
#pragma unroll
                            for (int i = 0; i < kMaxContrib; ++i)
                                if (i < nc) v[i] = __ldcg(reinterpret_cast<const float4*>(sp[i] + size_t(r) * GN));
                            float4 a = v[0];
#pragma unroll
                            for (int i = 1; i < kMaxContrib; ++i)
                                if (i < nc) a = make_float4(a.x + v[i].x, a.y + v[i].y, a.z + v[i].z, a.w + v[i].w);
                            if (m0 + r < g.M) store_out<EPI>(g, m0 + r, n0 + 4 * lane, a, b);
                        }
                    }
                }
                drain_sync();
            }
            u += len;
        }
        if (!ok && dw == 0 && lane == 0) set_status(g.status, kStatusRingTimeout, 510, cta);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

// W -> (hi, lo), each TF32-exact.
__global__ void k_split_tf32(const float* __restrict__ w, float* __restrict__ hi, float* __restrict__ lo, size_t n4) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(w)[i];
        const float4 h = make_float4(rn_tf32(v.x), rn_tf32(v.y), rn_tf32(v.z), rn_tf32(v.w));
        reinterpret_cast<float4*>(hi)[i] = h;
        reinterpret_cast<float4*>(lo)[i] =
            make_float4(rn_tf32(v.x - h.x), rn_tf32(v.y - h.y), rn_tf32(v.z - h.z), rn_tf32(v.w - h.w));
    }
}

// bf16 W -> fp32 (the bf16 value is the high half of the fp32 word; exact in TF32).
__global__ void k_widen_bf16(const uint16_t* __restrict__ w, float* __restrict__ out, size_t n4) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const uint2 raw = reinterpret_cast<const uint2*>(w)[i];
        reinterpret_cast<float4*>(out)[i] = make_float4(__uint_as_float(raw.x << 16), __uint_as_float(raw.x & 0xffff0000u),
                                                         __uint_as_float(raw.y << 16), __uint_as_float(raw.y & 0xffff0000u));
    }
}

// ---- host side ----------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D map of a row-major fp32 [rows, cols] array read in 32-column x 128-row
// boxes with the 128-byte swizzle; rows past the end read as zero.
cudaError_t make_map(CUtensorMap* map, const float* base, uint64_t rows, uint64_t cols) {
    auto fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {GK, GM};  // GM == GN: one box shape for A and W
    static_assert(GM == GN, "A and W boxes share a shape");
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

constexpr int kMatN[4] = {kQkv, kWidth, kFfn, kWidth};
constexpr int kMatK[4] = {kWidth, kWidth, kWidth, kFfn};

size_t mat_offset(int layer, int mat) {
    size_t per_layer = 0;
    for (int i = 0; i < 4; ++i) per_layer += 2 * size_t(kMatN[i]) * kMatK[i];
    size_t o = per_layer * layer;
    for (int i = 0; i < mat; ++i) o += 2 * size_t(kMatN[i]) * kMatK[i];
    return o;
}

CUtensorMap* wmaps(TmaPrefill* p) { return static_cast<CUtensorMap*>(p->maps); }

template <int EPI>
cudaError_t launch_epi(const CUtensorMap* ma, const CUtensorMap* mw, const GemmArgs& g, cudaStream_t s) {
    static std::once_flag once[64];
    static cudaError_t attr_err[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::call_once(once[dev], [&] {
        attr_err[dev] =
            cudaFuncSetAttribute(k_gemm_tma<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmemBytes);
    });
    if (attr_err[dev] != cudaSuccess) return attr_err[dev];
    return launch_pdl(k_gemm_tma<EPI>, dim3(g.ctas), kGemmThreads, kGemmSmemBytes, s, ma[0], ma[1], mw[0], mw[1],
                      g);
}

int sm_count() {
    static std::once_flag once[64];
    static int n[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kMaxCtas;
    std::call_once(once[dev], [&] {
        if (cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n[dev] = kMaxCtas;
    });
    return n[dev];
}

}  // namespace

cudaError_t tma_prefill_init(TmaPrefill* p, const ModelW& hw, bool wbf16, cudaStream_t s) {
    if (!encode_fn()) return cudaErrorNotSupported;
    p->layers = hw.layers;
    // fp32 weights: hi and lo per matrix.  bf16 weights are exact in TF32:
    // hi is the widened matrix, and every lo map reads one shared zero matrix.
    const size_t zero_floats = size_t(kFfn) * kWidth;
    const size_t wfloats = wbf16 ? mat_offset(hw.layers, 0) / 2 + zero_floats : mat_offset(hw.layers, 0);
    cudaError_t e = cudaMalloc(&p->wsplit, wfloats * sizeof(float));
    if (e != cudaSuccess) return e;
    float* zero = p->wsplit + (wfloats - zero_floats);
    if (wbf16 && (e = cudaMemsetAsync(zero, 0, zero_floats * sizeof(float), s)) != cudaSuccess) return e;
    const size_t act = size_t(kMaxPrefix) * (4 * kWidth + 2 * kFfn);
    float* a = nullptr;
    if ((e = cudaMalloc(&a, act * sizeof(float))) != cudaSuccess) return e;
    p->x_hi = a;
    p->x_lo = p->x_hi + size_t(kMaxPrefix) * kWidth;
    p->att_hi = p->x_lo + size_t(kMaxPrefix) * kWidth;
    p->att_lo = p->att_hi + size_t(kMaxPrefix) * kWidth;
    p->ff_hi = p->att_lo + size_t(kMaxPrefix) * kWidth;
    p->ff_lo = p->ff_hi + size_t(kMaxPrefix) * kFfn;
    if ((e = cudaMalloc(&p->ws, kWsFloats * sizeof(float))) != cudaSuccess) return e;
    if ((e = cudaMalloc(&p->counters, TmaPrefill::kCounters * sizeof(int))) != cudaSuccess) return e;
    if ((e = cudaMemsetAsync(p->counters, 0, TmaPrefill::kCounters * sizeof(int), s)) != cudaSuccess) return e;
    p->maps = new (std::nothrow) CUtensorMap[size_t(hw.layers) * 8];
    if (!p->maps) return cudaErrorMemoryAllocation;
    for (int l = 0; l < hw.layers; ++l) {
        const LayerW& L = hw.layer[l];
        const float* src[4] = {L.w_qkv, L.w_o, L.w_fc, L.w_mp};
        for (int mat = 0; mat < 4; ++mat) {
            const size_t n = size_t(kMatN[mat]) * kMatK[mat];
            float* hi = p->wsplit + (wbf16 ? mat_offset(l, mat) / 2 : mat_offset(l, mat));
            float* lo = wbf16 ? zero : hi + n;
            if (wbf16)
                k_widen_bf16<<<592, 256, 0, s>>>(reinterpret_cast<const uint16_t*>(src[mat]), hi, n / 4);
            else
                k_split_tf32<<<592, 256, 0, s>>>(src[mat], hi, lo, n / 4);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            if ((e = make_map(&wmaps(p)[(l * 4 + mat) * 2], hi, kMatN[mat], kMatK[mat])) != cudaSuccess) return e;
            if ((e = make_map(&wmaps(p)[(l * 4 + mat) * 2 + 1], lo, kMatN[mat], kMatK[mat])) != cudaSuccess) return e;
        }
    }
    p->act_rows = -1;
    return cudaSuccess;
}

void tma_prefill_free(TmaPrefill* p) {
    for (void* q : {(void*)p->wsplit, (void*)p->x_hi, (void*)p->ws, (void*)p->counters})
        if (q) cudaFree(q);
    delete[] static_cast<CUtensorMap*>(p->maps);
    *p = TmaPrefill{};
}

// Encodes the activation maps for `rows` rows (once per distinct row count).
cudaError_t tma_prefill_rows(TmaPrefill* p, int rows) {
    if (p->act_rows == rows) return cudaSuccess;
    static_assert(sizeof(CUtensorMap) == 128 && alignof(CUtensorMap) == 64, "tensor map layout");
    const float* base[6] = {p->x_hi, p->x_lo, p->att_hi, p->att_lo, p->ff_hi, p->ff_lo};
    const int cols[6] = {kWidth, kWidth, kWidth, kWidth, kFfn, kFfn};
    for (int i = 0; i < 6; ++i) {
        CUtensorMap m;  // encoded in an aligned object, then stored
        const cudaError_t e = make_map(&m, base[i], uint64_t(rows), uint64_t(cols[i]));
        if (e != cudaSuccess) return e;
        std::memcpy(p->act_maps[i], &m, sizeof m);
    }
    p->act_rows = rows;
    return cudaSuccess;
}

namespace {

// One GEMM C = epi(A W^T + bias) from A's and W's (hi, lo) tensor maps.
cudaError_t run_gemm(const CUtensorMap* ma, const CUtensorMap* mw, int epi, const float* bias, const float* R,
                     float* C, float* C_lo, int M, int N, int K, float* ws, int* counters, int counters_n,
                     int* status, cudaStream_t s, const float* gamma = nullptr) {
    if (M < 1 || N % GN || K % GK || K < GK) return cudaErrorInvalidValue;
    const int kbt = K / GK, tiles = ((M + GM - 1) / GM) * (N / GN);
    if (tiles > counters_n) return cudaErrorInvalidValue;
    // One CTA per SM, every CTA the same number of K blocks (to one); at least
    // one accumulation chunk per CTA, and few tiles spread over at most
    // kCtasPerTile CTAs each.
    const long long units = (long long)tiles * kbt;
    const int sms = std::min(sm_count(), kMaxCtas);
    int ctas = int(std::max(1LL, std::min({(long long)sms, (long long)kCtasPerTile * tiles, units / kChunk})));
    // Between 3/4 of the SMs and all of them in tiles, one CTA per tile: no
    // tile is split, so no partial goes through the workspace (measured: 451-row
    // prefill 5.81 -> 5.61 ms, 1024-code codec decode 0.955 -> 0.880 ms).
    if (tiles <= sms && tiles * 4 >= sms * 3) ctas = tiles;
    GemmArgs g{bias, R, C, C_lo, M, N, K, kbt, N / GN, ctas, units, ws, counters, status, gamma};
    switch (epi) {
        case kEpiGelu: return launch_epi<kEpiGelu>(ma, mw, g, s);
        case kEpiResid: return launch_epi<kEpiResid>(ma, mw, g, s);
        case kEpiGeluErf: return launch_epi<kEpiGeluErf>(ma, mw, g, s);
        case kEpiScaleResid: return R && gamma ? launch_epi<kEpiScaleResid>(ma, mw, g, s) : cudaErrorInvalidValue;
        case kEpiSwiGLU: return C_lo ? launch_epi<kEpiSwiGLU>(ma, mw, g, s) : cudaErrorInvalidValue;
        default: return launch_epi<kEpiBias>(ma, mw, g, s);
    }
}

}  // namespace

// One prefill GEMM of layer `layer`: matrix `mat` (TmaMatrix) against the
// split activation that feeds it (x for qkv and c_fc, att for c_proj, ff for
// mlp.c_proj).
cudaError_t launch_gemm_tma(TmaPrefill* p, int layer, int mat, const float* bias, const float* R, float* C,
                            float* C_lo, int M, int* status, cudaStream_t s) {
    cudaError_t e = tma_prefill_rows(p, M);
    if (e != cudaSuccess) return e;
    CUtensorMap ma[2];
    std::memcpy(ma, p->act_maps[mat == kMatO ? 2 : mat == kMatMp ? 4 : 0], sizeof ma);
    const CUtensorMap* mw = &wmaps(p)[(layer * 4 + mat) * 2];
    const int epi = mat == kMatFc ? kEpiGelu : mat == kMatQkv ? kEpiBias : kEpiResid;
    return run_gemm(ma, mw, epi, bias, R, C, C_lo, M, kMatN[mat], kMatK[mat], p->ws, p->counters,
                    TmaPrefill::kCounters, status, s);
}

cudaError_t tma_make_map(TmaMap* m, const float* base, uint64_t rows, uint64_t cols) {
    static_assert(sizeof(TmaMap) == sizeof(CUtensorMap), "tensor map storage");
    CUtensorMap t;
    const cudaError_t e = make_map(&t, base, rows, cols);
    if (e == cudaSuccess) std::memcpy(m->bytes, &t, sizeof t);
    return e;
}

cudaError_t tma_split(const float* src, float* hi, float* lo, size_t n, cudaStream_t s) {
    if (n % 4) return cudaErrorInvalidValue;
    k_split_tf32<<<592, 256, 0, s>>>(src, hi, lo, n / 4);
    return cudaGetLastError();
}

size_t tma_workspace_floats() { return kWsFloats; }

cudaError_t tma_gemm(const TmaGemm& q, cudaStream_t s) {
    CUtensorMap ma[2], mw[2];
    std::memcpy(ma, q.a, sizeof ma);
    std::memcpy(mw, q.w, sizeof mw);
    return run_gemm(ma, mw, q.epi, q.bias, q.R, q.C, q.C_lo, q.M, q.N, q.K, q.ws, q.counters, q.counters_n,
                    q.status, s, q.gamma);
}

}  // namespace itts
