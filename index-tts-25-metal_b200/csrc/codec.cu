// Semantic codec decode of IndexTTS 2.5 on B200 (sm_100a): semantic codes ->
// 1024-d features at twice the code rate, the stage that consumes the GPT's
// codes (src/codec.cpp:50-69, EnhancedCodec::lookup + decode).
//
//   lookup        x[t] = out_project(codebook[code_t])           [T, 1024]
//   vocos decoder embed conv k=7 1024 -> 384, LayerNorm (eps 1e-6),
//                 12 ConvNeXt blocks: depthwise conv k=7, LayerNorm,
//                 pwconv1 384 -> 2048, GELU (erf form), pwconv2 2048 -> 384,
//                 x += gamma * (.), then LayerNorm and linear 384 -> 1024
//   upsample      nearest x2 over time, then conv k=3 1024 -> 1024  [2T, 1024]
//
// Every linear and convolution is one GEMM C[M, N] = A[M, K] . W[N, K]^T:
// a k-wide same-padded convolution reads its A operand as the implicit
// window A[t][c * k + j] = x[t + j - k/2][c] (zero outside), which is the
// reference's weight layout [out][in][k] read as [out][in * k]
// (kernels.metal:1397-1425 sums over in_c, then k); the final convolution's
// window reads the nearest-upsampled rows x[floor(s / 2)] directly
// (kernels.metal:1376-1395 with scale in/out = 0.5).  Epilogues fuse the bias,
// the GELU of pwconv1 and the layer scale + residual of pwconv2.  Two GEMM
// paths: by default the TMA-fed tcgen05 GEMM of gemm_tma.cu on TF32 hi / lo
// operands (the convolutions' windows written out as split im2col rows, the
// activations that feed a GEMM split by the kernel producing them, the chain
// launched with PDL); in GEMM mode 1 fp32 on the CUDA cores (k_codec_gemm,
// 64 x 64 tiles, k-tiles of 32, each output summing its K products in k
// order, reading the windows directly).
#include <vector>

#include "codec.hpp"
#include "common.cuh"

namespace itts {
namespace {

enum CodecLoad : int { kLoadPlain = 0, kLoadConv = 1, kLoadConvUp2 = 2 };
enum CodecEpi : int { kCEpiBias = 0, kCEpiGelu = 1, kCEpiScaleResid = 2 };

struct ConvSrc {
    const float* x;  // [rows, ch] source rows (before upsampling for kLoadConvUp2)
    int ch, ks, rows_out;  // channels, kernel width, output rows (time steps)
};

// A[m][kk] of the GEMM.
template <int LOAD>
__device__ __forceinline__ float load_a(const float* A, int K, const ConvSrc& cs, int m, int kk) {
    if (LOAD == kLoadPlain) return A[(size_t)m * K + kk];
    const int c = kk / cs.ks, j = kk - c * cs.ks;
    const int s = m + j - cs.ks / 2;
    if (s < 0 || s >= cs.rows_out) return 0.0f;
    const int src = LOAD == kLoadConvUp2 ? s >> 1 : s;  // nearest x2: floor(s * 0.5)
    return cs.x[(size_t)src * cs.ch + c];
}

// C[M, N] = A[M, K] . W[N, K]^T + bias, epilogue EPI; K % 32 == 0.
template <int LOAD, int EPI>
__global__ void __launch_bounds__(256) k_codec_gemm(const float* __restrict__ A, ConvSrc cs, const float* __restrict__ W,
                                                    const float* __restrict__ bias, const float* __restrict__ gamma,
                                                    const float* R, float* C, int M, int N, int K) {
    constexpr int BM = 64, BN = 64, BK = 32;
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Ws[2][BK][BN + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int lr = tid >> 2, lk = (tid & 3) * 4;  // rows lr, k lk..lk+3 and lk+16..lk+19
    float ra[8], rw[8];
    auto gload = [&](int k0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int kk = k0 + lk + 16 * h;
            const int m = m0 + lr, n = n0 + lr;
            if (LOAD == kLoadPlain && m < M) {
                const float4 v = *reinterpret_cast<const float4*>(A + (size_t)m * K + kk);
                ra[4 * h] = v.x, ra[4 * h + 1] = v.y, ra[4 * h + 2] = v.z, ra[4 * h + 3] = v.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) ra[4 * h + e] = m < M ? load_a<LOAD>(A, K, cs, m, kk + e) : 0.0f;
            }
            if (n < N) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(W + (size_t)n * K + kk));
                rw[4 * h] = v.x, rw[4 * h + 1] = v.y, rw[4 * h + 2] = v.z, rw[4 * h + 3] = v.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) rw[4 * h + e] = 0.0f;
            }
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                As[buf][lk + 16 * h + e][lr] = ra[4 * h + e];
                Ws[buf][lk + 16 * h + e][lr] = rw[4 * h + e];
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
            if (EPI == kCEpiGelu)
                out = gelu_erf(y);
            else if (EPI == kCEpiScaleResid)
                out = R[(size_t)m * N + n] + y * gamma[n];  // x + gamma * pwconv2(.) (codec.cpp:46)
            else
                out = y;
            C[(size_t)m * N + n] = out;
        }
    }
}

// EnhancedCodec::lookup (codec.cpp:50-56): codebook row (8 values) of each
// code, then out_project 8 -> 1024 with its bias.
__global__ void k_codec_lookup(const uint32_t* __restrict__ codes, const float* __restrict__ cb,
                               const float* __restrict__ W, const float* __restrict__ b, float* __restrict__ out, int T) {
    const int t = blockIdx.x;
    __shared__ float e[8];
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x < 8) e[threadIdx.x] = cb[(size_t)codes[t] * 8 + threadIdx.x];
    __syncthreads();
    for (int o = threadIdx.x; o < 1024; o += blockDim.x) {
        float acc = 0.f;
#pragma unroll
        for (int d = 0; d < 8; ++d) acc = fmaf(W[o * 8 + d], e[d], acc);
        out[(size_t)t * 1024 + o] = acc + b[o];
    }
}

// LayerNorm over rows of `width` (<= 1024) values: mean, then the mean of
// squared deviations (biased), eps inside the root (kernels.metal:618-669).
__global__ void __launch_bounds__(128) k_codec_ln(const float* __restrict__ x, const float* __restrict__ g,
                                                  const float* __restrict__ be, float* __restrict__ out, int width,
                                                  float eps, float* __restrict__ out_lo = nullptr) {
    __shared__ float red[32];
    pdl_trigger();
    pdl_wait();
    const float* row = x + (size_t)blockIdx.x * width;
    float v[8];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = threadIdx.x + 128 * j;
        v[j] = c < width ? row[c] : 0.f;
        s += v[j];
    }
    const float mean = block_sum(s, red) / float(width);
    float q = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = threadIdx.x + 128 * j;
        if (c < width) {
            const float d = v[j] - mean;
            q = fmaf(d, d, q);
        }
    }
    const float var = block_sum(q, red) / float(width);
    const float inv = 1.0f / sqrtf(var + eps);
    float* o = out + (size_t)blockIdx.x * width;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int c = threadIdx.x + 128 * j;
        if (c < width) {
            const float y = (v[j] - mean) * inv * g[c] + be[c];
            if (out_lo) {  // split for the tensor-core GEMM: y = hi + lo
                const float hi = rn_tf32(y);
                o[c] = hi;
                out_lo[(size_t)blockIdx.x * width + c] = rn_tf32(y - hi);
            } else {
                o[c] = y;
            }
        }
    }
}

// im2col of a same-padded convolution over time, split into TF32 hi / lo for
// the tensor-core GEMM: row t, column c * ks + j holds x[t + j - ks/2][c]
// (zero outside [0, rows_out)), read from the nearest x2 upsampled rows
// x[floor(s / 2)] when up2 (the A operand load_a computes on the fly).
__global__ void k_codec_im2col(const float* __restrict__ x, int ch, int ks, int rows_out, int up2,
                               float* __restrict__ hi, float* __restrict__ lo) {
    const size_t width = (size_t)ch * ks, n = (size_t)rows_out * width;
    pdl_trigger();
    pdl_wait();
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int t = int(e / width), kk = int(e % width), c = kk / ks, j = kk - c * ks;
        const int s = t + j - ks / 2;
        const float v = s >= 0 && s < rows_out ? x[(size_t)(up2 ? s >> 1 : s) * ch + c] : 0.0f;
        const float h = rn_tf32(v);
        hi[e] = h;
        lo[e] = rn_tf32(v - h);
    }
}

// Depthwise same-padded convolution over time (kernels.metal:1516-1540).
__global__ void k_codec_dwconv(const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ b,
                               float* __restrict__ out, int T, int ch, int ks) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    pdl_trigger();
    pdl_wait();
    if (c >= ch) return;
    float acc = 0.f;
    for (int j = 0; j < ks; ++j) {
        const int s = t + j - ks / 2;
        if (s >= 0 && s < T) acc = fmaf(x[(size_t)s * ch + c], w[c * ks + j], acc);
    }
    out[(size_t)t * ch + c] = acc + b[c];
}

template <int LOAD, int EPI>
cudaError_t gemm(const float* A, ConvSrc cs, const float* W, const float* bias, const float* gamma, const float* R,
                 float* C, int M, int N, int K, cudaStream_t s) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    k_codec_gemm<LOAD, EPI><<<grid, 256, 0, s>>>(A, cs, W, bias, gamma, R, C, M, N, K);
    return cudaGetLastError();
}

}  // namespace

namespace {

constexpr int kD = 384, kF = 2048, kH = 1024;

// Tensor maps of the split activations for T rows (re-encoded when T changes;
// the block grows to the largest T seen).
cudaError_t codec_tc_rows(CodecTc* tc, int T) {
    if (tc->rows == T) return cudaSuccess;
    const size_t per_row = size_t(kH) * 7 + kD + kF + 2 * size_t(kH) * 3;  // col_e, ln, u, col_u (2 rows)
    cudaError_t e;
    if (T > tc->act_cap) {
        if (tc->act) cudaFree(tc->act);
        tc->act = nullptr;
        tc->act_cap = 0;
        if ((e = cudaMalloc(&tc->act, 2 * per_row * size_t(T) * sizeof(float))) != cudaSuccess) return e;
        tc->act_cap = T;
    }
    float* p = tc->act;
    auto take = [&](float* (&pair)[2], size_t n) {
        pair[0] = p;
        pair[1] = p + n;
        p += 2 * n;
    };
    const size_t cap = size_t(tc->act_cap);
    take(tc->col_e, cap * kH * 7);
    take(tc->ln, cap * kD);
    take(tc->u, cap * kF);
    take(tc->col_u, 2 * cap * kH * 3);
    for (int h = 0; h < 2; ++h) {
        if ((e = tma_make_map(&tc->a_col_e[h], tc->col_e[h], T, kH * 7)) != cudaSuccess ||
            (e = tma_make_map(&tc->a_ln[h], tc->ln[h], T, kD)) != cudaSuccess ||
            (e = tma_make_map(&tc->a_u[h], tc->u[h], T, kF)) != cudaSuccess ||
            (e = tma_make_map(&tc->a_col_u[h], tc->col_u[h], 2 * T, kH * 3)) != cudaSuccess)
            return e;
    }
    tc->rows = T;
    return cudaSuccess;
}

cudaError_t tc_gemm(CodecTc* tc, const TmaMap* a, const TmaMap* w, int epi, const float* bias, const float* R,
                    const float* gamma, float* C, float* C_lo, int M, int N, int K, cudaStream_t s) {
    TmaGemm g{a, w, bias, R, C, C_lo, M, N, K, epi, tc->ws, tc->counters, kCodecCounters, tc->status, gamma};
    return tma_gemm(g, s);
}

}  // namespace

cudaError_t codec_tc_init(CodecTc* tc, const CodecWeights& w, cudaStream_t s) {
    struct Mat {
        const float* src;
        int rows, cols;
        TmaMap* maps;
    };
    std::vector<Mat> mats;
    mats.push_back({w.embed_w, kD, kH * 7, tc->w_embed});
    for (int i = 0; i < 12; ++i) {
        mats.push_back({w.block[i].pw1_w, kF, kD, tc->w_pw1[i]});
        mats.push_back({w.block[i].pw2_w, kD, kF, tc->w_pw2[i]});
    }
    mats.push_back({w.head_w, kH, kD, tc->w_head});
    mats.push_back({w.up_w, kH, kH * 3, tc->w_up});
    size_t total = 0;
    for (const Mat& m : mats) total += 2 * size_t(m.rows) * m.cols;
    cudaError_t e;
    if ((e = cudaMalloc(&tc->wsplit, total * sizeof(float))) != cudaSuccess) return e;
    float* p = tc->wsplit;
    for (const Mat& m : mats) {
        const size_t n = size_t(m.rows) * m.cols;
        if ((e = tma_split(m.src, p, p + n, n, s)) != cudaSuccess ||
            (e = tma_make_map(&m.maps[0], p, m.rows, m.cols)) != cudaSuccess ||
            (e = tma_make_map(&m.maps[1], p + n, m.rows, m.cols)) != cudaSuccess)
            return e;
        p += 2 * n;
    }
    if ((e = cudaMalloc(&tc->ws, tma_workspace_floats() * sizeof(float))) != cudaSuccess ||
        (e = cudaMalloc(&tc->counters, (kCodecCounters + 1) * sizeof(int))) != cudaSuccess)
        return e;
    tc->status = tc->counters + kCodecCounters;
    if ((e = cudaMemsetAsync(tc->counters, 0, (kCodecCounters + 1) * sizeof(int), s)) != cudaSuccess) return e;
    return cudaStreamSynchronize(s);
}

void codec_tc_free(CodecTc* tc) {
    for (void* p : {(void*)tc->wsplit, (void*)tc->act, (void*)tc->ws, (void*)tc->counters})
        if (p) cudaFree(p);
    *tc = CodecTc{};
}

// The decode of T codes (host-validated: 1 <= T <= 5000, codes < 8192) on
// stream s; out receives [2T, 1024].
cudaError_t codec_decode_device(const CodecWeights& w, const CodecScratch& sc, CodecTc* tc, const uint32_t* d_codes,
                                int T, float* out, cudaStream_t s) {
    constexpr int D = kD, F = kF, H = kH;
    const ConvSrc none{nullptr, 0, 1, 0};
    cudaError_t e;
    k_codec_lookup<<<T, 256, 0, s>>>(d_codes, w.codebook, w.out_w, w.out_b, sc.hidden, T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (tc) {
        // tensor-core GEMMs (TF32 hi / lo, three products): the activations
        // that feed a GEMM are written split by the kernel producing them
        if ((e = codec_tc_rows(tc, T)) != cudaSuccess) return e;
        // a CTA that gave up leaves its tile's counter behind
        if ((e = cudaMemsetAsync(tc->counters, 0, kCodecCounters * sizeof(int), s)) != cudaSuccess) return e;
        // every kernel of this chain is launched with PDL (it waits for its
        // predecessor before touching the buffers they share)
        const int grid = 148 * 8;
        float* none_lo = nullptr;
        if ((e = launch_pdl(k_codec_im2col, dim3(grid), 256, 0, s, (const float*)sc.hidden, H, 7, T, 0, tc->col_e[0],
                            tc->col_e[1])) != cudaSuccess ||
            (e = tc_gemm(tc, tc->a_col_e, tc->w_embed, TmaEpiBias, w.embed_b, nullptr, nullptr, sc.h, nullptr, T, D,
                         H * 7, s)) != cudaSuccess ||
            (e = launch_pdl(k_codec_ln, dim3(T), 128, 0, s, (const float*)sc.h, w.norm_g, w.norm_b, sc.x, D, 1e-6f,
                            none_lo)) != cudaSuccess)
            return e;
        for (int i = 0; i < 12; ++i) {
            const CodecBlockW& bw = w.block[i];
            if ((e = launch_pdl(k_codec_dwconv, dim3((D + 127) / 128, T), 128, 0, s, (const float*)sc.x, bw.dw_w,
                                bw.dw_b, sc.h, T, D, 7)) != cudaSuccess ||
                (e = launch_pdl(k_codec_ln, dim3(T), 128, 0, s, (const float*)sc.h, bw.ln_g, bw.ln_b, tc->ln[0], D,
                                1e-6f, tc->ln[1])) != cudaSuccess)
                return e;
            if ((e = tc_gemm(tc, tc->a_ln, tc->w_pw1[i], TmaEpiGeluErf, bw.pw1_b, nullptr, nullptr, tc->u[0],
                             tc->u[1], T, F, D, s)) != cudaSuccess ||
                (e = tc_gemm(tc, tc->a_u, tc->w_pw2[i], TmaEpiScaleResid, bw.pw2_b, sc.x, bw.gamma, sc.x, nullptr, T,
                             D, F, s)) != cudaSuccess)
                return e;
        }
        if ((e = launch_pdl(k_codec_ln, dim3(T), 128, 0, s, (const float*)sc.x, w.final_g, w.final_b, tc->ln[0], D,
                            1e-6f, tc->ln[1])) != cudaSuccess ||
            (e = tc_gemm(tc, tc->a_ln, tc->w_head, TmaEpiBias, w.head_b, nullptr, nullptr, sc.hidden, nullptr, T, H,
                         D, s)) != cudaSuccess ||
            (e = launch_pdl(k_codec_im2col, dim3(grid), 256, 0, s, (const float*)sc.hidden, H, 3, 2 * T, 1,
                            tc->col_u[0], tc->col_u[1])) != cudaSuccess)
            return e;
        return tc_gemm(tc, tc->a_col_u, tc->w_up, TmaEpiBias, w.up_b, nullptr, nullptr, out, nullptr, 2 * T, H,
                       H * 3, s);
    }
    // CUDA-core GEMMs
    // embed conv k=7 1024 -> 384, LayerNorm
    if ((e = gemm<kLoadConv, kCEpiBias>(nullptr, ConvSrc{sc.hidden, H, 7, T}, w.embed_w, w.embed_b, nullptr, nullptr,
                                        sc.h, T, D, H * 7, s)) != cudaSuccess)
        return e;
    k_codec_ln<<<T, 128, 0, s>>>(sc.h, w.norm_g, w.norm_b, sc.x, D, 1e-6f);
    for (int i = 0; i < 12; ++i) {
        const CodecBlockW& bw = w.block[i];
        k_codec_dwconv<<<dim3((D + 127) / 128, T), 128, 0, s>>>(sc.x, bw.dw_w, bw.dw_b, sc.h, T, D, 7);
        k_codec_ln<<<T, 128, 0, s>>>(sc.h, bw.ln_g, bw.ln_b, sc.h, D, 1e-6f);
        if ((e = gemm<kLoadPlain, kCEpiGelu>(sc.h, none, bw.pw1_w, bw.pw1_b, nullptr, nullptr, sc.u, T, F, D, s)) !=
            cudaSuccess)
            return e;
        // x <- x + gamma * (pwconv2(u) + b), in place (each output reads only its own residual)
        if ((e = gemm<kLoadPlain, kCEpiScaleResid>(sc.u, none, bw.pw2_w, bw.pw2_b, bw.gamma, sc.x, sc.x, T, D, F, s)) !=
            cudaSuccess)
            return e;
    }
    k_codec_ln<<<T, 128, 0, s>>>(sc.x, w.final_g, w.final_b, sc.h, D, 1e-6f);
    if ((e = gemm<kLoadPlain, kCEpiBias>(sc.h, none, w.head_w, w.head_b, nullptr, nullptr, sc.hidden, T, H, D, s)) !=
        cudaSuccess)
        return e;
    // nearest x2 + conv k=3 1024 -> 1024 over 2T rows
    return gemm<kLoadConvUp2, kCEpiBias>(nullptr, ConvSrc{sc.hidden, H, 3, 2 * T}, w.up_w, w.up_b, nullptr, nullptr,
                                         out, 2 * T, H, H * 3, s);
}

}  // namespace itts
