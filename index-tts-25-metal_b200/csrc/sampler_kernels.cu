// Single-CTA kernels around the sampler (sampler.cuh): the layered decode
// path's per-token selection, the processors entry point and the beam-search
// candidate scores.
#include "common.cuh"
#include "model.hpp"
#include "sampler.cuh"

namespace itts {

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
    // The reference sums std::exp(v - peak) in float, one term after another
    // in index order, then adds std::log(sum) to the peak.  Each exp and the
    // log are rounded once from double (correctly rounded up to rare ties,
    // where the host's libm may round differently) and one thread adds the
    // terms in index order.
    float* terms = big->sv_s;  // the sampler's workspace is free until run_sampler
#pragma unroll
    for (int k = 0; k < kPer; ++k)
        if (k < cnt) terms[base + k] = (float)exp((double)(v[k] - peak));
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.f;
        for (int i = 0; i < kVocab; ++i) sum += terms[i];
        sm.redf[0] = peak + (float)log((double)sum);
    }
    __syncthreads();
    const float log_sum = sm.redf[0];
    __syncthreads();  // sm.redf is reused by the sampler below
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

// Layered batched generate loop, global draw st->step of every active row (one
// CTA per row; row m's draw index is st->step - base[m]):
// the processors and the token choice of the batch-1 loop (k_decode's
// sample_next) on the row's logits, then the row's bookkeeping -- code,
// count, stop (gpt_sampling.cpp:178-187) and repetition-penalty set.  The last
// CTA to finish advances st->step.
__global__ void __launch_bounds__(kThreads, 1) k_batch_sample(BatchArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    SamplerBig* big = reinterpret_cast<SamplerBig*>(smem_raw + kSamplerSmallBytes);
    BatchState* st = a.st;
    const uint32_t m = blockIdx.x;
    const uint32_t gstep = (uint32_t)ld_volatile((const int*)&st->step);
    const uint32_t i = gstep - st->base[m];
    const bool active = (ld_volatile((const int*)&st->active) >> m) & 1;
    int* status = a.d.b.ctl->status;
    if (active) {
        uint32_t* seen = a.seen + (size_t)m * kSeenWords;
        for (int k = threadIdx.x; k < kBits; k += kThreads) sm.seen[k] = seen[k];
        __syncthreads();
        const SampleOpts& o = a.opts[m];
        // draw 0 reads the prefill's raw logits; later draws read the head's scaled scores
        const uint32_t token = run_sampler(a.logits + (size_t)m * kBatchLogitsStride, o, i, o.do_sample == 0, sm, big,
                                           nullptr, status, a.scaled_head && i > 0);
        if (threadIdx.x == 0) {
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
    }
    if (threadIdx.x == 0) {
        __threadfence();
        const uint32_t old = atomicAdd(&st->sample_arrivals, 1u);
        if (old == a.M - 1) {
            st->sample_arrivals = 0;
            st->step = gstep + 1;
        }
    }
}

// ------------------------------------------------------------ host side
size_t sampler_big_bytes() { return sizeof(SamplerBig); }
size_t sampler_dyn_smem_bytes() { return kSamplerDynSmem; }

cudaError_t sampler_configure() {
    for (const void* f : {(const void*)k_layer_sample, (const void*)k_processors, (const void*)k_beam_scores,
                          (const void*)k_batch_sample}) {
        const cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSamplerDynSmem);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_layer_sample(const DecodeArgs& a, uint32_t i, cudaStream_t s) {
    k_layer_sample<<<1, kThreads, kSamplerDynSmem, s>>>(a, i);
    return cudaGetLastError();
}

cudaError_t launch_layer_finish(const DecodeArgs& a, cudaStream_t s) {
    k_layer_finish<<<1, 1, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_batch_sample(const BatchArgs& a, cudaStream_t s) {
    k_batch_sample<<<a.M, kThreads, kSamplerDynSmem, s>>>(a);
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
