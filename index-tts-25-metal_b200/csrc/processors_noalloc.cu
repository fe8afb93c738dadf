// itts_gpt_apply_processors_noalloc: the logits processors of
// itts_gpt_apply_processors for callers that must not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc/cudaFree are off limits --
// a latency-critical serving thread (cudaMalloc and cudaFree can synchronise
// the whole device and stall every stream on it), or a process whose device
// memory is already fully reserved by another allocator (a serving framework's
// memory pool that takes nearly all of HBM up front).  The regular entry point
// stages its inputs in buffers owned by a context and may grow its history
// buffer with cudaMalloc; this one needs no context and allocates nothing.
// It is synchronous: it copies the inputs in, runs one kernel and copies the
// scores back with blocking cudaMemcpy calls, and returns when they are on
// the host.
//
// Scratch: one file-scope __device__ array (kNoAllocScratchBytes, below) that
// every GPU loading this library holds until the process exits.  It stages the
// 8194 input logits, the output scores, up to kNoAllocMaxHistory history
// tokens and the status word.  All calls share it and it keeps the last call's
// contents: the status word is cleared on every call; logits, history and
// scores are overwritten in full before they are read.  Calls that overlap on
// the same GPU (two host threads at once) race on the array; serialise them.
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress while that device is current and caches it; make that
// first call before any stream capture begins.
#include <mutex>
#include <string>

#include "common.cuh"
#include "itts_gpt.h"
#include "model.hpp"
#include "sampler.cuh"

namespace itts {

// Stores `msg` where itts_gpt_last_error(NULL) reads it (itts_gpt.cpp).
void set_thread_error(const std::string& msg);

constexpr uint32_t kNoAllocMaxHistory = 16384;
constexpr int kNoAllocMaxDevices = 64;

struct NoAllocScratch {
    float logits[8448];
    float scores[8448];
    uint32_t history[kNoAllocMaxHistory];
    int status[4];
};
constexpr size_t kNoAllocScratchBytes = sizeof(NoAllocScratch);  // 133,136 bytes

// Device-side storage.  In host code this name is only a stand-in symbol: its
// device address comes from cudaGetSymbolAddress (see scratch_on()).
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

size_t sampler_dyn_smem_bytes();
constexpr size_t kSmallBytes = (sizeof(SamplerSmem) + 15) & ~size_t(15);

__global__ void __launch_bounds__(kThreads, 1) k_processors_noalloc(NoAllocScratch* s, SampleOpts o, uint32_t hist_n) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(smem_raw);
    SamplerBig* big = reinterpret_cast<SamplerBig*>(smem_raw + kSmallBytes);
    sampler_init_seen(sm, s->history, hist_n);
    run_sampler(s->logits, o, 0, false, sm, big, s->scores, s->status);
}

namespace {
std::mutex g_setup_mu;
NoAllocScratch* g_scratch_ptr[kNoAllocMaxDevices] = {};

// One-time set-up per device (the caller has made `device` current).
cudaError_t scratch_on(int device, NoAllocScratch** out) {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(k_processors_noalloc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sampler_dyn_smem_bytes());
        if (e != cudaSuccess) return e;
        g_scratch_ptr[device] = static_cast<NoAllocScratch*>(p);
    }
    *out = g_scratch_ptr[device];
    return cudaSuccess;
}

int fail(int code, const std::string& msg) {
    set_thread_error(msg);
    return code;
}
}  // namespace

}  // namespace itts

extern "C" int itts_gpt_apply_processors_noalloc(int device, const float* logits, size_t n, const uint32_t* history,
                                                 size_t history_n, const itts_gen_opts* opts, float* out) {
    using namespace itts;
    set_thread_error("");
    if (!logits || !out || !opts || (history_n && !history)) return fail(ITTS_ERR_INVALID_ARGUMENT, "null argument");
    if (n != (size_t)kVocab) return fail(ITTS_ERR_INVALID_ARGUMENT, "logits must have 8194 entries");
    if (history_n > kNoAllocMaxHistory)
        return fail(ITTS_ERR_INVALID_ARGUMENT, "history has " + std::to_string(history_n) +
                                                   " tokens; the allocation-free entry point stages at most " +
                                                   std::to_string(kNoAllocMaxHistory));
    if (device < 0 || device >= kNoAllocMaxDevices) return fail(ITTS_ERR_INVALID_ARGUMENT, "device index out of range");
    // gpt_sampling.cpp:33-71 error checks (same as itts_gpt_apply_processors)
    if (opts->repetition_penalty != 1.0f && opts->repetition_penalty <= 0.0f)
        return fail(ITTS_ERR_RUNTIME, "GPT repetition penalty must be positive");
    if (opts->temperature <= 0.0f) return fail(ITTS_ERR_RUNTIME, "GPT sampling temperature must be positive");
    if (opts->top_p < 1.0f && opts->top_p <= 0.0f) return fail(ITTS_ERR_RUNTIME, "GPT top_p must be in (0, 1]");

    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return fail(ITTS_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if ((e = cudaSetDevice(device)) != cudaSuccess)
        return fail(ITTS_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    NoAllocScratch* s = nullptr;
    int rc = ITTS_OK;
    std::string msg;
    auto ck = [&](cudaError_t err, const char* what) {
        if (err != cudaSuccess && rc == ITTS_OK) {
            rc = ITTS_ERR_CUDA;
            msg = std::string(what) + ": " + cudaGetErrorString(err);
        }
        return rc == ITTS_OK;
    };
    if (ck(scratch_on(device, &s), "cudaGetSymbolAddress") &&
        ck(cudaMemcpy(s->logits, logits, kVocab * sizeof(float), cudaMemcpyHostToDevice), "logits upload") &&
        (!history_n || ck(cudaMemcpy(s->history, history, history_n * 4, cudaMemcpyHostToDevice), "history upload")) &&
        ck(cudaMemset(s->status, 0, sizeof(s->status)), "status clear")) {
        const SampleOpts o{opts->do_sample, opts->top_k, opts->seed, opts->temperature, opts->top_p,
                           opts->repetition_penalty, opts->num_beams, opts->rng};
        k_processors_noalloc<<<1, kThreads, sampler_dyn_smem_bytes()>>>(s, o, uint32_t(history_n));
        int status[4] = {0, 0, 0, 0};
        if (ck(cudaGetLastError(), "processors launch") &&
            ck(cudaMemcpy(out, s->scores, kVocab * sizeof(float), cudaMemcpyDeviceToHost), "scores read") &&
            ck(cudaMemcpy(status, s->status, sizeof(status), cudaMemcpyDeviceToHost), "status read") && status[0]) {
            // the device status codes the processors can raise, mapped as the
            // context entry points map them (check_status in itts_gpt.cpp)
            rc = ITTS_ERR_RUNTIME;
            switch (status[0]) {
                case kStatusNoFiniteLogits: msg = "GPT top_p filtering removed all logits"; break;
                case kStatusZeroMass: msg = "GPT sampling probability mass is zero"; break;
                default:
                    msg = "device error " + std::to_string(status[0]) + " (site " + std::to_string(status[1]) +
                          ", detail " + std::to_string(status[3]) + ")";
                    break;
            }
        }
    }
    cudaSetDevice(prev);
    if (rc != ITTS_OK) return fail(rc, msg);
    return ITTS_OK;
}
