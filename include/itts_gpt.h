/*
 * itts_gpt.h — C-ABI of the B200 (sm_100a) IndexTTS 2.5 GPT (UnifiedVoice)
 * decoder.  It replaces, one for one, the interface the reference exposes in
 * include/itts25/gpt.hpp:7-43 (GenerationOptions, GenerationResult, GptState,
 * GptDecoder and apply_gpt_sampling_processors), so that a host (the C++
 * adapter in index-tts-25-metal_b200/host/gpt_decoder.hpp, a ctypes or cgo
 * binding) can drop it in where src/pipeline.cpp:23-25 and
 * src/native_runtime.cpp:99 call GptDecoder.
 *
 * Conventions
 *  - Every call returns an itts_status; 0 is success.  No C++ exception
 *    crosses this boundary.  The message of the last failure on a context is
 *    returned by itts_gpt_last_error(ctx); failures of itts_gpt_create (no
 *    context yet) are reported by itts_gpt_last_error(NULL) on the same thread.
 *  - Status classes mirror the exceptions of the reference:
 *      ITTS_ERR_INVALID_ARGUMENT  <- std::invalid_argument (shapes, capacity,
 *                                    ids, options: gpt.cpp:42-85,
 *                                    gpt_sampling.cpp:168-173)
 *      ITTS_ERR_RUNTIME           <- std::runtime_error (bundle/shape checks,
 *                                    invalid generated code, empty sampling
 *                                    mass: gpt.cpp:8-23, gpt_sampling.cpp)
 *      ITTS_ERR_LOGIC             <- std::logic_error (call-order misuse)
 *    plus device-side classes the reference does not have.
 *  - Threading: a context is not thread-safe; use one context per host thread
 *    and device.  There is no global mutable state besides the per-thread
 *    create-error string.  Calls are synchronous unless named *_async.
 *  - Float arrays are row-major fp32; code ids are uint32.
 */
#ifndef ITTS_GPT_H
#define ITTS_GPT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ITTS_GPT_WIDTH 1280        /* d_model (gpt.cpp:7) */
#define ITTS_GPT_VOCAB 8194        /* mel code vocabulary incl. start/stop */
#define ITTS_GPT_START_CODE 8192
#define ITTS_GPT_STOP_CODE 8193
#define ITTS_GPT_KV_CAPACITY 4096  /* cache_capacity (gpt.cpp:7) */
#define ITTS_GPT_MAX_PREFIX_ROWS 1024
#define ITTS_GPT_SPEAKER_DIM 192
#define ITTS_GPT_MAX_BEAMS 10

typedef enum itts_status {
    ITTS_OK = 0,
    ITTS_ERR_INVALID_ARGUMENT = -1,
    ITTS_ERR_RUNTIME = -2,
    ITTS_ERR_LOGIC = -3,
    ITTS_ERR_CUDA = -4,           /* a CUDA runtime call failed */
    ITTS_ERR_OUT_OF_MEMORY = -5,  /* device or pinned-host allocation failed */
    ITTS_ERR_DEVICE_TIMEOUT = -6  /* a bounded device-side wait gave up */
} itts_status;

typedef enum itts_weight_dtype {
    ITTS_WEIGHTS_F32 = 0,  /* fp32 weights, fp32 KV (reference numerics) */
    ITTS_WEIGHTS_BF16 = 1  /* bf16 matrices, fp32 LN/bias/KV/accumulation */
} itts_weight_dtype;

typedef enum itts_rng {
    ITTS_RNG_SPLITMIX64 = 0, /* the reference's stream (gpt_sampling.cpp:11-26) */
    ITTS_RNG_PHILOX = 1      /* Philox4x32-10, counter = draw index, key = seed */
} itts_rng;

/* GenerationOptions (include/itts25/gpt.hpp:7-16) plus the uniform-stream
 * selector.  itts_gen_opts_default() fills the reference defaults. */
typedef struct itts_gen_opts {
    int32_t do_sample;
    uint32_t top_k;
    uint64_t seed;
    float temperature;
    float top_p;
    float repetition_penalty;
    uint32_t num_beams;
    float length_penalty;
    int32_t rng; /* itts_rng */
} itts_gen_opts;

typedef struct itts_gpt_ctx itts_gpt_ctx;
/* GptState (gpt.hpp:18): a KV-cache checkpoint held in device memory. */
typedef struct itts_gpt_state itts_gpt_state;

typedef struct itts_gpt_info {
    uint32_t layers;          /* transformer blocks found in the bundle */
    uint32_t mel_pos_rows;    /* rows of gpt.mel_pos_embedding */
    uint32_t text_pos_rows;   /* rows of gpt.text_pos_embedding */
    uint32_t sm_count;        /* SMs of the device (persistent grid size) */
    uint64_t weight_bytes;    /* device bytes held by the weights */
    uint64_t stream_bytes;    /* weight bytes one decode step reads */
    int32_t weight_dtype;
    int32_t device;
} itts_gpt_info;

/* ---- options ---------------------------------------------------------- */
void itts_gen_opts_default(itts_gen_opts* opts);

/* ---- lifecycle (replaces GptDecoder::GptDecoder, gpt.cpp:8-23) ----------
 * Loads an MIT2 bundle (manifest.json + weights.bin, target "index-tts2.5"),
 * validates the GPT tensor shapes, uploads the weights to `device` (Conv1D
 * matrices transposed on the device) and allocates the KV arena.  The layer
 * count is taken from the bundle (1..24); the reference requires 24. */
int itts_gpt_create(const char* bundle_dir, int device, int weight_dtype, itts_gpt_ctx** out);
void itts_gpt_destroy(itts_gpt_ctx* ctx);
const char* itts_gpt_last_error(const itts_gpt_ctx* ctx);  /* NULL: this thread's last create / noalloc error */
int itts_gpt_get_info(const itts_gpt_ctx* ctx, itts_gpt_info* info);

/* ---- GptDecoder::prepare (gpt.cpp:42-71) ----------------------------------
 * speaker[192], emotion[1280], text ids (0 and 1 are dropped, framed by 0..1),
 * language < 107.  Writes rows*1280 floats (rows = 3 + ids + 2 + 1) into out
 * (capacity out_floats) and the row count into *rows. */
int itts_gpt_prepare(itts_gpt_ctx* ctx, const float* speaker, size_t speaker_n, const float* emotion,
                     size_t emotion_n, const uint32_t* text, size_t text_n, uint32_t language, float* out,
                     size_t out_floats, size_t* rows);

/* ---- GptDecoder::prefill (gpt.cpp:72-78) ----------------------------------
 * prefix: n_floats = rows*1280 host floats, 1 <= rows <= 1024.  Resets the KV
 * cache, runs the prefix, writes the last row's 8194 logits. */
int itts_gpt_prefill(itts_gpt_ctx* ctx, const float* prefix, size_t n_floats, float* logits);

/* ---- GptDecoder::step (gpt.cpp:79-85) -------------------------------------
 * One cached decode step for `code` (< 8194) at mel position `position`. */
int itts_gpt_step(itts_gpt_ctx* ctx, uint32_t code, uint32_t position, float* logits);

/* ---- GptDecoder::generate (gpt_sampling.cpp:168-245) ----------------------
 * Prefill + the whole token loop on the device (greedy or sampled; beam search
 * for num_beams > 1).  codes needs max_tokens entries; the stop code is not
 * stored; *stopped is 1 when the stop code ended the loop. */
int itts_gpt_generate(itts_gpt_ctx* ctx, const float* prefix, size_t n_floats, const itts_gen_opts* opts,
                      uint32_t max_tokens, uint32_t* codes, uint32_t* n_codes, int* stopped);

/* ---- batch of independent requests ----------------------------------------
 * Request i is the prefix prefixes[i] (n_floats[i] floats) with options
 * opts[i].  Requests without beams are decoded together, up to 16 per group:
 * each is prefilled into its own KV arena, then one batched forward step per
 * token reads every weight once for all of them.  Each request's codes are
 * exactly those itts_gpt_generate returns for it alone (same arithmetic per
 * row).  Beam requests run one at a time.  Codes of request i go to
 * codes + i * max_tokens, its count to n_codes[i], its stop flag to
 * stopped[i].  Every request is validated before any runs.  No single call
 * of the reference corresponds: its server runs GptDecoder::generate once per
 * request (src/server.cpp:41-47); this is that loop behind one call.
 * Afterwards the context holds no prefill (itts_gpt_step needs a new
 * itts_gpt_prefill); the same holds after a beam-search generate. */
int itts_gpt_generate_batch(itts_gpt_ctx* ctx, size_t batch, const float* const* prefixes, const size_t* n_floats,
                            const itts_gen_opts* opts, uint32_t max_tokens, uint32_t* codes, uint32_t* n_codes,
                            int* stopped);

/* ---- continuous batching --------------------------------------------------
 * The serving loop: request i (prefix prefixes[i], options opts[i], at most
 * max_tokens[i] codes into codes[i]) is decoded as generate would decode it
 * alone, with up to max_rows (<= 16) requests in flight on the device: each
 * batched step reads the weights once for every row in flight, and a row
 * whose request finished takes the next request (in the given order) at the
 * next host sync point.  n_codes[i] / stopped[i] as in itts_gpt_generate.
 * Requests with num_beams > 1 are rejected.  No single call of the
 * reference corresponds: its server runs GptDecoder::generate once per
 * request (src/server.cpp:41-47, gpt_sampling.cpp:168-189).  Afterwards the
 * context holds no prefill. */
int itts_gpt_serve(itts_gpt_ctx* ctx, size_t n, const float* const* prefixes, const size_t* n_floats,
                   const itts_gen_opts* opts, const uint32_t* max_tokens, uint32_t max_rows, uint32_t* const* codes,
                   uint32_t* n_codes, int* stopped);

/* ---- GptDecoder::checkpoint / restore / cached_tokens (gpt.cpp:86-87) ----- */
int itts_gpt_checkpoint(itts_gpt_ctx* ctx, itts_gpt_state** out);
int itts_gpt_restore(itts_gpt_ctx* ctx, const itts_gpt_state* state);
void itts_gpt_state_free(itts_gpt_state* state);
uint32_t itts_gpt_cached_tokens(const itts_gpt_ctx* ctx);

/* ---- apply_gpt_sampling_processors (gpt.hpp:19, gpt_sampling.cpp:28-128) --
 * Runs the on-device logits processors (repetition penalty over the unique
 * history, temperature, top-k, top-p) on n = 8194 host logits; removed entries
 * become -inf.  Options are taken as given (no do_sample remapping). */
int itts_gpt_apply_processors(itts_gpt_ctx* ctx, const float* logits, size_t n, const uint32_t* history,
                              size_t history_n, const itts_gen_opts* opts, float* out);

/* ---- device-resident, stream-ordered interface -----------------------------
 * For callers whose data already lives on the device (and for benchmarking
 * with inputs resident in HBM).  Work is queued on the context's stream; the
 * pointers are device pointers.  itts_gpt_decode_async continues from the
 * most recent prefill and samples its first code from that prefill's logits;
 * d_info receives {n_codes, stopped, status, forward_steps}.  itts_gpt_sync
 * waits for the stream and reports device-side failures. */
int itts_gpt_stream(itts_gpt_ctx* ctx, void** cuda_stream);
int itts_gpt_prefill_async(itts_gpt_ctx* ctx, const float* d_prefix, uint32_t rows, float* d_logits);
int itts_gpt_decode_async(itts_gpt_ctx* ctx, const itts_gen_opts* opts, uint32_t max_tokens, uint32_t* d_codes,
                          uint32_t* d_info);
int itts_gpt_sync(itts_gpt_ctx* ctx);

/* ---- diagnostics ------------------------------------------------------------
 * mode 0: persistent decode (one cooperative launch per token loop, grid
 * barriers between phases; default); mode 1: layered decode (one launch per
 * phase, same device code).  Counters: kernel launches issued by the context. */
int itts_gpt_set_decode_mode(itts_gpt_ctx* ctx, int mode);
/* Prefill GEMMs of an fp32-weight context.  mode 0 (default): tcgen05 tensor
 * cores, operands split into two TF32 words (hi, lo) and three products per
 * term, accumulator drained to fp32 every 128 K; mode 1: fp32 FMA tiles on the
 * CUDA cores.  bf16-weight contexts always use the tensor cores.  Both modes
 * replace the fp32 MPS GEMMs of the reference's prefill (gpt.cpp:88-125). */
int itts_gpt_set_prefill_mode(itts_gpt_ctx* ctx, int mode);
uint64_t itts_gpt_launch_count(const itts_gpt_ctx* ctx);

/* Device time of the last itts_gpt_generate / itts_gpt_generate_batch call,
 * from CUDA events on the context's stream: the prefill(s), then the token
 * loop (for beam search including the host's candidate choice between
 * steps).  forward_steps counts decode forward steps (batched steps count
 * once for all their rows); rows is the largest number of rows per step.
 * No counterpart in the reference (its timing is per command buffer). */
typedef struct itts_gpt_timing {
    float prefill_ms;
    float decode_ms;
    uint32_t forward_steps;
    uint32_t rows;
} itts_gpt_timing;
int itts_gpt_last_timing(const itts_gpt_ctx* ctx, itts_gpt_timing* out);

/* ---- failure detection -------------------------------------------------------
 * Every device-side wait of the decode kernels (weight-ring slots, hand-off
 * polls, arrival counters, the grid barrier) gives up after a time limit and
 * records a status that the next host check turns into ITTS_ERR_DEVICE_TIMEOUT
 * (the reference throws std::runtime_error on a failed command buffer,
 * metal_context.mm:4624-4626).  itts_gpt_set_wait_limit sets that limit for
 * later decode launches of the context (0: the default of 2 s).
 * itts_gpt_wait_probe runs one decode phase that waits for a hand-off no phase
 * publishes, so it ends at the limit and returns ITTS_ERR_DEVICE_TIMEOUT; the
 * context stays usable.  No counterpart in the reference. */
int itts_gpt_set_wait_limit(itts_gpt_ctx* ctx, uint64_t ns);
int itts_gpt_wait_probe(itts_gpt_ctx* ctx);

/* ---- allocation-free processors --------------------------------------------
 * No counterpart in the reference.  The logits processors of
 * itts_gpt_apply_processors for callers that cannot allocate device memory:
 * a latency-critical serving thread (cudaMalloc/cudaFree can synchronise the
 * whole device) or a process whose device memory is fully reserved by another
 * allocator.  It needs no context and calls no cudaMalloc/cudaFree: inputs and
 * outputs are host arrays staged through one static device array of 133,136
 * bytes that every GPU loading this library holds until exit.  The call is
 * synchronous (blocking copies in, one kernel, blocking copies out).
 * history_n is limited to 16384 tokens (larger values return
 * ITTS_ERR_INVALID_ARGUMENT).  The first call on a device looks up that
 * array's address; make it before any stream capture.  All calls share the
 * array: calls that overlap on one GPU (from two host threads) race, so
 * serialise them.  Errors are reported by itts_gpt_last_error(NULL) on the
 * calling thread. */
int itts_gpt_apply_processors_noalloc(int device, const float* logits, size_t n, const uint32_t* history,
                                      size_t history_n, const itts_gen_opts* opts, float* out);

#ifdef __cplusplus
}
#endif

#endif /* ITTS_GPT_H */
