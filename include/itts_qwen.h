/* C-ABI of the B200 Qwen3-0.6B decoder (the emotion-text model of IndexTTS 2.5).
 *
 * Replaces itts25::QwenDecoder (include/itts25/qwen.hpp:6-19, src/qwen.cpp):
 *   itts_qwen_create   <- QwenDecoder(Weights&) (qwen.cpp:5-14: shape checks)
 *   itts_qwen_prefill  <- QwenDecoder::prefill (qwen.cpp:19-22)
 *   itts_qwen_step     <- QwenDecoder::step (qwen.cpp:23)
 *   itts_qwen_generate <- QwenDecoder::generate (qwen.cpp:44-50)
 * Errors use the status codes of itts_gpt.h with the reference's messages:
 * std::invalid_argument -> ITTS_ERR_INVALID_ARGUMENT, std::runtime_error ->
 * ITTS_ERR_RUNTIME.  One context is not thread-safe. */
#ifndef ITTS_QWEN_H
#define ITTS_QWEN_H

#include <stddef.h>
#include <stdint.h>

#include "itts_gpt.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ITTS_QWEN_VOCAB 151936     /* embed_tokens rows; the head is tied (qwen.cpp:7, :40) */
#define ITTS_QWEN_EOS 151643       /* generation ends here (qwen.cpp:48) */
#define ITTS_QWEN_MAX_PROMPT 3072  /* qwen.cpp:20, :47 */
#define ITTS_QWEN_CAPACITY 4096    /* KV capacity (qwen.cpp:21 gptKvCacheCreate(28, 4096, 1024)) */
#define ITTS_QWEN_MAX_GENERATE 1024

typedef struct itts_qwen_ctx itts_qwen_ctx;

/* Loads the 28-layer decoder from an MIT2 bundle (target index-tts2.5) onto
 * `device`.  Failure: "Unsupported Qwen shape: <name>" (invalid argument), or
 * the bundle's own errors. */
int itts_qwen_create(const char* bundle_dir, int device, itts_qwen_ctx** out);
void itts_qwen_destroy(itts_qwen_ctx* ctx);
/* Message of the last failure of ctx (or of the last create when ctx is NULL). */
const char* itts_qwen_last_error(const itts_qwen_ctx* ctx);

/* Runs the prompt `ids` (1..3072 ids < 151936) from an empty cache; `logits`
 * (151936 floats, may be NULL) receives the last position's logits.
 * "Qwen prompt capacity is 3072 tokens", "Invalid Qwen token". */
int itts_qwen_prefill(itts_qwen_ctx* ctx, const uint32_t* ids, size_t n, float* logits);
/* One token at the next position after a prefill.  "Qwen cache capacity
 * exceeded" without a prefill or at 4096 cached tokens; "Invalid Qwen token". */
int itts_qwen_step(itts_qwen_ctx* ctx, uint32_t id, float* logits);
/* Greedy ids after the prompt, up to and including EOS (at most `maximum`,
 * 1..1024, with n + maximum <= 4096): "Qwen generation capacity exceeded",
 * then the prompt checks; a run that selects `maximum` ids without EOS fails
 * with "Qwen did not reach EOS within 1024 generated tokens" (runtime). The
 * ids go to out[0 .. *n_out) (out_cap >= maximum). */
int itts_qwen_generate(itts_qwen_ctx* ctx, const uint32_t* ids, size_t n, uint32_t maximum, uint32_t* out,
                       size_t out_cap, uint32_t* n_out);
uint32_t itts_qwen_cached_tokens(const itts_qwen_ctx* ctx);

/* Device time of the last prefill / generate call (CUDA events on the
 * context's stream): the prompt pass, then the token steps. */
typedef struct itts_qwen_timing {
    float prefill_ms;
    float decode_ms;
    uint32_t steps;  /* decode steps run (one CUDA graph per step) */
    uint32_t prompt; /* prompt tokens */
} itts_qwen_timing;
int itts_qwen_last_timing(const itts_qwen_ctx* ctx, itts_qwen_timing* out);

#ifdef __cplusplus
}
#endif

#endif /* ITTS_QWEN_H */
