/*
 * itts_codec.h — C-ABI of the B200 (sm_100a) semantic-codec decoder of
 * IndexTTS 2.5: the stage that turns the GPT's semantic codes into 1024-d
 * features at twice the code rate.  It replaces the decode half of the
 * reference's itts25::EnhancedCodec (include/itts25/codec.hpp, src/codec.cpp).
 * Conventions as in itts_gpt.h: status codes (ITTS_OK = 0, the same negative
 * classes), the message of the last failure from itts_codec_last_error.
 */
#ifndef ITTS_CODEC_H
#define ITTS_CODEC_H

#include <stddef.h>
#include <stdint.h>

#include "itts_gpt.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ITTS_CODEC_WIDTH 1024      /* feature width */
#define ITTS_CODEC_MAX_CODES 5000  /* codec.cpp:51 */

typedef struct itts_codec_ctx itts_codec_ctx;

/* EnhancedCodec::EnhancedCodec (codec.cpp:6-22): loads the codec tensors of an
 * MIT2 bundle (target "index-tts2.5"), checks the reference's shapes
 * (ITTS_ERR_RUNTIME "Unsupported 2.5 codec shape: ..." otherwise) and uploads
 * the decoder to `device`.  Errors of a failed create: itts_codec_last_error(NULL). */
int itts_codec_create(const char* bundle_dir, int device, itts_codec_ctx** out);
void itts_codec_destroy(itts_codec_ctx* ctx);
const char* itts_codec_last_error(const itts_codec_ctx* ctx);

/* EnhancedCodec::decode (codec.cpp:50-69): n codes (1 <= n <= 5000, each
 * < 8192; ITTS_ERR_INVALID_ARGUMENT otherwise) -> out[2n][1024] fp32
 * (out_floats >= 2n * 1024).  Synchronous.  ITTS_ERR_DEVICE_TIMEOUT when a
 * bounded wait of a tensor-core GEMM gave up (the context stays usable). */
int itts_codec_decode(itts_codec_ctx* ctx, const uint32_t* codes, size_t n, float* out, size_t out_floats);

/* GEMMs of the decode: 0 (default) the TMA-fed tcgen05 GEMM on TF32 hi / lo
 * operands (three products, fp32 accuracy), 1 the fp32 CUDA-core tiles (kept
 * for comparison).  No counterpart in the reference. */
int itts_codec_set_gemm_mode(itts_codec_ctx* ctx, int mode);

/* Device time of the last successful itts_codec_decode: CUDA events on the
 * context's stream around the decoder's kernels (the code upload and the
 * feature read excluded), the codes it decoded and the kernels it launched.
 * No counterpart in the reference (measurement only). */
typedef struct itts_codec_timing {
    float decode_ms;
    uint32_t codes;
    uint32_t launches;
} itts_codec_timing;
int itts_codec_last_timing(const itts_codec_ctx* ctx, itts_codec_timing* out);

#ifdef __cplusplus
}
#endif

#endif /* ITTS_CODEC_H */
