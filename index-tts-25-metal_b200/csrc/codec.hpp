// Device-side description of the IndexTTS 2.5 semantic codec's decoder
// (weights in device memory, scratch buffers) shared by codec.cu and the host
// runtime itts_codec.cpp.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace itts {

struct CodecBlockW {  // codec.decoder.0.convnext.i
    const float *dw_w, *dw_b;    // depthwise conv [384, 1, 7]
    const float *ln_g, *ln_b;    // LayerNorm 384, eps 1e-6
    const float *pw1_w, *pw1_b;  // [2048, 384]
    const float *pw2_w, *pw2_b;  // [384, 2048]
    const float* gamma;          // [384] layer scale
};

struct CodecWeights {
    const float* codebook;        // [8192, 8]
    const float *out_w, *out_b;   // quantizer out_project [1024, 8]
    const float *embed_w, *embed_b;  // decoder embed conv [384, 1024, 7]
    const float *norm_g, *norm_b;
    CodecBlockW block[12];
    const float *final_g, *final_b;
    const float *head_w, *head_b;  // codec.decoder.1 [1024, 384]
    const float *up_w, *up_b;      // codec.up [1024, 1024, 3]
};

struct CodecScratch {  // sized for the largest T decoded so far
    float* hidden;  // [T, 1024]
    float* h;       // [T, 384]
    float* x;       // [T, 384]
    float* u;       // [T, 2048]
};

cudaError_t codec_decode_device(const CodecWeights& w, const CodecScratch& sc, const uint32_t* d_codes, int T,
                                float* out, cudaStream_t s);

}  // namespace itts
