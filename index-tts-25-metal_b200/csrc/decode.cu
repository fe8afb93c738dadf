// The decode kernels with fp32 weight matrices (see decode_body.cuh).
#define ITTS_WNS wf32
#define ITTS_WBF16 0
#include "decode_body.cuh"
#include "decode_batch.cuh"
