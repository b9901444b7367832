// Public C declaration of the allocation-free sampler entry point (implemented in sample_noalloc.cu).
// Include this header from a host runtime that links the extension library directly.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest number of logits rows that one call accepts (the static scratch holds this many rows).
#define ACCERL_NOALLOC_MAX_ROWS 1024
// Return codes besides 0 (success) and positive cudaError_t values:
#define ACCERL_NOALLOC_BAD_SHAPE (-1)          // V or ld not a multiple of 8, or logits not 16-byte aligned
#define ACCERL_NOALLOC_TOO_MANY_ROWS (-30)     // rows < 0 or rows > ACCERL_NOALLOC_MAX_ROWS; nothing launched
#define ACCERL_NOALLOC_BAD_DEVICE (-31)        // current device index >= 64; nothing launched

// Samples one token per row of bf16 logits [rows, V] (row stride ld elements) at temperature[row]
// (<= 0: argmax) and writes the token and its log-probability under the untempered softmax. The
// random stream of a row is keyed by (seeds[row], offsets[row]). All pointers are device pointers;
// the launch goes to stream s. Allocates no memory: see sample_noalloc.cu for the scratch contract.
int accerl_sample_logits_noalloc(const void* logits, long long ld, int rows, int V, const float* temperature,
                                 const unsigned long long* seeds, const long long* offsets, long long* out_tokens,
                                 float* out_logprobs, cudaStream_t s);

#ifdef __cplusplus
}
#endif
