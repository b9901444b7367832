// Token sampler kernels shared by sampler.cu (workspace entry point) and sample_noalloc.cu (static-scratch
// entry point). Both entry points launch the same two kernels; only the scratch memory differs.
#pragma once

#include "common.cuh"

namespace accerl {

// Floats per (row, chunk) partial: {chunk max, sum exp(x - max), sum exp((x - max) / T), argmax index}.
constexpr int kSamplePartFloats = 4;

// grid (rows, num_chunks), 256 threads. Rows that the filtered kernel owns (top_k / top_p active) are
// skipped; top_k and top_p may be null.
__global__ void sample_partial_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int V,
                                      const float* __restrict__ temperature, const int* __restrict__ top_k,
                                      const float* __restrict__ top_p, float* __restrict__ part, int num_chunks);

// grid (rows), 256 threads: merges a row's chunk partials, draws the token and writes its log-probability.
__global__ void sample_final_kernel(const __nv_bfloat16* __restrict__ logits, long long ld, int V,
                                    const float* __restrict__ temperature, const int* __restrict__ top_k,
                                    const float* __restrict__ top_p, const unsigned long long* __restrict__ seeds,
                                    const long long* __restrict__ offsets, const float* __restrict__ part,
                                    int num_chunks, long long* __restrict__ out_tokens,
                                    float* __restrict__ out_logprobs);

}  // namespace accerl
