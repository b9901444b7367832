// accerl_sample_logits_noalloc: the token sampler for callers that cannot allocate device memory.
//
// This entry point has no counterpart in the reference, which samples inside its inference engine.
// It is the sampler of sampler.cu (per-chunk partial sums, then an inverse-CDF draw per bf16 logits
// row; log-probability of the sampled token under the untempered distribution; -inf logits allowed),
// but it takes no workspace argument and allocates nothing: its per-call scratch is the file-scope
// device array below. The prototype and return codes are declared in accerl_noalloc.h.
//
// Who needs it: a host runtime that links this library directly and calls the sampler from its
// decode loop without a device allocator at hand. Typical cases are serving runtimes that reserve
// all free device memory for the KV cache at start-up (a later cudaMalloc fails or eats into that
// reservation) and loops that must not pay cudaMalloc/cudaFree in steady state (cudaFree
// synchronises the device). Everything else should use accerl_sample_logits with a caller-owned
// workspace, which has no row limit.
//
// Contract:
//  * rows <= 1024 per call. The scratch holds 1024 rows x 16 vocabulary chunks x 4 floats
//    (256 KiB per device, in the module's static device memory). Larger calls are rejected with
//    ACCERL_NOALLOC_TOO_MANY_ROWS (-30) before anything is launched; split them into batches.
//  * V and ld must be multiples of 8 and logits 16-byte aligned (ACCERL_NOALLOC_BAD_SHAPE, -1,
//    otherwise), as for accerl_sample_logits. No top-k / top-p: those rows need accerl_sample_logits.
//  * The device index must be below 64 (ACCERL_NOALLOC_BAD_DEVICE, -31, otherwise): the per-device
//    address cache has 64 entries.
//  * The scratch is shared by every call on a device. Calls that may overlap in time (different
//    streams without an ordering event between them, or different host threads) race on it: issue
//    them on one stream, or order them. Its contents persist from call to call; nothing in it has
//    to start at zero, because each call writes every scratch slot it reads before reading it.
//  * Set-up happens on the first call on each device: the scratch address is looked up with
//    cudaGetSymbolAddress once per device and cached (an error there is returned as its
//    cudaError_t code). If the caller captures streams, make the first call on each device before
//    any capture begins.
//  * Returns 0 on success, a cudaError_t code (> 0) from the lookup or the launch, or a negative
//    code above. On a negative code nothing was launched.
#include <atomic>

#include "accerl_noalloc.h"
#include "sampler.cuh"

namespace {
constexpr int kNoAllocMaxRows = ACCERL_NOALLOC_MAX_ROWS;
constexpr int kNoAllocChunks = 16;
constexpr int kMaxDevices = 64;

// [row][chunk][max, sumexp, tempered sumexp, argmax index]
static __device__ __align__(256) float g_sampler_scratch[kNoAllocMaxRows * kNoAllocChunks * accerl::kSamplePartFloats];

std::atomic<float*> g_scratch_addr[kMaxDevices];
}  // namespace

extern "C" int accerl_sample_logits_noalloc(const void* logits, long long ld, int rows, int V, const float* temperature,
                                            const unsigned long long* seeds, const long long* offsets,
                                            long long* out_tokens, float* out_logprobs, cudaStream_t s) {
  using namespace accerl;
  if (rows == 0) return 0;
  if (rows < 0 || rows > kNoAllocMaxRows) return ACCERL_NOALLOC_TOO_MANY_ROWS;
  if (V <= 0 || V % 8 || ld % 8 || (reinterpret_cast<uintptr_t>(logits) & 15)) return ACCERL_NOALLOC_BAD_SHAPE;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return ACCERL_NOALLOC_BAD_DEVICE;
  float* scratch = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sampler_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    scratch = static_cast<float*>(p);
    g_scratch_addr[dev].store(scratch, std::memory_order_release);  // same value from every racing thread
  }
  const auto* lg = static_cast<const __nv_bfloat16*>(logits);
  sample_partial_kernel<<<dim3(rows, kNoAllocChunks), 256, 0, s>>>(lg, ld, V, temperature, nullptr, nullptr, scratch,
                                                                   kNoAllocChunks);
  sample_final_kernel<<<rows, 256, 0, s>>>(lg, ld, V, temperature, nullptr, nullptr, seeds, offsets, scratch,
                                           kNoAllocChunks, out_tokens, out_logprobs);
  return static_cast<int>(cudaGetLastError());
}
