// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (UMMA) descriptors / MMA / TMEM management, and small numeric utilities.
//
// Every wait that depends on another agent (TMA completion, MMA completion, another warp) is a
// bounded spin against %globaltimer. When the deadline passes, the waiting thread records an error
// code in the caller-provided status word and gives up instead of hanging the GPU; kernels then
// drain to their common tear-down path (TMEM is always freed) and the host raises on the status.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#define ACCERL_DEVINL __device__ __forceinline__

namespace accerl {

// ----------------------------------------------------------------------------------------------
// per-device host-side set-up
// ----------------------------------------------------------------------------------------------
// Function attributes (the dynamic shared-memory opt-in) and occupancy answers belong to a device, so
// a process that drives several GPUs sets them once per device. The flags are atomics: two host
// threads that race both set the attribute, which is harmless.
constexpr int kMaxHostDevices = 64;

inline int host_current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

// Opt kernel `Kern` into `bytes` of dynamic shared memory on the current device (once per device).
template <auto Kern>
inline cudaError_t smem_attr_once(int bytes) {
  static std::atomic<unsigned long long> done{0};  // bit d: set on device d
  const int dev = host_current_device();
  const unsigned long long bit = (dev >= 0 && dev < kMaxHostDevices) ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return cudaSuccess;
  const cudaError_t e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && bit) done.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// Number of SMs of the current device (cached per device).
inline int device_sm_count() {
  static std::atomic<int> cache[kMaxHostDevices];
  const int dev = host_current_device();
  if (dev >= 0 && dev < kMaxHostDevices) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev < 0 ? 0 : dev) != cudaSuccess || n <= 0) n = 148;
  if (dev >= 0 && dev < kMaxHostDevices) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// Status codes written to the status word (first writer wins).
enum StatusCode : int {
  kStatusOk = 0,
  kStatusTimeoutProducer = 1,
  kStatusTimeoutMma = 2,
  kStatusTimeoutEpilogue = 3,
  kStatusTimeoutPeer = 4,
  kStatusBadArgument = 5,
};

// ----------------------------------------------------------------------------------------------
// debug-checks build
// ----------------------------------------------------------------------------------------------
// Built with -DACCERL_DEBUG_CHECKS (``ACCERL_DEBUG_CHECKS=1 python setup.py build_ext --inplace``),
// every data-dependent index (token ids, KV-cache slots, page ids, MoE row positions) is range-checked
// before it is used. A failing check records (check code, offending index) in its translation unit's
// debug record, first failure wins, and the access is skipped, so the kernel still returns and the
// host reads the record with accerl_debug_status_<unit>() (``ops.debug_status()``). The checks never
// trap. Release builds compile them away (``ACCERL_DBG_OK`` is the constant true).
enum DebugCheck : int {
  kDbgEmbeddingId = 1,
  kDbgKvSlot = 2,
  kDbgPageId = 3,
  kDbgMoeRow = 4,
};

#ifdef ACCERL_DEBUG_CHECKS
static __device__ unsigned long long g_debug_record[2];
ACCERL_DEVINL bool debug_fail(int code, long long index) {
  if (atomicCAS(&g_debug_record[0], 0ull, static_cast<unsigned long long>(code)) == 0ull)
    g_debug_record[1] = static_cast<unsigned long long>(index);
  return false;
}
#define ACCERL_DBG_OK(cond, code, index) ((cond) ? true : ::accerl::debug_fail((code), (index)))
// Host reader of this translation unit's record: out = {code, index}; returns 1 in a debug build.
#define ACCERL_DEBUG_EXPORT(unit)                                                                    \
  extern "C" int accerl_debug_status_##unit(long long* out, int reset) {                             \
    unsigned long long r[2] = {0, 0};                                                                \
    if (cudaMemcpyFromSymbol(r, ::accerl::g_debug_record, sizeof(r)) != cudaSuccess) return -1;      \
    out[0] = static_cast<long long>(r[0]);                                                           \
    out[1] = static_cast<long long>(r[1]);                                                           \
    if (reset) {                                                                                     \
      const unsigned long long z[2] = {0, 0};                                                        \
      if (cudaMemcpyToSymbol(::accerl::g_debug_record, z, sizeof(z)) != cudaSuccess) return -1;      \
    }                                                                                                \
    return 1;                                                                                        \
  }
#else
#define ACCERL_DBG_OK(cond, code, index) true
#define ACCERL_DEBUG_EXPORT(unit)                                        \
  extern "C" int accerl_debug_status_##unit(long long* out, int reset) { \
    (void)reset;                                                         \
    out[0] = 0;                                                          \
    out[1] = 0;                                                          \
    return 0;                                                            \
  }
#endif

// Default deadline for a single barrier wait: 2 seconds of GPU time.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

ACCERL_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

ACCERL_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

ACCERL_DEVINL uint32_t lane_id() { return threadIdx.x & 31u; }

ACCERL_DEVINL bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n"
      ".reg .b32 %%rx;\n"
      ".reg .pred %%px;\n"
      "elect.sync %%rx|%%px, %1;\n"
      "@%%px mov.s32 %0, 1;\n"
      "}\n"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ----------------------------------------------------------------------------------------------
// mbarrier
// ----------------------------------------------------------------------------------------------
ACCERL_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

ACCERL_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

ACCERL_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

ACCERL_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

ACCERL_DEVINL bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false (and records
// `code` in *status) when the deadline passes or another thread already flagged an error.
ACCERL_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                             uint64_t timeout_ns = kWaitTimeoutNs) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t iter = 0;
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((++iter & 255u) == 0) {
      if (globaltimer_ns() - start > timeout_ns) {
        if (status) atomicCAS(status, 0, code);
        return false;
      }
      if (status && *(volatile int*)status != 0) return false;
    }
  }
}

// ----------------------------------------------------------------------------------------------
// TMA (no cluster multicast anywhere in this code base)
// ----------------------------------------------------------------------------------------------
ACCERL_DEVINL void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

ACCERL_DEVINL void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

ACCERL_DEVINL void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------------------------
// tcgen05 / TMEM
// ----------------------------------------------------------------------------------------------
// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile (sm_100 format: start
// address bits 0-13, leading byte offset 16-29, stride byte offset 32-45, version=1 at bit 46,
// layout type SWIZZLE_128B=2 at bits 61-63; all offsets in 16-byte units).
//  * K-major tiles: rows of 64 bf16 (128 B), 8-row groups 1024 B apart -> LBO=16 B (unused), SBO=1024 B.
//  * MN-major tiles: 64-element MN chunks holding all K rows (128 B each) -> LBO = chunk stride,
//    SBO = 1024 B between groups of 8 K rows.
ACCERL_DEVINL uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 inputs and an fp32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
         | (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);     // M / 16
}

ACCERL_DEVINL void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D (+)= A * B with A read from tensor memory (M rows = TMEM lanes, K packed two bf16 per 32-bit
// column, so a K step of 16 advances 8 columns) and B from shared memory.
ACCERL_DEVINL void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Signal `bar` once every previously issued tcgen05.mma of this thread has completed.
ACCERL_DEVINL void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

ACCERL_DEVINL void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

ACCERL_DEVINL void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- TMA stores (shared -> global), bulk-group completion ------------------------------------
ACCERL_DEVINL void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// element-wise add of the shared tile into global memory (performed at L2)
ACCERL_DEVINL void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int32_t x, int32_t y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
ACCERL_DEVINL void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
ACCERL_DEVINL void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
ACCERL_DEVINL void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// byte offset of 16-byte chunk j of row r in a 128-byte-row tile with the TMA 128B swizzle
ACCERL_DEVINL uint32_t swz128(uint32_t r, uint32_t j) { return r * 128u + (((j ^ (r & 7u)) & 7u) << 4); }
// the same for 64-byte rows and the 64B swizzle (address bits [4,5] ^= bits [7,8])
ACCERL_DEVINL uint32_t swz64(uint32_t r, uint32_t j) { return r * 64u + (((j ^ (r >> 1)) & 3u) << 4); }

// ---- CTA pairs (cluster of 2, tcgen05 cta_group::2) ------------------------------------------
// The two CTAs of a cluster share one MMA: the even CTA (rank 0) issues tcgen05.mma.cta_group::2,
// which reads A (M/2 rows) and B (N/2 rows) from the same shared-memory offsets in both CTAs and
// writes each CTA's M/2 x N accumulator into that CTA's TMEM.
ACCERL_DEVINL uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

ACCERL_DEVINL void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// shared::cluster address of the same shared variable in CTA `rank` of this cluster
ACCERL_DEVINL uint32_t map_shared_rank(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}

ACCERL_DEVINL void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA 2-D load into this CTA's shared memory whose completion is signalled on an mbarrier that may
// live in the peer CTA of the pair (`bar_cluster` is a shared::cluster address). Not a multicast load.
ACCERL_DEVINL void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

ACCERL_DEVINL void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n"
      "}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at this shared offset in every CTA of `mask` once the pair's prior MMAs finish.
ACCERL_DEVINL void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// Collective over the pair: one warp (the same warp index) in each CTA; both give the same smem slot.
ACCERL_DEVINL void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

ACCERL_DEVINL void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

ACCERL_DEVINL void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ACCERL_DEVINL void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Load 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane i -> row i of the warp slice).
ACCERL_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Load 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
ACCERL_DEVINL void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Store 32 consecutive fp32 columns of this warp's 32 TMEM lanes.
ACCERL_DEVINL void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Store 16 consecutive 32-bit columns of this warp's 32 TMEM lanes.
ACCERL_DEVINL void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

ACCERL_DEVINL void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
ACCERL_DEVINL void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Fire-and-forget vector reduction into global fp32 memory (no return value, so the issuing warp does
// not wait for the round trip the way a value-returning atomic does).
ACCERL_DEVINL void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// System-scope release store / acquire load of a 32-bit flag (cross-GPU signalling over NVLink).
ACCERL_DEVINL void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
ACCERL_DEVINL int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// 16-byte load cached in L2 only (no L1): peer data that changes between kernel launches.
ACCERL_DEVINL uint4 ld_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Make generic-proxy shared-memory writes visible to the async proxy (tcgen05.mma operand reads).
ACCERL_DEVINL void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Named barrier among a subset of warps (id 1..15; id 0 is __syncthreads).
ACCERL_DEVINL void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ANDs a predicate over its threads: every participant gets the same answer,
// so a bounded wait that ran out in any thread turns the whole group back together.
ACCERL_DEVINL bool named_bar_and(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n"
      ".reg .pred pin, pout;\n"
      "setp.ne.u32 pin, %1, 0;\n"
      "bar.red.and.pred pout, %2, %3, pin;\n"
      "selp.u32 %0, 1, 0, pout;\n"
      "}\n"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return out != 0;
}

// ----------------------------------------------------------------------------------------------
// numeric helpers
// ----------------------------------------------------------------------------------------------
ACCERL_DEVINL uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

ACCERL_DEVINL float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// SwiGLU on bf16 inputs g (gate) and u (up): h = bf16(silu(g)) * u, and its gradients for an output
// gradient d (all three already rounded to bf16). Shared by the elementwise kernels and the GEMM
// epilogues that fuse them, so fused and unfused paths give identical bits.
ACCERL_DEVINL float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }
ACCERL_DEVINL float swiglu_h(float g, float u) { return bf16_round(g / (1.f + __expf(-g))) * u; }
ACCERL_DEVINL void swiglu_grads(float g, float u, float d, float& dg, float& du) {
  const float sig = 1.f / (1.f + __expf(-g));
  const float act = bf16_round(g * sig);
  const float dact = sig * (1.f + g * (1.f - sig));
  dg = d * u * dact;
  du = d * act;
}

// Rotary embedding coefficients of frequency i (0 <= i < D/2) at position p: inv_freq = theta^(-2i/D),
// angle in fp32, cos / sin rounded to bf16 (as the reference module does). Shared by the RoPE kernel
// and the attention backward's fused inverse rotation, so both give identical bits.
ACCERL_DEVINL void rope_cos_sin(float p, int i, int D, float log2_theta, float& c, float& s) {
  const float inv_freq = exp2f(-log2_theta * (2.0f * i) / static_cast<float>(D));
  float sn, cn;
  sincosf(p * inv_freq, &sn, &cn);
  c = __bfloat162float(__float2bfloat16(cn));
  s = __bfloat162float(__float2bfloat16(sn));
}

ACCERL_DEVINL float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

ACCERL_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace accerl
