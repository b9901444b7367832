// Persistent warp-specialised bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M,N] = alpha * sum_k A(m,k) * B(n,k)  (+ beta * C_old) (+ bias[n]) (+ residual[m,n])
//
// Operand storage is flexible so the three GEMMs of a linear layer run without transposes:
//   A(m,k): K-major  -> A[m*lda + k]   ([M,K] row-major)      MN-major -> A[k*lda + m] ([K,M])
//   B(n,k): K-major  -> B[n*ldb + k]   ([N,K], weight layout) MN-major -> B[k*ldb + n] ([K,N])
//   forward  Y = X W^T : A=X (K-major),  B=W (K-major)
//   dgrad   dX = dY W  : A=dY (K-major), B=W (MN-major)
//   wgrad   dW = dY^T X: A=dY (MN-major), B=X (MN-major)
//
// Structure (one CTA per SM, 6 warps):
//   warp 0    : TMA producer. 128B-swizzled tiles of A and B land in a STAGES-deep smem ring;
//               each stage completes an mbarrier by transaction bytes.
//   warp 1    : allocates TMEM and issues tcgen05.mma (M=128, N=BN, K=16) from one elected lane;
//               tcgen05.commit frees smem stages and publishes finished accumulators.
//   warps 2-5 : epilogue. tcgen05.ld the fp32 accumulator (one TMEM lane = one output row per
//               thread), apply alpha/beta/bias/residual, convert and store.
// Accumulators are double-buffered in TMEM (2 x BN columns) so the epilogue of tile i overlaps the
// main loop of tile i+1. Tiles are visited in grouped-M order for L2 reuse of B.
// Dense GEMMs can also run as CTA pairs (clusters of 2, tcgen05.mma.cta_group::2, 256 x 256 tiles):
// each SM then stages half of B, which lifts the shared-memory-bound single-CTA tile by 8-29 %.
// No cluster multicast is used: every CTA loads its own tiles.
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"

namespace accerl {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
// Relative cost per k-block of a 256 x 256 CTA-pair work item against a 128 x 256 single-CTA one run
// by each of the pair's SMs: measured 1.08-1.29x the single-CTA throughput on the 1.5B-shape GEMMs.
constexpr double kPairCost = 0.88;
constexpr bool kPairAuto = true;

struct GemmParams {
  int M, N, K;
  void* C;
  long long ldc;
  int c_f32;
  float alpha, beta;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  long long ldr;
  int* status;
  int tiles_m, tiles_n, num_tiles, group_m;
  int splits, kb_per_split;  // split-K: work item = (tile, split); splits > 1 adds fp32 partials atomically
  // grouped (mixture-of-experts) problems; expert row segments are padded to multiples of 128 rows
  //  mode 1: A rows are grouped by expert; tile_expert[m_blk] names the expert whose B slice is used
  //          (K-major B: rows e*b_group_stride.., MN-major B: reduction rows e*b_group_stride..);
  //          a negative entry marks a tile past the last segment, which is skipped
  //  mode 2: per-expert weight gradient; work item = (expert, m_blk, n_blk), reduction over the expert's
  //          rows [group_row_start[e], +group_rows[e]), output rows offset by e*c_group_stride
  int group_mode;
  const int* tile_expert;
  const int* group_row_start;
  const int* group_rows;
  int b_group_stride;
  long long c_group_stride;
  int num_groups;
  // scatter epilogue: bf16 output row r is stored at address row_dst[r] (0 = drop the row); used to
  // write expert outputs straight into the source rank's buffer over NVLink
  const long long* row_dst;
  // SwiGLU forward epilogue (glu_I > 0, K-major B = [gate; up] of 2*glu_I rows, BN = 256): work item n
  // multiplies gate rows [n*128, +128) and up rows [glu_I + n*128, +128); the epilogue stores
  // h = silu(g) * u into glu_out (and g, u into C when C is set, for the backward)
  int glu_I;
  __nv_bfloat16* glu_out;
  long long ld_glu;
  // SwiGLU backward epilogue (dglu_gu set): the accumulator is d(h) for columns [0, N) of the SwiGLU;
  // the epilogue reads g, u from dglu_gu (row stride ld_dglu, up at +N) and stores d(gate) at column
  // c and d(up) at column N + c of C
  const __nv_bfloat16* dglu_gu;
  long long ld_dglu;
  // epilogue output path: 0 = per-thread stores, 1 = TMA tile stores of C (bf16 or fp32, beta = 0),
  // 2 = TMA reduce-add of fp32 tiles into C (beta = 1, split-K partials)
  int tma_store;
  // rotary embedding in the bf16 TMA-store epilogue: output columns [0, rope_cols) form heads of 128
  // that are rotated (rotate-half) at position rope_pos[row], inv_freq = theta^(-2i/128)
  const long long* rope_pos;
  int rope_cols;
  float rope_log2_theta;
};

// Epilogue staging: per epilogue warp two 32-row x 128-byte tiles (64 bf16 or 32 fp32 columns),
// written with the 128B swizzle and drained by TMA stores while the next chunk is converted.
constexpr int kEpiChunkBytes = 32 * 128;
constexpr int kEpiBytes = 4 * 2 * kEpiChunkBytes;

struct WorkItem {
  int m_blk, n_blk, kb0, kb1, b_n_off, b_k_off;
  long long c_row_off;
};

// Per-CTA shared-memory stage. A CTA pair (PAIR) splits B's BN rows: each CTA stages BN/2 of them.
template <int BN, bool PAIR = false>
struct GemmSmem {
  static constexpr int kBRows = PAIR ? BN / 2 : BN;
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kBRows * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
};

__device__ __forceinline__ void tile_coords(const GemmParams& p, int t, int& m_blk, int& n_blk) {
  t /= p.splits;
  const int per_group = p.group_m * p.tiles_n;
  const int group = t / per_group;
  const int first_m = group * p.group_m;
  const int gsize = min(p.tiles_m - first_m, p.group_m);
  const int r = t % per_group;
  m_blk = first_m + r % gsize;
  n_blk = r / gsize;
}

template <bool B_MN>
__device__ __forceinline__ WorkItem work_item(const GemmParams& p, int t, int k_blocks) {
  WorkItem w;
  w.b_n_off = 0;
  w.b_k_off = 0;
  w.c_row_off = 0;
  if (p.group_mode == 2) {
    const int per_e = p.tiles_m * p.tiles_n;
    const int e = t / per_e;
    const int local = t % per_e;
    w.m_blk = local % p.tiles_m;
    w.n_blk = local / p.tiles_m;
    w.kb0 = p.group_row_start[e] / kBK;
    w.kb1 = w.kb0 + p.group_rows[e] / kBK;
    w.c_row_off = static_cast<long long>(e) * p.c_group_stride;
    return w;
  }
  tile_coords(p, t, w.m_blk, w.n_blk);
  w.kb0 = (t % p.splits) * p.kb_per_split;
  w.kb1 = min(k_blocks, w.kb0 + p.kb_per_split);
  if (p.group_mode == 1) {
    const int e = p.tile_expert[w.m_blk];
    if (e < 0) {  // a tile past the last expert segment (device-side layouts bound the tile count)
      w.kb1 = w.kb0;
      return w;
    }
    if (B_MN) w.b_k_off = e * p.b_group_stride;
    else w.b_n_off = e * p.b_group_stride;
  }
  return w;
}

// PAIR: the kernel runs as clusters of 2 CTAs on the two SMs of a TPC and computes 256 x BN tiles
// with tcgen05.mma.cta_group::2 (M = 256): each CTA stages its 128 rows of A and BN/2 rows of B, so per
// SM the operand traffic per MMA FLOP halves for B. The even CTA issues the MMAs; stage-full
// barriers live in the even CTA (both CTAs' loads complete there), stage-empty and accumulator-full
// barriers are signalled in both CTAs by multicast commits, and both CTAs' epilogues release an
// accumulator on the even CTA's barrier. Loads are plain per-CTA TMA loads (no multicast).
template <int BN, int STAGES, bool A_MN, bool B_MN, bool PAIR, bool ROPE = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmH,
                      const GemmParams p) {
  using S = GemmSmem<BN, PAIR>;
  constexpr int TM = PAIR ? 2 * kBM : kBM;  // rows of C per work item
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * S::kABytes;
  uint8_t* smEpi = smem + STAGES * S::kStageBytes;  // 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smEpi + kEpiBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = 2 * BN;
  const int k_blocks = (p.K + kBK - 1) / kBK;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0 = the CTA that issues the pair's MMAs
  const int first_item = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int item_stride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 256 : 128);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if constexpr (PAIR) {
    if (warp == 1) tmem_alloc_pair(tmem_slot, kTmemCols);
  } else {
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  }
  tc_fence_before();
  if constexpr (PAIR) cluster_sync();  // barriers of both CTAs initialised before any remote signal
  else __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;
      uint32_t last_parity = 0;  // bit s = parity of the last load issued into stage s
      bool ok = true;
      for (int t = first_item; t < p.num_tiles && ok; t += item_stride) {
        const WorkItem w = work_item<B_MN>(p, t, k_blocks);
        if (w.kb1 <= w.kb0) continue;
        const int m0 = w.m_blk * TM + static_cast<int>(rank) * kBM;
        const int n0 = w.n_blk * BN + static_cast<int>(rank) * S::kBRows;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const int k0 = kb * kBK;
          uint8_t* a_dst = smA + stage * S::kABytes;
          uint8_t* b_dst = smB + stage * S::kBBytes;
          if constexpr (PAIR) {
            // both CTAs' bytes complete the even CTA's stage barrier
            const uint32_t bar = map_shared_rank(&full[stage], 0);
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * S::kStageBytes);
            if constexpr (A_MN) {
#pragma unroll
              for (int j = 0; j < kBM / 64; ++j) tma_load_2d_pair(a_dst + j * 64 * kBK * 2, &tmA, bar, m0 + 64 * j, k0);
            } else {
              tma_load_2d_pair(a_dst, &tmA, bar, k0, m0);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < S::kBRows / 64; ++j)
                tma_load_2d_pair(b_dst + j * 64 * kBK * 2, &tmB, bar, n0 + 64 * j, k0 + w.b_k_off);
            } else if (p.glu_I) {
              // the even CTA stages the gate block, the odd CTA the matching up block
              tma_load_2d_pair(b_dst, &tmB, bar, k0, (rank ? p.glu_I : 0) + w.n_blk * 128);
            } else {
              tma_load_2d_pair(b_dst, &tmB, bar, k0, n0 + w.b_n_off);
            }
          } else {
            mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
            if constexpr (A_MN) {
#pragma unroll
              for (int j = 0; j < kBM / 64; ++j)
                tma_load_2d(a_dst + j * 64 * kBK * 2, &tmA, &full[stage], m0 + 64 * j, k0);
            } else {
              tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                tma_load_2d(b_dst + j * 64 * kBK * 2, &tmB, &full[stage], n0 + 64 * j, k0 + w.b_k_off);
            } else if (p.glu_I) {
              tma_load_2d(b_dst, &tmB, &full[stage], k0, w.n_blk * 128);
              tma_load_2d(b_dst + 128 * kBK * 2, &tmB, &full[stage], k0, p.glu_I + w.n_blk * 128);
            } else {
              tma_load_2d(b_dst, &tmB, &full[stage], k0, n0 + w.b_n_off);
            }
          }
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (PAIR && ok) {
        // Tail: wait until the MMAs have consumed every stage this CTA filled, so no commit of the
        // even CTA arrives in this CTA's shared memory after it exits (bounded waits).
        for (int i = 0; i < STAGES; ++i) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status, kStatusTimeoutProducer)) break;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      } else if (!ok && rank == 0) {
        // Drain: never leave a bulk copy in flight into shared memory of a finished CTA (in a pair the
        // even CTA's stage barriers count both CTAs' bytes).
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s)) mbar_wait(&full[s], (last_parity >> s) & 1u, nullptr, 0, 20000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc = make_idesc_bf16_f32(TM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int t = first_item; t < p.num_tiles && ok; t += item_stride) {
        const WorkItem w = work_item<B_MN>(p, t, k_blocks);
        if (w.kb1 <= w.kb0) continue;
        const int kb0 = w.kb0, kb1 = w.kb1;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tbase + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smA + stage * S::kABytes);
          const uint32_t b_addr = smem_u32(smB + stage * S::kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            uint64_t adesc, bdesc;
            if constexpr (A_MN) adesc = make_sw128_desc(a_addr + kk * 16 * 128, 64 * kBK * 2, 1024);
            else adesc = make_sw128_desc(a_addr + kk * 32, 16, 1024);
            if constexpr (B_MN) bdesc = make_sw128_desc(b_addr + kk * 16 * 128, 64 * kBK * 2, 1024);
            else bdesc = make_sw128_desc(b_addr + kk * 32, 16, 1024);
            if constexpr (PAIR) umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb != kb0) || (kk != 0));
            else umma_bf16(d_tmem, adesc, bdesc, idesc, (kb != kb0) || (kk != 0));
          }
          if constexpr (PAIR) umma_commit_pair(&empty[stage], 0x3);
          else umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) umma_commit_pair(&tfull[acc], 0x3);
        else umma_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int local = 0;
    int epi_chunk = 0;
    const uint32_t tempty_even = PAIR ? map_shared_rank(&tempty[0], 0) : 0u;
    for (int t = first_item; t < p.num_tiles; t += item_stride) {
      const WorkItem w = work_item<B_MN>(p, t, k_blocks);
      if (w.kb1 <= w.kb0) continue;
      const int m_blk = w.m_blk, n_blk = w.n_blk;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      if (!mbar_wait(&tfull[acc], acc_phase, p.status, kStatusTimeoutEpilogue)) break;
      tc_fence_after();
      const int row_in_c = m_blk * TM + static_cast<int>(rank) * kBM + row_in_tile;
      const bool row_ok = row_in_c < p.M;
      const long long row = w.c_row_off + row_in_c;
      const uint32_t t_row = tbase + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN;
      if (p.tma_store) {
        // stage 32-row chunks in swizzled shared memory and write them with TMA (full-line, async)
        uint8_t* wbuf = smEpi + quarter * (2 * kEpiChunkBytes);
        const int chunk_cols = p.c_f32 ? 32 : 64;
        const int y0 = static_cast<int>(w.c_row_off) + m_blk * TM + static_cast<int>(rank) * kBM + quarter * 32;
        // rotary heads of this tile: both halves of a head (columns d and d + 64) in registers, rotated,
        // then written as two 64-column chunks
        int c_start = 0;
        if (ROPE && p.rope_pos && !p.c_f32) {
          const float pos = static_cast<float>(row_ok ? p.rope_pos[row] : 0);
#pragma unroll 1
          for (int hd = 0; hd < BN && n_blk * BN + hd < p.rope_cols; hd += 128) {
            uint32_t a[64], b[64];
            tmem_ld32(t_row + hd, *reinterpret_cast<uint32_t(*)[32]>(a));
            tmem_ld32(t_row + hd + 32, *reinterpret_cast<uint32_t(*)[32]>(a + 32));
            tmem_ld32(t_row + hd + 64, *reinterpret_cast<uint32_t(*)[32]>(b));
            tmem_ld32(t_row + hd + 96, *reinterpret_cast<uint32_t(*)[32]>(b + 32));
            tmem_wait_ld();
            const int colh = n_blk * BN + hd;
#pragma unroll 1
            for (int part = 0; part < 2; ++part) {
              uint8_t* buf = wbuf + (epi_chunk & 1) * kEpiChunkBytes;
              ++epi_chunk;
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                uint32_t o[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  float r2[2];
#pragma unroll
                  for (int e = 0; e < 2; ++e) {
                    const int d = 8 * j + 2 * i + e;  // frequency index 0..63
                    float x1 = __uint_as_float(a[d]) * p.alpha, x2 = __uint_as_float(b[d]) * p.alpha;
                    if (p.bias) {
                      x1 += __bfloat162float(p.bias[colh + d]);
                      x2 += __bfloat162float(p.bias[colh + 64 + d]);
                    }
                    x1 = bf16_round(x1);  // the rotation sees the bf16 projection, as the separate kernel does
                    x2 = bf16_round(x2);
                    float cs, sn;
                    rope_cos_sin(pos, d, 128, p.rope_log2_theta, cs, sn);
                    r2[e] = part == 0 ? x1 * cs - x2 * sn : x2 * cs + x1 * sn;
                  }
                  o[i] = pack_bf16x2(r2[0], r2[1]);
                }
                *reinterpret_cast<uint4*>(buf + swz128(lane, j)) = make_uint4(o[0], o[1], o[2], o[3]);
              }
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmC, buf, colh + part * 64, y0);
                bulk_commit();
              }
            }
            c_start = hd + 128;
          }
        }
#pragma unroll 1
        for (int c0 = c_start; c0 < BN; c0 += chunk_cols) {
          uint8_t* buf = wbuf + (epi_chunk & 1) * kEpiChunkBytes;
          ++epi_chunk;
          if (lane == 0) bulk_wait_read<1>();  // the store issued from this buffer two chunks ago
          __syncwarp();
          const int col0 = n_blk * BN + c0;
          if (p.c_f32) {
            uint32_t v[32];
            tmem_ld32(t_row + c0, v);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float f[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int col = col0 + 4 * j + i;
                f[i] = __uint_as_float(v[4 * j + i]) * p.alpha;
                if (p.bias && col < p.N) f[i] += __bfloat162float(p.bias[col]);
                if (p.residual && row_ok && col < p.N) f[i] += __bfloat162float(p.residual[row * p.ldr + col]);
              }
              *reinterpret_cast<float4*>(buf + swz128(lane, j)) = make_float4(f[0], f[1], f[2], f[3]);
            }
          } else {
            uint32_t v[32], v2[32];
            tmem_ld32(t_row + c0, v);
            tmem_ld32(t_row + c0 + 32, v2);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int col = col0 + 8 * j;
              float f[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(j < 4 ? v[8 * j + i] : v2[8 * (j - 4) + i]) * p.alpha;
              if (col < p.N) {
                if (p.bias) {
                  const uint4 b = *reinterpret_cast<const uint4*>(p.bias + col);
                  const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    const float2 bb = unpack_bf16x2(bw[i]);
                    f[2 * i] += bb.x;
                    f[2 * i + 1] += bb.y;
                  }
                }
                if (p.residual && row_ok) {
                  const uint4 r = *reinterpret_cast<const uint4*>(p.residual + row * p.ldr + col);
                  const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    const float2 rr = unpack_bf16x2(rw[i]);
                    f[2 * i] += rr.x;
                    f[2 * i + 1] += rr.y;
                  }
                }
              }
              *reinterpret_cast<uint4*>(buf + swz128(lane, j)) =
                  make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                             pack_bf16x2(f[6], f[7]));
            }
          }
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            if (p.tma_store == 2) tma_reduce_add_2d(&tmC, buf, col0, y0);
            else tma_store_2d(&tmC, buf, col0, y0);
            bulk_commit();
          }
        }
        tc_fence_before();
        if constexpr (PAIR) mbar_arrive_cluster(tempty_even + acc * 8);
        else mbar_arrive(&tempty[acc]);
        continue;
      }
      if (BN == 256 && p.glu_I) {
        // SwiGLU forward: accumulator columns [0,128) are gate, [128,256) the matching up columns.
        // Per 32-column chunk the warp writes h (and g, u when C is set) as 32 x 32 bf16 tiles through
        // four 2 KB staging slots (64B swizzle) and TMA stores.
        uint8_t* wbuf = smEpi + quarter * (2 * kEpiChunkBytes);
        const int y0 = m_blk * TM + static_cast<int>(rank) * kBM + quarter * 32;
        const int nout = p.C ? 3 : 1;
#pragma unroll 1
        for (int c0 = 0; c0 < 128; c0 += 32) {
          uint32_t vg[32], vu[32];
          tmem_ld32(t_row + c0, vg);
          tmem_ld32(t_row + 128 + c0, vu);
          tmem_wait_ld();
          const int x = n_blk * 128 + c0;
#pragma unroll 1
          for (int o = 0; o < nout; ++o) {
            uint8_t* buf = wbuf + (epi_chunk & 3) * 2048;
            ++epi_chunk;
            if (lane == 0) bulk_wait_read<3>();  // the store issued from this slot four stores ago
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t w4[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t g2 = pack_bf16x2(__uint_as_float(vg[8 * j + 2 * i]), __uint_as_float(vg[8 * j + 2 * i + 1]));
                const uint32_t u2 = pack_bf16x2(__uint_as_float(vu[8 * j + 2 * i]), __uint_as_float(vu[8 * j + 2 * i + 1]));
                if (o == 0) {
                  const float2 fg = unpack_bf16x2(g2), fu = unpack_bf16x2(u2);
                  w4[i] = pack_bf16x2(swiglu_h(fg.x, fu.x), swiglu_h(fg.y, fu.y));
                } else {
                  w4[i] = o == 1 ? g2 : u2;
                }
              }
              *reinterpret_cast<uint4*>(buf + swz64(lane, j)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0) {
              if (o == 0) tma_store_2d(&tmH, buf, x, y0);
              else tma_store_2d(&tmC, buf, (o == 2 ? p.glu_I : 0) + x, y0);
              bulk_commit();
            }
          }
        }
        tc_fence_before();
        if constexpr (PAIR) mbar_arrive_cluster(tempty_even + acc * 8);
        else mbar_arrive(&tempty[acc]);
        continue;
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tbase + (static_cast<uint32_t>(quarter * 32) << 16) + acc * BN + c0, v);
        tmem_wait_ld();
        const int col0 = n_blk * BN + c0;
        if (!row_ok) continue;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int col = col0 + g * 8;
          if (col >= p.N) break;
          float f[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(v[g * 8 + i]) * p.alpha;
          if (p.bias) {
            const uint4 b = *reinterpret_cast<const uint4*>(p.bias + col);
            const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 bb = unpack_bf16x2(bw[i]);
              f[2 * i] += bb.x;
              f[2 * i + 1] += bb.y;
            }
          }
          if (p.residual) {
            const uint4 r = *reinterpret_cast<const uint4*>(p.residual + row * p.ldr + col);
            const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 rr = unpack_bf16x2(rw[i]);
              f[2 * i] += rr.x;
              f[2 * i + 1] += rr.y;
            }
          }
          if (p.splits > 1) {
            // split-K partial: add into the fp32 output (pre-initialised by the caller)
            float* c = reinterpret_cast<float*>(p.C) + row * p.ldc + col;
            red_add_v4(c, f[0], f[1], f[2], f[3]);
            red_add_v4(c + 4, f[4], f[5], f[6], f[7]);
          } else if (p.c_f32 && p.beta == 1.f) {
            // accumulate into fp32 (weight gradients): each element has one writer, so a fire-and-forget
            // L2 reduction gives the same sum as load + add + store without a DRAM round trip per chunk
            float* c = reinterpret_cast<float*>(p.C) + row * p.ldc + col;
            red_add_v4(c, f[0], f[1], f[2], f[3]);
            red_add_v4(c + 4, f[4], f[5], f[6], f[7]);
          } else if (p.c_f32) {
            float* c = reinterpret_cast<float*>(p.C) + row * p.ldc + col;
            if (p.beta != 0.f) {
              const float4 o0 = *reinterpret_cast<const float4*>(c);
              const float4 o1 = *reinterpret_cast<const float4*>(c + 4);
              f[0] += p.beta * o0.x; f[1] += p.beta * o0.y; f[2] += p.beta * o0.z; f[3] += p.beta * o0.w;
              f[4] += p.beta * o1.x; f[5] += p.beta * o1.y; f[6] += p.beta * o1.z; f[7] += p.beta * o1.w;
            }
            *reinterpret_cast<float4*>(c) = make_float4(f[0], f[1], f[2], f[3]);
            *reinterpret_cast<float4*>(c + 4) = make_float4(f[4], f[5], f[6], f[7]);
          } else if (p.dglu_gu) {
            // SwiGLU backward: d(h) -> d(gate) at column col, d(up) at column N + col
            const __nv_bfloat16* gu = p.dglu_gu + row * p.ld_dglu + col;
            const uint4 gv = *reinterpret_cast<const uint4*>(gu);
            const uint4 uv = *reinterpret_cast<const uint4*>(gu + p.N);
            const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
            uint32_t og[4], ou[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float2 fg = unpack_bf16x2(gw[i]), fu = unpack_bf16x2(uw[i]);
              float dg0, du0, dg1, du1;
              swiglu_grads(fg.x, fu.x, bf16_round(f[2 * i]), dg0, du0);
              swiglu_grads(fg.y, fu.y, bf16_round(f[2 * i + 1]), dg1, du1);
              og[i] = pack_bf16x2(dg0, dg1);
              ou[i] = pack_bf16x2(du0, du1);
            }
            __nv_bfloat16* c = reinterpret_cast<__nv_bfloat16*>(p.C) + row * p.ldc + col;
            *reinterpret_cast<uint4*>(c) = make_uint4(og[0], og[1], og[2], og[3]);
            *reinterpret_cast<uint4*>(c + p.N) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
          } else {
            __nv_bfloat16* c;
            if (p.row_dst) {
              const long long dst = p.row_dst[row];
              if (dst == 0) continue;
              c = reinterpret_cast<__nv_bfloat16*>(dst) + col;
            } else {
              c = reinterpret_cast<__nv_bfloat16*>(p.C) + row * p.ldc + col;
            }
            if (p.beta != 0.f) {
              const uint4 o = *reinterpret_cast<const uint4*>(c);
              const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 oo = unpack_bf16x2(ow[i]);
                f[2 * i] += p.beta * oo.x;
                f[2 * i + 1] += p.beta * oo.y;
              }
            }
            uint4 o;
            o.x = pack_bf16x2(f[0], f[1]);
            o.y = pack_bf16x2(f[2], f[3]);
            o.z = pack_bf16x2(f[4], f[5]);
            o.w = pack_bf16x2(f[6], f[7]);
            *reinterpret_cast<uint4*>(c) = o;
          }
        }
      }
      tc_fence_before();
      if constexpr (PAIR) mbar_arrive_cluster(tempty_even + acc * 8);  // the even CTA's barrier
      else mbar_arrive(&tempty[acc]);
    }
    if (lane == 0) bulk_wait<0>();  // TMA stores of this warp complete before the CTA exits
  }

  if constexpr (PAIR) {
    tc_fence_before();
    cluster_sync();  // neither CTA leaves while the pair may still signal into its shared memory
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tbase, kTmemCols);
    }
  } else {
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tbase, kTmemCols);
    }
  }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapKey {
  uintptr_t ptr;
  uint64_t d0, d1, stride;
  uint32_t b0, b1, esize;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && d0 == o.d0 && d1 == o.d1 && stride == o.stride && b0 == o.b0 && b1 == o.b1 &&
           esize == o.esize;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.ptr);
    h ^= std::hash<uint64_t>()(k.d0 * 1315423911ull + k.d1) + 0x9e3779b97f4a7c15ull + (h << 6) + (h >> 2);
    h ^= std::hash<uint64_t>()(k.stride * 2654435761ull + (uint64_t(k.b0) << 32 | k.b1) + k.esize) + (h << 6) + (h >> 2);
    return h;
  }
};

std::mutex g_map_mutex;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_map_cache;

// 2-D tensor map (bf16, or fp32 with esize 4), 128B swizzle: inner dimension d0 (contiguous), outer d1
// with a row stride in elements.
bool make_map_2d(CUtensorMap* out, const void* ptr, uint64_t d0, uint64_t d1, uint64_t stride_elems, uint32_t b0,
                 uint32_t b1, uint32_t esize = 2, bool swizzle64 = false) {
  MapKey key{reinterpret_cast<uintptr_t>(ptr), d0, d1, stride_elems, b0, b1, esize + (swizzle64 ? 16u : 0u)};
  {
    std::lock_guard<std::mutex> g(g_map_mutex);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) {
      *out = it->second;
      return true;
    }
  }
  auto fn = get_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {d0, d1};
  cuuint64_t strides[1] = {stride_elems * esize};
  cuuint32_t box[2] = {b0, b1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(out, esize == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  std::lock_guard<std::mutex> g(g_map_mutex);
  if (g_map_cache.size() > 8192) g_map_cache.clear();
  g_map_cache.emplace(key, *out);
  return true;
}

int num_sms() { return device_sm_count(); }

template <int BN, int STAGES, bool A_MN, bool B_MN, bool PAIR, bool ROPE = false>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mh,
                GemmParams p, cudaStream_t stream, int max_ctas) {
  auto kern = gemm_bf16_tcgen05<BN, STAGES, A_MN, B_MN, PAIR, ROPE>;
  constexpr int smem_bytes =
      STAGES * GemmSmem<BN, PAIR>::kStageBytes + kEpiBytes + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(smem_bytes <= 232448, "shared memory per CTA");
  // per instantiation and device: clusters of 2 that can be resident at once, stored + 1 (0 = not yet known)
  static std::atomic<int> cluster_cache[kMaxHostDevices];
  const int dev = host_current_device();
  if (dev < 0 || dev >= kMaxHostDevices) return -14;
  int max_clusters = cluster_cache[dev].load(std::memory_order_acquire) - 1;
  if (max_clusters < 0) {
    cudaError_t e = smem_attr_once<gemm_bf16_tcgen05<BN, STAGES, A_MN, B_MN, PAIR, ROPE>>(smem_bytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (PAIR) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = smem_bytes;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess) return static_cast<int>(e);
      if (n < 1) return -13;
      max_clusters = n;
    } else {
      max_clusters = 0;
    }
    cluster_cache[dev].store(max_clusters + 1, std::memory_order_release);
  }
  if (!PAIR) {
    int grid = std::min(p.num_tiles, max_ctas > 0 ? max_ctas : num_sms());
    kern<<<grid, kThreads, smem_bytes, stream>>>(ma, mb, mc, mh, p);
    return static_cast<int>(cudaGetLastError());
  }
  int clusters = std::min(p.num_tiles, max_clusters);
  if (max_ctas > 0) clusters = std::max(1, std::min(clusters, max_ctas / 2));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * clusters, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return static_cast<int>(cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mh, p));
}

template <int BN, int STAGES, bool PAIR>
int dispatch_major(bool a_mn, bool b_mn, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc,
                   const CUtensorMap& mh, const GemmParams& p, cudaStream_t s, int max_ctas) {
  if (!a_mn && !b_mn) return launch_gemm<BN, STAGES, false, false, PAIR>(ma, mb, mc, mh, p, s, max_ctas);
  if (!a_mn && b_mn) return launch_gemm<BN, STAGES, false, true, PAIR>(ma, mb, mc, mh, p, s, max_ctas);
  if (a_mn && !b_mn) return launch_gemm<BN, STAGES, true, false, PAIR>(ma, mb, mc, mh, p, s, max_ctas);
  return launch_gemm<BN, STAGES, true, true, PAIR>(ma, mb, mc, mh, p, s, max_ctas);
}

// Output tensor map for the TMA-store epilogue, or 0 when the per-thread store path must be used
// (scatter rows, bf16 accumulation, the SwiGLU epilogues, beta other than 0 / 1, odd strides).
int output_map(CUtensorMap* mc, const GemmParams& p, uint64_t rows_total) {
  if (p.row_dst || p.glu_I || p.dglu_gu || !p.C) return 0;
  const uint32_t esize = p.c_f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(p.C) & 15) || ((p.ldc * esize) & 15)) return 0;
  int mode;
  if (p.c_f32 && (p.beta == 1.f || p.splits > 1)) mode = 2;
  else if (p.beta == 0.f && p.splits == 1) mode = 1;
  else return 0;
  if (!make_map_2d(mc, p.C, (uint64_t)p.N, rows_total, (uint64_t)p.ldc, p.c_f32 ? 32 : 64, 32, esize)) return 0;
  return mode;
}

}  // namespace
}  // namespace accerl

namespace {
struct EpilogueExtras {
  const long long* rope_pos = nullptr;
  int rope_cols = 0;
  float rope_log2_theta = 0.f;
  int glu_I = 0;
  void* glu_out = nullptr;
  long long ld_glu = 0;
  const void* dglu_gu = nullptr;
  long long ld_dglu = 0;
};

int gemm_dense(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn, void* C, long long ldc,
               int c_f32, int M, int N, int K, float alpha, float beta, const void* bias, const void* residual,
               long long ldr, int* status, int block_n, int max_ctas, int splits, cudaStream_t stream,
               const EpilogueExtras& ex) {
  using namespace accerl;
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0) return -1;
  // TMA needs 16-byte row strides; the per-thread epilogue needs N % 8 == 0 (the TMA-store epilogue
  // clips columns, so an fp32 output without bias / residual / accumulation may have any N). K and M
  // are free.
  const bool ragged_n_ok = c_f32 && !bias && !residual && beta == 0.f && splits <= 1 && (ldc % 4) == 0;
  if (((N % 8) != 0 && !ragged_n_ok) || ((N % 8) == 0 && (ldc % 8) != 0) || (lda % 8) != 0 || (ldb % 8) != 0)
    return -2;
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(C)) & 15) return -3;
  if (residual && ((ldr % 8) != 0 || (reinterpret_cast<uintptr_t>(residual) & 15))) return -4;
  if (bias && (reinterpret_cast<uintptr_t>(bias) & 15)) return -5;
  // Tile width and split-K are chosen to minimise wave quantisation: estimated time ~
  // ceil(work_items / SMs) * (k_blocks / splits) * tile_cost, with a 128-wide tile costing ~0.68x a
  // 256-wide one. Split-K is only possible for fp32 outputs accumulated with beta = 1.
  const int sms = num_sms();
  const int k_blocks_all = (K + kBK - 1) / kBK;
  const bool can_split = c_f32 && beta == 1.f && !bias && !residual;
  // block_n: 0 = choose, 128 / 256 = one CTA per tile of that width, -256 = CTA pair (256 x 256 tiles).
  int bn = block_n < 0 ? -block_n : block_n;
  bool pair = block_n < 0;
  int best_split = 1;
  {
    double best = 1e30;
    struct Opt { int bn; bool pair; double cost; };
    // Relative time per 64-deep k-block of one work item. A 128-wide tile moves as many A bytes per
    // MMA as B bytes and sits at the shared-memory operand bandwidth limit (measured tensor-pipe
    // utilisation 0.47 vs 0.66 for 256-wide tiles); a CTA pair halves each SM's B traffic and covers
    // twice the rows per work item.
    const Opt opts[3] = {{256, false, 2.0}, {128, false, 1.35}, {256, true, 2.0 * kPairCost}};
    for (const Opt& o : opts) {
      if (block_n != 0 && (o.bn != bn || o.pair != pair)) continue;
      if (ex.glu_I && o.bn != 256) continue;  // a SwiGLU tile is 128 gate + 128 up columns
      if (block_n == 0 && o.bn == 256 && N <= 128) continue;
      if (block_n == 0 && o.pair && !kPairAuto) continue;
      const int tm = o.pair ? 256 : 128;
      const int units = o.pair ? sms / 2 : sms;
      const long long tiles = (long long)((M + tm - 1) / tm) * ((N + o.bn - 1) / o.bn);
      // splitting only pays while the tile grid leaves SMs idle (partials cost extra fp32 traffic)
      const int max_split = (splits > 0) ? splits : ((can_split && tiles < units) ? 8 : 1);
      for (int sp = (splits > 0 ? splits : 1); sp <= max_split; ++sp) {
        if (sp > 1 && k_blocks_all / sp < 4) break;
        const long long items = tiles * sp;
        const double waves = (double)((items + units - 1) / units);
        const double t = waves * ((double)((k_blocks_all + sp - 1) / sp)) * o.cost;
        if (t < best * 0.97) {
          best = t;
          bn = o.bn;
          pair = o.pair;
          best_split = sp;
        }
      }
    }
  }
  if (splits <= 0) splits = best_split;
  CUtensorMap ma, mb;
  bool ok;
  if (a_mn) ok = make_map_2d(&ma, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, 64);
  else ok = make_map_2d(&ma, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 64, 128);
  if (!ok) return -7;
  if (b_mn) ok = make_map_2d(&mb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, 64);
  else ok = make_map_2d(&mb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 64,
                        (uint32_t)((pair || ex.glu_I) ? bn / 2 : bn));
  if (!ok) return -8;
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = C;
  p.ldc = ldc;
  p.c_f32 = c_f32;
  p.alpha = alpha;
  p.beta = beta;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.ldr = ldr;
  p.status = status;
  p.tiles_m = (M + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM);
  p.tiles_n = (N + bn - 1) / bn;
  const int k_blocks = k_blocks_all;
  if (splits > 1 && (!c_f32 || bias || residual || beta != 1.f)) return -9;
  p.kb_per_split = (k_blocks + splits - 1) / splits;
  p.splits = (k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.num_tiles = p.tiles_m * p.tiles_n * p.splits;
  p.group_m = 8;
  p.group_mode = 0;
  p.tile_expert = nullptr;
  p.group_row_start = nullptr;
  p.group_rows = nullptr;
  p.b_group_stride = 0;
  p.c_group_stride = 0;
  p.num_groups = 0;
  p.row_dst = nullptr;
  p.glu_I = ex.glu_I;
  p.glu_out = reinterpret_cast<__nv_bfloat16*>(ex.glu_out);
  p.ld_glu = ex.ld_glu;
  p.dglu_gu = reinterpret_cast<const __nv_bfloat16*>(ex.dglu_gu);
  p.ld_dglu = ex.ld_dglu;
  CUtensorMap mc = ma, mh = ma;
  p.tma_store = output_map(&mc, p, (uint64_t)M);
  if ((N % 8) != 0 && p.tma_store == 0) return -2;
  p.rope_pos = reinterpret_cast<const long long*>(ex.rope_pos);
  p.rope_cols = ex.rope_cols;
  p.rope_log2_theta = ex.rope_log2_theta;
  if (ex.rope_pos && (p.tma_store != 1 || c_f32 || (ex.rope_cols % 128) != 0 || a_mn || b_mn)) return -15;
  if (ex.rope_pos) {
    if (pair) return launch_gemm<256, 6, false, false, true, true>(ma, mb, mc, mh, p, stream, max_ctas);
    if (bn == 256) return launch_gemm<256, 4, false, false, false, true>(ma, mb, mc, mh, p, stream, max_ctas);
    return launch_gemm<128, 6, false, false, false, true>(ma, mb, mc, mh, p, stream, max_ctas);
  }
  if (ex.glu_I) {
    // the SwiGLU epilogue writes 32 x 32 tiles of h (and of g | u when kept) with TMA
    if (!make_map_2d(&mh, ex.glu_out, (uint64_t)ex.glu_I, (uint64_t)M, (uint64_t)ex.ld_glu, 32, 32, 2, true)) return -7;
    if (C && !make_map_2d(&mc, C, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, 32, 32, 2, true)) return -7;
  }
  if (pair) return dispatch_major<256, 6, true>(a_mn, b_mn, ma, mb, mc, mh, p, stream, max_ctas);
  if (bn == 256) return dispatch_major<256, 4, false>(a_mn, b_mn, ma, mb, mc, mh, p, stream, max_ctas);
  return dispatch_major<128, 6, false>(a_mn, b_mn, ma, mb, mc, mh, p, stream, max_ctas);
}
}  // namespace

// Returns 0 on success, a cudaError_t value on launch failure, or -1..-9 for argument errors.
extern "C" int accerl_gemm_bf16(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                                void* C, long long ldc, int c_f32, int M, int N, int K, float alpha, float beta,
                                const void* bias, const void* residual, long long ldr, int* status, int block_n,
                                int max_ctas, int splits, cudaStream_t stream) {
  return gemm_dense(A, lda, a_mn, B, ldb, b_mn, C, ldc, c_f32, M, N, K, alpha, beta, bias, residual, ldr, status,
                    block_n, max_ctas, splits, stream, EpilogueExtras{});
}

// Projection whose first rope_cols output columns (heads of 128) get the rotary embedding at position
// pos[row] in the epilogue (the qkv projection: q and k heads rotated, v untouched). bf16 output.
extern "C" int accerl_gemm_rope_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc,
                                     int M, int N, int K, const void* bias, const long long* pos, int rope_cols,
                                     float theta, int* status, int block_n, int max_ctas, cudaStream_t stream) {
  if (!pos || rope_cols <= 0 || rope_cols > N || !(theta > 0.f)) return -15;
  EpilogueExtras ex;
  ex.rope_pos = pos;
  ex.rope_cols = rope_cols;
  ex.rope_log2_theta = log2f(theta);
  return gemm_dense(A, lda, 0, B, ldb, 0, C, ldc, 0, M, N, K, 1.f, 0.f, bias, nullptr, 0, status, block_n, max_ctas, 1,
                    stream, ex);
}

// Gate/up projection fused with SwiGLU: for W = [gate; up] ([2I, K], K-major) computes g, u = X W^T
// and h = silu(g) * u ([M, I], row stride ldh); gu ([M, 2I], row stride ldgu) receives g | u when
// non-null (training keeps it for the backward). I must be a multiple of 128. -14: bad I.
extern "C" int accerl_gemm_glu_bf16(const void* X, long long ldx, const void* W, long long ldw, void* gu,
                                    long long ldgu, void* h, long long ldh, int M, int I, int K, int* status,
                                    int block_n, int max_ctas, cudaStream_t stream) {
  if (I <= 0 || I % 128) return -14;
  if (block_n != 0 && block_n != 256 && block_n != -256) return -14;
  if ((ldh % 8) || (reinterpret_cast<uintptr_t>(h) & 15)) return -3;
  EpilogueExtras ex;
  ex.glu_I = I;
  ex.glu_out = h;
  ex.ld_glu = ldh;
  // C (= gu) may be null: pass a valid dummy pointer/stride for the argument checks
  return gemm_dense(X, ldx, 0, W, ldw, 0, gu, gu ? ldgu : 8, 0, M, 2 * I, K, 1.f, 0.f, nullptr, nullptr, 0, status,
                    block_n, max_ctas, 1, stream, ex);
}

// Down-projection input gradient fused with the SwiGLU backward: dA = dY Wd ([M, I]; dY [M, K],
// Wd [K, I] row-major) is turned, with g | u from gu ([M, 2I], row stride ldgu), into
// d(gate) | d(up) in dgu ([M, 2I], row stride lddgu).
extern "C" int accerl_gemm_dglu_bf16(const void* dY, long long lddy, const void* Wd, long long ldwd, const void* gu,
                                     long long ldgu, void* dgu, long long lddgu, int M, int I, int K, int* status,
                                     int block_n, int max_ctas, cudaStream_t stream) {
  if (I <= 0 || I % 8 || (ldgu % 8) || (reinterpret_cast<uintptr_t>(gu) & 15)) return -14;
  EpilogueExtras ex;
  ex.dglu_gu = gu;
  ex.ld_dglu = ldgu;
  return gemm_dense(dY, lddy, 0, Wd, ldwd, 1, dgu, lddgu, 0, M, I, K, 1.f, 0.f, nullptr, nullptr, 0, status, block_n,
                    max_ctas, 1, stream, ex);
}

// out_bf16[m, n] = bf16(acc[m, n] + bias[n] + residual[m, n]) : finishing pass of a split-K GEMM.
__global__ void splitk_finish_kernel(const float* __restrict__ acc, long long lda, const __nv_bfloat16* __restrict__ bias,
                                     const __nv_bfloat16* __restrict__ residual, long long ldr,
                                     __nv_bfloat16* __restrict__ out, long long ldo, int M, int N) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (idx >= static_cast<long long>(M) * N) return;
  const int m = static_cast<int>(idx / N), n = static_cast<int>(idx % N);
  const float4 a0 = *reinterpret_cast<const float4*>(acc + m * lda + n);
  const float4 a1 = *reinterpret_cast<const float4*>(acc + m * lda + n + 4);
  float f[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
  if (bias) {
    for (int i = 0; i < 8; ++i) f[i] += __bfloat162float(bias[n + i]);
  }
  if (residual) {
    for (int i = 0; i < 8; ++i) f[i] += __bfloat162float(residual[m * ldr + n + i]);
  }
  uint4 o;
  o.x = accerl::pack_bf16x2(f[0], f[1]);
  o.y = accerl::pack_bf16x2(f[2], f[3]);
  o.z = accerl::pack_bf16x2(f[4], f[5]);
  o.w = accerl::pack_bf16x2(f[6], f[7]);
  *reinterpret_cast<uint4*>(out + m * ldo + n) = o;
}

extern "C" int accerl_splitk_finish(const float* acc, long long lda, const void* bias, const void* residual,
                                    long long ldr, void* out, long long ldo, int M, int N, cudaStream_t stream) {
  if (N % 8) return -1;
  const long long n8 = (long long)M * N / 8;
  if (n8 == 0) return 0;
  splitk_finish_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, stream>>>(
      acc, lda, (const __nv_bfloat16*)bias, (const __nv_bfloat16*)residual, ldr, (__nv_bfloat16*)out, ldo, M, N);
  return (int)cudaGetLastError();
}

// Grouped GEMM for expert MLPs (see GemmParams group_mode). Dimensions:
//  mode 1: A [M_total, K] (K-major) or the dgrad/fwd convention of accerl_gemm_bf16 with stacked B
//          of b_rows_total rows; C [M_total, N].
//  mode 2: A [rows_total, M] and B [rows_total, N] (both MN-major, K = rows_total); C is the stacked
//          [num_groups * c_group_stride, N] weight gradient (fp32, accumulated with beta = 1).
extern "C" int accerl_grouped_gemm_bf16(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn,
                                        void* C, long long ldc, int c_f32, int M, int N, int K, long long b_rows_total,
                                        float beta, int mode, const int* tile_expert, const int* group_row_start,
                                        const int* group_rows, int num_groups, int b_group_stride,
                                        long long c_group_stride, const long long* row_dst, int* status,
                                        cudaStream_t stream) {
  using namespace accerl;
  if (M <= 0 || N <= 0 || K <= 0 || num_groups <= 0) return 0;
  if ((N % 8) != 0 || (ldc % 8) != 0 || (lda % 8) != 0 || (ldb % 8) != 0) return -2;
  if (mode != 1 && mode != 2) return -10;
  if (mode == 2 && !(a_mn && b_mn && c_f32)) return -11;
  const int bn = N >= 256 ? 256 : 128;
  CUtensorMap ma, mb;
  bool ok;
  if (a_mn) ok = make_map_2d(&ma, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, 64, 64);
  else ok = make_map_2d(&ma, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, 64, 128);
  if (!ok) return -7;
  if (b_mn) ok = make_map_2d(&mb, B, (uint64_t)N, (uint64_t)b_rows_total, (uint64_t)ldb, 64, 64);
  else ok = make_map_2d(&mb, B, (uint64_t)K, (uint64_t)b_rows_total, (uint64_t)ldb, 64, (uint32_t)bn);
  if (!ok) return -8;
  GemmParams p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = C;
  p.ldc = ldc;
  p.c_f32 = c_f32;
  p.alpha = 1.f;
  p.beta = beta;
  p.bias = nullptr;
  p.residual = nullptr;
  p.ldr = 0;
  p.status = status;
  p.tiles_m = (M + kBM - 1) / kBM;
  p.tiles_n = (N + bn - 1) / bn;
  p.splits = 1;
  p.kb_per_split = (K + kBK - 1) / kBK;
  p.group_m = 8;
  p.group_mode = mode;
  p.rope_pos = nullptr;
  p.rope_cols = 0;
  p.rope_log2_theta = 0.f;
  p.glu_I = 0;
  p.glu_out = nullptr;
  p.ld_glu = 0;
  p.dglu_gu = nullptr;
  p.ld_dglu = 0;
  p.tile_expert = tile_expert;
  p.group_row_start = group_row_start;
  p.group_rows = group_rows;
  p.b_group_stride = b_group_stride;
  p.c_group_stride = c_group_stride;
  p.num_groups = num_groups;
  p.row_dst = row_dst;
  if (row_dst && (c_f32 || beta != 0.f)) return -12;
  p.num_tiles = p.tiles_m * p.tiles_n * (mode == 2 ? num_groups : 1);
  CUtensorMap mc = ma;
  // a per-expert weight-gradient tile must not spill into the next expert's rows
  if (mode == 1 || (p.M % kBM) == 0)
    p.tma_store = output_map(&mc, p, mode == 2 ? (uint64_t)num_groups * (uint64_t)c_group_stride : (uint64_t)M);
  else
    p.tma_store = 0;
  if (bn == 256) return dispatch_major<256, 4, false>(a_mn, b_mn, ma, mb, mc, ma, p, stream, 0);
  return dispatch_major<128, 6, false>(a_mn, b_mn, ma, mb, mc, ma, p, stream, 0);
}
