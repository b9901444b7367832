// Packed-varlen causal attention (GQA) on the sm_100a tensor cores, head_dim 128.
//
// Forward, one CTA per (128-query tile, q head, sequence), 6 warps:
//   warp 4     TMA producer: the Q tile once, then K/V tiles of 128 keys into a 2-stage ring.
//   warp 5     MMA issuer: S_j = Q K_j^T into one of two TMEM score buffers, then O += P_{j-1} V_{j-1}
//              with P read from TMEM (V as an MN-major smem operand) into a TMEM output accumulator.
//   warps 0-3  softmax, one query row per thread (= one TMEM lane): tcgen05.ld the score row, mask,
//              online max/sum in the log2 domain, write P as bf16 back into the first 64 columns of
//              the same score buffer. O is rescaled in TMEM only when the running max grows by more
//              than 2^8, and only then does the tile wait for the previous PV MMA, so the softmax of
//              tile j+1 overlaps the PV MMA of tile j; the final normalisation uses the same stale max.
// Backward, one CTA per (128-key tile, q head, sequence): S^T = K Q^T and dP^T = V dO^T land in TMEM,
// the softmax warps (one key row per thread) rebuild P^T and dS^T into smem, then dV += P^T dO,
// dK += dS^T Q (accumulated in TMEM over all query tiles) and dQ_i = dS_i K (TMEM, drained with fp32
// vector atomics). dS^T in smem serves both as the K-major A of dK and the MN-major A of dQ.
// K/V gradients are written per q head in fp32 and summed over each GQA group by a reduction kernel.
// No cluster multicast is used.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"

namespace accerl {

constexpr int kHd = 128;        // head dim
constexpr int kTile = 128;      // rows per q / kv tile
constexpr int kChunk = 16384;   // one [128 rows x 64 bf16] 128B-swizzled chunk
constexpr int kTileBytes = 2 * kChunk;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// K-major descriptor of a [128 rows x 128 elems] tile stored as two 64-element chunks; kk = 16-elem K step.
ACCERL_DEVINL uint64_t desc_kmajor(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * kChunk + (kk & 3) * 32, 16, 1024);
}
// MN-major descriptor of the same physical tile when its rows are the K dimension.
ACCERL_DEVINL uint64_t desc_mnmajor(uint32_t base, int kk) {
  return make_sw128_desc(base + kk * 16 * 128, kChunk, 1024);
}

// Byte offset of 16-byte unit u (0..15) of row r inside a two-chunk swizzled tile.
ACCERL_DEVINL uint32_t swz_offset(int r, int u) {
  return (u >> 3) * kChunk + r * 128 + (((u & 7) ^ (r & 7)) << 4);
}

// Max of a 128-value row with eight independent comparison chains.
ACCERL_DEVINL float row_max128(const float (&x)[128]) {
  float m[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) m[i] = x[i];
#pragma unroll
  for (int e = 8; e < 128; ++e) m[e & 7] = fmaxf(m[e & 7], x[e]);
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

struct AttnFwdParams {
  __nv_bfloat16* o;
  float* lse;
  const int* cu;
  const int* cu_k;  // key boundaries; equal to cu for self-attention over packed sequences
  int max_tiles, T, Hq, Hkv;
  long long ldo;
  float scale_log2;
  int causal;
  int* status;
  // paged keys (prefill over a paged KV cache): key position kp of sequence b lives in cache row
  // block_table[b * max_blocks + kp / block_size] * block_size + kp % block_size; null = contiguous
  const int* block_table;
  int max_blocks, block_size;
};

// Work order of the varlen kernels, launched as a (max_tiles * Hq) x num_seqs grid: blocks start in
// increasing linear index, and the linear index is read tile-major -- tile rank outermost, then the
// sequence, then the head -- so the longest-running tiles of EVERY sequence of a pack start first
// (causal: the last query tiles in the forward, the first key tiles in the backward) instead of one
// sequence after the other, which left the long tiles of the last sequences running alone at the end.
struct TileSeqHead {
  int tile, seq, head;
};

ACCERL_DEVINL TileSeqHead tile_major(int Hq) {
  // the grid has far fewer than 2^32 blocks (tiles x heads x sequences of one pack)
  const unsigned lin = blockIdx.y * gridDim.x + blockIdx.x;
  const unsigned per_tile = static_cast<unsigned>(Hq) * gridDim.y;
  const unsigned r = lin % per_tile;
  return {static_cast<int>(lin / per_tile), static_cast<int>(r / Hq), static_cast<int>(r % Hq)};
}

__global__ void __launch_bounds__(192, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnFwdParams p) {
  const TileSeqHead at = tile_major(p.Hq);
  const int head = at.head;
  const int q_tile = p.max_tiles - 1 - at.tile;
  const int b = at.seq;
  const int seq_start = p.cu[b];
  const int len = p.cu[b + 1] - seq_start;
  if (q_tile * kTile >= len) return;
  // Keys may outnumber queries (a chunk of new queries over a cached prefix): query i sits at key
  // position i + k_off, and causal masking is aligned to the end of the key range.
  const int k_start = p.cu_k[b];
  const int len_k = p.cu_k[b + 1] - k_start;
  const int k_off = len_k - len;
  const int kv_tiles = (len_k + kTile - 1) / kTile;
  const int n_kv = p.causal ? min(kv_tiles, (q_tile * kTile + kTile - 1 + k_off) / kTile + 1) : kv_tiles;
  const int kvh = head / (p.Hq / p.Hkv);
  if (n_kv <= 0) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;
  uint8_t* sV = sK + 2 * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* kv_empty = bars + 5;   // [2]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;
  uint64_t* o_done = bars + 10;   // after every PV (waited only before a rescale: at most one behind)
  uint64_t* o_final = bars + 11;  // once, after the last PV
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
    }
    mbar_init(p_full, 128);
    mbar_init(o_done, 1);
    mbar_init(o_final, 1);
    fence_mbar_init();
  }
  if (warp == 5) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase;         // two score buffers: columns [0,128) and [128,256)
  const uint32_t tO = tbase + 256;   // output accumulator: columns [256,384)

  if (warp == 4 && p.block_table) {
    // ---- paged keys: one TMA box per page; lane i looks up page i's block id in parallel ----
    __shared__ int s_blk[kTile / 8];
    const int bs = p.block_size;
    const int pages = kTile / bs;
    const int* table = p.block_table + static_cast<long long>(b) * p.max_blocks;
    if (lane == 0) {
      const int qy = seq_start + q_tile * kTile;
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tmQ, q_full, head * kHd, qy);
      tma_load_2d(sQ + kChunk, &tmQ, q_full, head * kHd + 64, qy);
    }
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      const int s = j & 1;
      int blk = 0;
      if (lane < pages) {
        const int kp = j * kTile + lane * bs;
        blk = kp < len_k ? table[kp / bs] : 0;  // pages past the keys: any valid block, masked
      }
      int good = 1;
      if (lane == 0) good = mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1u, p.status, kStatusTimeoutProducer) ? 1 : 0;
      good = __shfl_sync(0xffffffffu, good, 0);
      if (!good) {
        ok = false;
        break;
      }
      if (lane < pages) s_blk[lane] = blk;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        for (int pg = 0; pg < pages; ++pg) {
          uint8_t* dst = sK + s * kTileBytes + pg * bs * 128;
          tma_load_2d(dst, &tmK, &k_full[s], kvh * kHd, s_blk[pg] * bs);
          tma_load_2d(dst + kChunk, &tmK, &k_full[s], kvh * kHd + 64, s_blk[pg] * bs);
        }
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        for (int pg = 0; pg < pages; ++pg) {
          uint8_t* dst = sV + s * kTileBytes + pg * bs * 128;
          tma_load_2d(dst, &tmV, &v_full[s], kvh * kHd, s_blk[pg] * bs);
          tma_load_2d(dst + kChunk, &tmV, &v_full[s], kvh * kHd + 64, s_blk[pg] * bs);
        }
      }
      __syncwarp();
    }
    if (!ok && lane == 0) mbar_wait(q_full, 0, nullptr, 0, 20000000ull);
  } else if (warp == 4) {
    if (lane == 0) {
      const int qy = seq_start + q_tile * kTile;
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_2d(sQ, &tmQ, q_full, head * kHd, qy);
      tma_load_2d(sQ + kChunk, &tmQ, q_full, head * kHd + 64, qy);
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1u, p.status, kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        const int ky = k_start + j * kTile;
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_2d(sK + s * kTileBytes, &tmK, &k_full[s], kvh * kHd, ky);
        tma_load_2d(sK + s * kTileBytes + kChunk, &tmK, &k_full[s], kvh * kHd + 64, ky);
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_2d(sV + s * kTileBytes, &tmV, &v_full[s], kvh * kHd, ky);
        tma_load_2d(sV + s * kTileBytes + kChunk, &tmV, &v_full[s], kvh * kHd + 64, ky);
      }
      if (!ok) {
        mbar_wait(q_full, 0, nullptr, 0, 20000000ull);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, p.status, kStatusTimeoutMma);
      for (int j = 0; j <= n_kv && ok; ++j) {
        if (j < n_kv) {
          const int s = j & 1;
          if (!mbar_wait(&k_full[s], (j >> 1) & 1, p.status, kStatusTimeoutMma)) break;
          // buffer s held P_{j-2}; PV_{j-2} was issued before this MMA, and tcgen05.mma executes in issue order
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + s * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(tS + s * 128, desc_kmajor(q_addr, kk), desc_kmajor(k_addr, kk), idesc_s, kk > 0);
          umma_commit(&s_full[s]);
        }
        if (j >= 1) {
          const int jj = j - 1;
          const int s2 = jj & 1;
          if (!mbar_wait(p_full, jj & 1, p.status, kStatusTimeoutMma)) break;
          if (!mbar_wait(&v_full[s2], (jj >> 1) & 1, p.status, kStatusTimeoutMma)) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + s2 * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16_ts(tO, tS + s2 * 128 + kk * 8, desc_mnmajor(v_addr, kk), idesc_o, (jj > 0) || (kk > 0));
          umma_commit(o_done);
          umma_commit(&kv_empty[s2]);
        }
      }
      umma_commit(o_final);
    }
  } else {
    // ---------------- softmax warps 0..3: thread = query row ----------------
    const int r = threadIdx.x;  // 0..127 == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const int q_pos = q_tile * kTile + r;
    float m_used = -INFINITY;
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int bsel = j & 1;
      if (!mbar_wait(&s_full[bsel], (j >> 1) & 1, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[128];
      {
        uint32_t v[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tS + bsel * 128 + c * 32 + lane_off, v[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(v[c][e]) * p.scale_log2;
      }
      const int kbase = j * kTile;
      if ((p.causal && kbase + kTile - 1 > q_tile * kTile + k_off) || kbase + kTile > len_k) {
        const int lim = q_pos + k_off;
#pragma unroll
        for (int e = 0; e < 128; ++e) {
          const int kp = kbase + e;
          if ((p.causal && kp > lim) || kp >= len_k) x[e] = -INFINITY;
        }
      }
      const float mx = row_max128(x);
      const float m_new = fmaxf(m_used, mx);
      const bool need = m_new > m_used + 8.0f;
      float alpha = 1.f;
      if (need) {
        alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
        m_used = m_new;
        l *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O may only be rescaled once PV_{j-1} has landed. s_full(j) covered every MMA issued before
        // S_j (PV_{j-2} included), so o_done is at most one completion behind and its parity is exact.
        if (!mbar_wait(o_done, (j - 1) & 1, p.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(tO + c * 32 + lane_off, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
          tmem_st32(tO + c * 32 + lane_off, v);
        }
        tmem_wait_st();
      }
      const float m_eff = (m_used == -INFINITY) ? 0.f : m_used;
      // P (bf16, two per 32-bit column) back into the first 64 columns of this tile's S buffer: the
      // PV MMA reads it as its TMEM A operand
      float ls[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums (no 128-long add chain)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t w[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const float p0 = exp2f(x[half * 64 + 2 * u] - m_eff);
          const float p1 = exp2f(x[half * 64 + 2 * u + 1] - m_eff);
          ls[u & 3] += p0 + p1;
          w[u] = pack_bf16x2(p0, p1);
        }
        tmem_st32(tS + bsel * 128 + half * 32 + lane_off, w);
      }
      l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(o_final, 0, p.status, kStatusTimeoutEpilogue)) {
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      const bool row_ok = q_pos < len;
      __nv_bfloat16* orow = p.o + static_cast<long long>(seq_start + q_pos) * p.ldo + head * kHd;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tO + c * 32 + lane_off, v);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 o;
            o.x = pack_bf16x2(__uint_as_float(v[g * 8 + 0]) * inv_l, __uint_as_float(v[g * 8 + 1]) * inv_l);
            o.y = pack_bf16x2(__uint_as_float(v[g * 8 + 2]) * inv_l, __uint_as_float(v[g * 8 + 3]) * inv_l);
            o.z = pack_bf16x2(__uint_as_float(v[g * 8 + 4]) * inv_l, __uint_as_float(v[g * 8 + 5]) * inv_l);
            o.w = pack_bf16x2(__uint_as_float(v[g * 8 + 6]) * inv_l, __uint_as_float(v[g * 8 + 7]) * inv_l);
            *reinterpret_cast<uint4*>(orow + c * 32 + g * 8) = o;
          }
        }
      }
      if (row_ok) {
        const float m_eff = (m_used == -INFINITY) ? 0.f : m_used;
        p.lse[static_cast<long long>(head) * p.T + seq_start + q_pos] = (m_eff + log2f(l)) * kLn2;
      }
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// paged decode on the tensor cores
// ------------------------------------------------------------------------------------------------
// One work item = (sequence, KV head, key split). The G query heads that share the KV head are the
// M rows of the MMAs (rows G..127 of Q are zero), so S = Q K^T and O += P V run as 128 x 128 x 128
// tcgen05 MMAs over 128-token key tiles whose pages TMA gathers from the paged cache (one box per
// page). The kernel is persistent: each CTA walks work items with a continuous 2-stage K/V ring, and
// writes the unnormalised partial output, the running max (natural log units) and the sum of each
// item for the split-merge kernel. Warp 0 builds Q and runs the softmax of the G rows; warp 4 loads;
// warp 5 issues the MMAs and owns TMEM.
constexpr int kDecStages = 3;  // K/V ring depth of the decode kernel (Q + 3 x (K, V) = 224 KB)

struct DecodeTcParams {
  const __nv_bfloat16* q;
  long long ldq;
  const int* block_table;
  int max_blocks;
  const int* seq_lens;
  int num_seqs, Hq, Hkv, G, block_size, num_splits;
  int num_blocks;  // pages in the cache (debug-checks build: page ids are range-checked)
  float scale_log2;
  float* part_o;
  float* part_ml;
  int* status;
};

struct DecodeItem {
  int s, kvh, split, t0, t1, ntiles;
};

ACCERL_DEVINL DecodeItem decode_item(const DecodeTcParams& p, int it) {
  DecodeItem d;
  d.split = it % p.num_splits;
  d.kvh = (it / p.num_splits) % p.Hkv;
  d.s = it / (p.num_splits * p.Hkv);
  const int len = p.seq_lens[d.s];
  // splits are whole 128-token tiles so every tile starts on a page boundary
  const int per = ((((len + p.num_splits - 1) / p.num_splits) + kTile - 1) / kTile) * kTile;
  d.t0 = d.split * per;
  d.t1 = min(len, d.t0 + per);
  d.ntiles = d.t1 > d.t0 ? (d.t1 - d.t0 + kTile - 1) / kTile : 0;
  return d;
}

__global__ void __launch_bounds__(192, 1)
    paged_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const DecodeTcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kTileBytes;
  uint8_t* sV = sK + kDecStages * kTileBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kDecStages * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;                    // [kDecStages]
  uint64_t* v_full = k_full + kDecStages;         // [kDecStages]
  uint64_t* kv_empty = v_full + kDecStages;       // [kDecStages]
  uint64_t* s_full = kv_empty + kDecStages;       // [2] (TMEM score buffers)
  uint64_t* p_full = s_full + 2;
  uint64_t* o_done = p_full + 1;  // after every PV
  uint64_t* o_item = p_full + 2;  // after the last PV of an item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(p_full + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_items = p.num_seqs * p.Hkv * p.num_splits;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 32);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(&s_full[s], 1);
    mbar_init(p_full, 32);
    mbar_init(o_done, 1);
    mbar_init(o_item, 1);
    fence_mbar_init();
  }
  // rows G..127 of Q stay zero for the whole kernel
  if (warp < 4)
    for (int i = threadIdx.x; i < kTileBytes / 16; i += 128) reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
  fence_async_shared();
  if (warp == 5) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase;        // two score buffers: columns [0,128) and [128,256)
  const uint32_t tO = tbase + 256;  // output accumulator: columns [256,384)

  if (warp == 4) {
    // ---------------- TMA producer: one box per page of the tile ----------------
    // Lane i looks up page i's block id (independent loads, issued before the stage wait so their
    // latency overlaps it); lane 0 then issues the page boxes from a shared-memory copy of the ids.
    __shared__ int s_blk[kTile / 8];
    const int bs = p.block_size;
    const int pages = kTile / bs;
    int g = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < num_items && ok; it += gridDim.x) {
      const DecodeItem d = decode_item(p, it);
      const int* table = p.block_table + static_cast<long long>(d.s) * p.max_blocks;
      for (int j = 0; j < d.ntiles; ++j, ++g) {
        int blk = 0;
        if (lane < pages) {
          const int tok = d.t0 + j * kTile + lane * bs;
          blk = tok < d.t1 ? table[tok / bs] : 0;  // pages past the end: any valid block, masked
          if (!ACCERL_DBG_OK(blk >= 0 && blk < p.num_blocks, kDbgPageId, blk)) blk = 0;
        }
        const int st = g % kDecStages;
        int good = 1;
        if (lane == 0)
          good = mbar_wait(&kv_empty[st], ((g / kDecStages) & 1) ^ 1u, p.status, kStatusTimeoutProducer) ? 1 : 0;
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
        if (lane < pages) s_blk[lane] = blk;
        __syncwarp();
        if (lane == 0) {
          mbar_arrive_expect_tx(&k_full[st], kTileBytes);
          for (int pg = 0; pg < pages; ++pg) {
            const int b = s_blk[pg] * bs;
            uint8_t* dst = sK + st * kTileBytes + pg * bs * 128;
            tma_load_2d(dst, &tmK, &k_full[st], d.kvh * kHd, b);
            tma_load_2d(dst + kChunk, &tmK, &k_full[st], d.kvh * kHd + 64, b);
          }
          mbar_arrive_expect_tx(&v_full[st], kTileBytes);
          for (int pg = 0; pg < pages; ++pg) {
            const int b = s_blk[pg] * bs;
            uint8_t* dst = sV + st * kTileBytes + pg * bs * 128;
            tma_load_2d(dst, &tmV, &v_full[st], d.kvh * kHd, b);
            tma_load_2d(dst + kChunk, &tmV, &v_full[st], d.kvh * kHd + 64, b);
          }
        }
        __syncwarp();  // s_blk is rewritten next tile
      }
    }
    if (lane == 0) {
      // never leave a bulk copy in flight into shared memory of a finished CTA
      for (int t = max(0, g - kDecStages); t < g; ++t)
        mbar_wait(&v_full[t % kDecStages], (t / kDecStages) & 1, nullptr, 0, 20000000ull);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      int g = 0, itn = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < num_items && ok; it += gridDim.x) {
        const DecodeItem d = decode_item(p, it);
        if (d.ntiles == 0) continue;
        if (!mbar_wait(q_full, itn & 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        for (int j = 0; j <= d.ntiles; ++j) {
          if (j < d.ntiles) {
            const int gg = g + j;
            const int st = gg % kDecStages;
            const int sb = gg & 1;  // TMEM score buffer
            if (!mbar_wait(&k_full[st], (gg / kDecStages) & 1, p.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            // score buffer sb held P of tile gg-2, whose PV was issued before this MMA (issue order)
            tc_fence_after();
            const uint32_t k_addr = smem_u32(sK + st * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16(tS + sb * 128, desc_kmajor(q_addr, kk), desc_kmajor(k_addr, kk), idesc_s, kk > 0);
            umma_commit(&s_full[sb]);
            if (j == d.ntiles - 1) umma_commit(q_empty);
          }
          if (j >= 1) {
            const int gg = g + j - 1;
            const int st2 = gg % kDecStages;
            const int sb2 = gg & 1;
            if (!mbar_wait(p_full, gg & 1, p.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            if (!mbar_wait(&v_full[st2], (gg / kDecStages) & 1, p.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(sV + st2 * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16_ts(tO, tS + sb2 * 128 + kk * 8, desc_mnmajor(v_addr, kk), idesc_o, (j > 1) || (kk > 0));
            umma_commit(o_done);
            umma_commit(&kv_empty[st2]);
          }
        }
        if (!ok) break;
        umma_commit(o_item);
        g += d.ntiles;
        ++itn;
      }
    }
  } else if (warp == 0) {
    // ---------------- Q rows and the softmax of the G real rows: thread = query head ----------------
    const int r = lane;
    int g = 0, itn = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < num_items && ok; it += gridDim.x) {
      const DecodeItem d = decode_item(p, it);
      const int hq = d.kvh * p.G + r;
      const long long pidx = (static_cast<long long>(d.s) * p.Hq + hq) * p.num_splits + d.split;
      if (d.ntiles == 0) {
        if (r < p.G) {
          for (int c = 0; c < kHd; c += 4)
            *reinterpret_cast<float4*>(p.part_o + pidx * kHd + c) = make_float4(0.f, 0.f, 0.f, 0.f);
          p.part_ml[pidx * 2] = -INFINITY;
          p.part_ml[pidx * 2 + 1] = 0.f;
        }
        continue;
      }
      if (itn > 0 && !mbar_wait(q_empty, (itn - 1) & 1, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      if (r < p.G) {
        const uint4* src = reinterpret_cast<const uint4*>(p.q + static_cast<long long>(d.s) * p.ldq + hq * kHd);
#pragma unroll
        for (int u = 0; u < 16; ++u) *reinterpret_cast<uint4*>(sQ + swz_offset(r, u)) = src[u];
      }
      fence_async_shared();
      mbar_arrive(q_full);
      const uint32_t lane_off = 0;  // warp 0 reads TMEM lanes 0..31
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < d.ntiles; ++j) {
        const int gg = g + j;
        const int bsel = gg & 1;
        if (!mbar_wait(&s_full[bsel], (gg >> 1) & 1, p.status, kStatusTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float x[128];
        {
          uint32_t v[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(tS + bsel * 128 + c * 32 + lane_off, v[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) x[c * 32 + e] = __uint_as_float(v[c][e]) * p.scale_log2;
        }
        const int kbase = d.t0 + j * kTile;
        if (kbase + kTile > d.t1) {
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (kbase + e >= d.t1) x[e] = -INFINITY;
        }
        const float mx = row_max128(x);
        const float m_new = fmaxf(m_used, mx);
        const bool need = m_new > m_used + 8.0f;
        float alpha = 1.f;
        if (need) {
          alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
          m_used = m_new;
          l *= alpha;
        }
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // rescale O once the previous PV has landed (o_done is at most one completion behind)
          if (!mbar_wait(o_done, (gg - 1) & 1, p.status, kStatusTimeoutEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld32(tO + c * 32 + lane_off, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * alpha);
            tmem_st32(tO + c * 32 + lane_off, v);
          }
          tmem_wait_st();
        }
        const float m_eff = (m_used == -INFINITY) ? 0.f : m_used;
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t w[32];
#pragma unroll
          for (int u = 0; u < 32; ++u) {
            const float p0 = exp2f(x[half * 64 + 2 * u] - m_eff);
            const float p1 = exp2f(x[half * 64 + 2 * u + 1] - m_eff);
            ls[u & 3] += p0 + p1;
            w[u] = pack_bf16x2(p0, p1);
          }
          tmem_st32(tS + bsel * 128 + half * 32 + lane_off, w);
        }
        l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(p_full);
      }
      if (!ok) break;
      if (!mbar_wait(o_item, itn & 1, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tO + c * 32 + lane_off, v);
        tmem_wait_ld();
        if (r < p.G) {
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(p.part_o + pidx * kHd + c * 32 + e) =
                make_float4(__uint_as_float(v[e]), __uint_as_float(v[e + 1]), __uint_as_float(v[e + 2]),
                            __uint_as_float(v[e + 3]));
        }
      }
      if (r < p.G) {
        p.part_ml[pidx * 2] = m_used == -INFINITY ? -INFINITY : m_used * kLn2;
        p.part_ml[pidx * 2 + 1] = l;
      }
      tc_fence_before();
      g += d.ntiles;
      ++itn;
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// paged decode with the keys on the TMEM lanes
// ------------------------------------------------------------------------------------------------
// Same work items, K/V ring, page gathers and split outputs as paged_decode_tc_kernel, with the
// products transposed so that the 128 keys of a tile, not the G query heads, are the MMA rows:
//   S^T [128 keys x NQ]  = K [128 keys x 128 dims] . Q^T     (A: K tile, K-major; B: Q rows, K-major)
//   O^T [128 dims x NQ] += V^T [128 dims x 128 keys] . P^T   (A: V tile, MN-major; B: P rows, K-major)
// with NQ = G rounded up to 16 or 32; the per-head softmax loops run over GM = G rounded up to a power
// of two, unrolled without per-head branches so the reductions of all heads overlap (heads G..GM-1
// have zero Q rows and their results are never written). Thread t of the four softmax warps owns key t of every tile
// (TMEM lane t) and head dim t of the output, so the exponentials of a tile are spread over all four
// SM sub-partitions (G per thread instead of 128 per query head in one warp) and the MMAs are NQ wide
// instead of 128. The per-head tile maximum is exchanged through shared memory once per tile; the
// sums stay per thread until the item ends. Rescaling stays lazy (only when the maximum grows by more
// than 2^8), as in the tile-per-head kernel.
template <int NQ, int GM>
__global__ void __launch_bounds__(192, 1)
    paged_decode_tq_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                           const DecodeTcParams p) {
  constexpr int kQChunk = NQ * 128;  // NQ rows x 64 bf16 (one 128-byte swizzled column chunk)
  constexpr int kQBytes = 2 * kQChunk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kDecStages * kTileBytes;
  uint8_t* sQ = sV + kDecStages * kTileBytes;
  uint8_t* sP = sQ + kQBytes;                                   // [2][NQ rows x 128 keys]
  float* s_max = reinterpret_cast<float*>(sP + 2 * kQBytes);    // [2][4 warps][NQ]
  float* s_sum = s_max + 2 * 4 * NQ;                            // [4 warps][NQ]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_sum + 4 * NQ);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;                // [kDecStages]
  uint64_t* v_full = k_full + kDecStages;     // [kDecStages]
  uint64_t* kv_empty = v_full + kDecStages;   // [kDecStages]
  uint64_t* s_full = kv_empty + kDecStages;   // [2] S^T buffers
  uint64_t* p_full = s_full + 2;              // [2] P buffers
  uint64_t* o_done = p_full + 2;              // after every PV
  uint64_t* o_item = o_done + 1;              // after the last PV of an item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_item + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_items = p.num_seqs * p.Hkv * p.num_splits;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 128);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 128);
    }
    mbar_init(o_done, 1);
    mbar_init(o_item, 1);
    fence_mbar_init();
  }
  // rows G..NQ-1 of Q and P stay zero for the whole kernel
  if (warp < 4)
    for (int i = threadIdx.x; i < 3 * kQBytes / 16; i += 128) reinterpret_cast<uint4*>(sQ)[i] = make_uint4(0, 0, 0, 0);
  fence_async_shared();
  if (warp == 5) tmem_alloc(tmem_slot, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase;           // two S^T buffers: columns [0, NQ) and [NQ, 2 NQ)
  const uint32_t tO = tbase + 2 * NQ;  // O^T accumulator: columns [2 NQ, 3 NQ)

  if (warp == 4) {
    // ---------------- TMA producer: lane i gathers page i of the tile ----------------
    // Every lane looks its block id up and issues the four boxes (K and V, two column halves) of its
    // own page, so the up to 32 bulk copies of a tile leave the warp in parallel instead of one
    // after another from a single thread.
    const int bs = p.block_size;
    const int pages = kTile / bs;
    int g = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < num_items && ok; it += gridDim.x) {
      const DecodeItem d = decode_item(p, it);
      const int* table = p.block_table + static_cast<long long>(d.s) * p.max_blocks;
      for (int j = 0; j < d.ntiles; ++j, ++g) {
        int blk = 0;
        if (lane < pages) {
          const int tok = d.t0 + j * kTile + lane * bs;
          blk = tok < d.t1 ? table[tok / bs] : 0;  // pages past the end: any valid block, masked
          if (!ACCERL_DBG_OK(blk >= 0 && blk < p.num_blocks, kDbgPageId, blk)) blk = 0;
        }
        const int st = g % kDecStages;
        int good = 1;
        if (lane == 0) {
          good = mbar_wait(&kv_empty[st], ((g / kDecStages) & 1) ^ 1u, p.status, kStatusTimeoutProducer) ? 1 : 0;
          if (good) {
            mbar_arrive_expect_tx(&k_full[st], kTileBytes);
            mbar_arrive_expect_tx(&v_full[st], kTileBytes);
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) {
          ok = false;
          break;
        }
        if (lane < pages) {
          const int b = blk * bs;
          uint8_t* dk = sK + st * kTileBytes + lane * bs * 128;
          uint8_t* dv = sV + st * kTileBytes + lane * bs * 128;
          tma_load_2d(dk, &tmK, &k_full[st], d.kvh * kHd, b);
          tma_load_2d(dk + kChunk, &tmK, &k_full[st], d.kvh * kHd + 64, b);
          tma_load_2d(dv, &tmV, &v_full[st], d.kvh * kHd, b);
          tma_load_2d(dv + kChunk, &tmV, &v_full[st], d.kvh * kHd + 64, b);
        }
      }
    }
    if (lane == 0) {
      // never leave a bulk copy in flight into shared memory of a finished CTA
      for (int t = max(0, g - kDecStages); t < g; ++t)
        mbar_wait(&v_full[t % kDecStages], (t / kDecStages) & 1, nullptr, 0, 20000000ull);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, NQ, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, NQ, true, false);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      int g = 0, itn = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < num_items && ok; it += gridDim.x) {
        const DecodeItem d = decode_item(p, it);
        if (d.ntiles == 0) continue;
        if (!mbar_wait(q_full, itn & 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        for (int j = 0; j <= d.ntiles; ++j) {
          if (j < d.ntiles) {
            const int gg = g + j;
            const int st = gg % kDecStages;
            const int sb = gg & 1;
            if (!mbar_wait(&k_full[st], (gg / kDecStages) & 1, p.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            // S^T buffer sb was read by the softmax of tile gg-2 before it released P of that tile,
            // whose PV this thread issued before this MMA
            tc_fence_after();
            const uint32_t k_addr = smem_u32(sK + st * kTileBytes);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16(tS + sb * NQ, desc_kmajor(k_addr, kk),
                        make_sw128_desc(q_addr + (kk >> 2) * kQChunk + (kk & 3) * 32, 16, 1024), idesc_s, kk > 0);
            umma_commit(&s_full[sb]);
            if (j == d.ntiles - 1) umma_commit(q_empty);
          }
          if (j >= 1) {
            const int gg = g + j - 1;
            const int st2 = gg % kDecStages;
            const int pb = gg & 1;
            if (!mbar_wait(&p_full[pb], (gg >> 1) & 1, p.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            if (!mbar_wait(&v_full[st2], (gg / kDecStages) & 1, p.status, kStatusTimeoutMma)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t v_addr = smem_u32(sV + st2 * kTileBytes);
            const uint32_t pbuf = p_addr + pb * kQBytes;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              umma_bf16(tO, desc_mnmajor(v_addr, kk),
                        make_sw128_desc(pbuf + (kk >> 2) * kQChunk + (kk & 3) * 32, 16, 1024), idesc_o,
                        (j > 1) || (kk > 0));
            umma_commit(o_done);
            umma_commit(&kv_empty[st2]);
          }
        }
        if (!ok) break;
        umma_commit(o_item);
        g += d.ntiles;
        ++itn;
      }
    }
  } else {
    // ---------------- softmax and output: thread t = key t of a tile = head dim t ----------------
    const int t = threadIdx.x;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;  // this warp's TMEM lane quadrant
    const int G = p.G;
    const float sl2 = p.scale_log2;
    int g = 0, itn = 0;
    for (int it = blockIdx.x; it < num_items; it += gridDim.x) {
      const DecodeItem d = decode_item(p, it);
      // partial index of query head h of this item: ((s * Hq + kvh * G + h) * num_splits + split)
      const long long pbase = (static_cast<long long>(d.s) * p.Hq + d.kvh * G) * p.num_splits + d.split;
      const long long pstep = p.num_splits;
      if (d.ntiles == 0) {
        for (int h = 0; h < G; ++h) p.part_o[(pbase + h * pstep) * kHd + t] = 0.f;
        if (t < G) {
          p.part_ml[(pbase + t * pstep) * 2] = -INFINITY;
          p.part_ml[(pbase + t * pstep) * 2 + 1] = 0.f;
        }
        continue;
      }
      if (itn > 0) {
        const bool good = mbar_wait(q_empty, (itn - 1) & 1, p.status, kStatusTimeoutEpilogue);
        if (!named_bar_and(1, 128, good)) break;
      }
      for (int i = t; i < G * 16; i += 128) {
        const int r = i >> 4, u = i & 15;
        const uint4 v = *reinterpret_cast<const uint4*>(p.q + static_cast<long long>(d.s) * p.ldq +
                                                        (d.kvh * G + r) * kHd + u * 8);
        *reinterpret_cast<uint4*>(sQ + (u >> 3) * kQChunk + r * 128 + (((u & 7) ^ (r & 7)) << 4)) = v;
      }
      fence_async_shared();
      mbar_arrive(q_full);
      float m_used[GM], lsum[GM];
#pragma unroll
      for (int h = 0; h < GM; ++h) {
        m_used[h] = -INFINITY;
        lsum[h] = 0.f;
      }
      bool ok = true;
      for (int j = 0; j < d.ntiles; ++j) {
        const int gg = g + j;
        const int sb = gg & 1;
        const bool good = mbar_wait(&s_full[sb], (gg >> 1) & 1, p.status, kStatusTimeoutEpilogue);
        if (!named_bar_and(1, 128, good)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float x[NQ];
        {
          uint32_t v[NQ];
          if constexpr (NQ == 16)
            tmem_ld16(tS + sb * NQ + lane_off, v);
          else
            tmem_ld32(tS + sb * NQ + lane_off, v);
          tmem_wait_ld();
          const bool live = d.t0 + j * kTile + t < d.t1;
#pragma unroll
          for (int h = 0; h < NQ; ++h) x[h] = live ? __uint_as_float(v[h]) * sl2 : -INFINITY;
        }
        // per-head maximum of this tile: warp shuffle, then the four warps through shared memory
        float* red = s_max + sb * 4 * NQ;
#pragma unroll
        for (int h = 0; h < GM; ++h) {
          float m = x[h];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          if (lane == 0) red[warp * NQ + h] = m;
        }
        named_bar_sync(2, 128);
        bool any = false;
        float alpha[GM];
#pragma unroll
        for (int h = 0; h < GM; ++h) {
          alpha[h] = 1.f;
          const float tm = fmaxf(fmaxf(red[h], red[NQ + h]), fmaxf(red[2 * NQ + h], red[3 * NQ + h]));
          const float m_new = fmaxf(m_used[h], tm);
          if (m_new > m_used[h] + 8.0f) {
            alpha[h] = (m_used[h] == -INFINITY) ? 0.f : exp2f(m_used[h] - m_new);
            m_used[h] = m_new;
            lsum[h] *= alpha[h];
            any = true;
          }
        }
        // P^T rows (one per head) into P buffer sb; the PV that last read it (tile gg-2) completed
        // before S^T of this tile did
        uint8_t* prow = sP + sb * kQBytes + (t >> 6) * kQChunk + (t & 7) * 2;
        const int unit = (t & 63) >> 3;
#pragma unroll
        for (int h = 0; h < GM; ++h) {
          const float m_eff = (m_used[h] == -INFINITY) ? 0.f : m_used[h];
          const float pv = exp2f(x[h] - m_eff);
          lsum[h] += pv;
          *reinterpret_cast<__nv_bfloat16*>(prow + h * 128 + ((unit ^ (h & 7)) << 4)) = __float2bfloat16_rn(pv);
        }
        if (j > 0 && any) {
          // rescale O^T once the previous PV has landed (o_done is at most one completion behind)
          const bool good2 = mbar_wait(o_done, (gg - 1) & 1, p.status, kStatusTimeoutEpilogue);
          if (!named_bar_and(1, 128, good2)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t v[NQ];
          if constexpr (NQ == 16)
            tmem_ld16(tO + lane_off, v);
          else
            tmem_ld32(tO + lane_off, v);
          tmem_wait_ld();
#pragma unroll
          for (int h = 0; h < GM; ++h) v[h] = __float_as_uint(__uint_as_float(v[h]) * alpha[h]);
          if constexpr (NQ == 16)
            tmem_st16(tO + lane_off, v);
          else
            tmem_st32(tO + lane_off, v);
          tmem_wait_st();
        }
        fence_async_shared();
        tc_fence_before();
        mbar_arrive(&p_full[sb]);
      }
      if (!ok) break;
      const bool good = mbar_wait(o_item, itn & 1, p.status, kStatusTimeoutEpilogue);
      if (!named_bar_and(1, 128, good)) break;
      tc_fence_after();
      {
        uint32_t v[NQ];
        if constexpr (NQ == 16)
          tmem_ld16(tO + lane_off, v);
        else
          tmem_ld32(tO + lane_off, v);
        tmem_wait_ld();
#pragma unroll
        for (int h = 0; h < GM; ++h)
          if (h < G) p.part_o[(pbase + h * pstep) * kHd + t] = __uint_as_float(v[h]);
      }
#pragma unroll
      for (int h = 0; h < GM; ++h) {
        float l = lsum[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) s_sum[warp * NQ + h] = l;
      }
      named_bar_sync(2, 128);
#pragma unroll
      for (int h = 0; h < GM; ++h) {
        if (h < G && t == h) {
          p.part_ml[(pbase + h * pstep) * 2] = m_used[h] == -INFINITY ? -INFINITY : m_used[h] * kLn2;
          p.part_ml[(pbase + h * pstep) * 2 + 1] = (s_sum[h] + s_sum[NQ + h]) + (s_sum[2 * NQ + h] + s_sum[3 * NQ + h]);
        }
      }
      tc_fence_before();
      g += d.ntiles;
      ++itn;
    }
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tbase, 128);
  }
}

// ------------------------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------------------------
// 8 elementwise warps (two warpgroups over the column halves), 1 TMA warp, 1 MMA warp
constexpr int kBwdThreads = 320;

struct AttnBwdParams {
  const float* lse;    // [Hq, T]
  const float* delta;  // [Hq, T]
  float* dq_acc;       // [T, Hq*128] fp32, pre-zeroed
  float* dk_part;      // [T, Hq*128] fp32
  float* dv_part;      // [T, Hq*128] fp32
  const int* cu;
  int max_tiles, T, Hq, Hkv;
  float scale, scale_log2;
  int causal;
  int* status;
};

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const __grid_constant__ CUtensorMap tmDQ, const AttnBwdParams p) {
  const TileSeqHead at = tile_major(p.Hq);
  const int head = at.head;
  const int kt = at.tile;
  const int b = at.seq;
  const int seq_start = p.cu[b];
  const int len = p.cu[b + 1] - seq_start;
  if (kt * kTile >= len) return;
  const int ntiles = (len + kTile - 1) / kTile;
  const int q_first = p.causal ? kt : 0;
  const int nq = ntiles - q_first;
  const int kvh = head / (p.Hq / p.Hkv);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTileBytes;
  uint8_t* sQ = sV + kTileBytes;
  uint8_t* sDO = sQ + kTileBytes;
  uint8_t* sDQ = sDO + kTileBytes;  // dQ staging: one 32 x 32 fp32 tile (4 KB) per elementwise warp
  uint8_t* sDS = sDQ + kTileBytes;
  float* s_lse = reinterpret_cast<float*>(sDS + kTileBytes);
  float* s_delta = s_lse + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_delta + 128);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = bars + 2;
  uint64_t* s_full = bars + 3;
  uint64_t* ps_full = bars + 4;
  uint64_t* dq_full = bars + 5;
  uint64_t* dq_free = bars + 6;
  uint64_t* acc_done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(ps_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 256);
    mbar_init(acc_done, 1);
    fence_mbar_init();
  }
  if (warp == 9) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase;          // S^T, then P^T (bf16 pairs: queries 0-63 in cols 0-31, 64-127 in 64-95)
  const uint32_t tDP = tbase + 128;   // dP^T, then dQ
  const uint32_t tDV = tbase + 256;
  const uint32_t tDK = tbase + 384;

  if (warp == 8) {
    if (lane == 0) {
      const int ky = seq_start + kt * kTile;
      mbar_arrive_expect_tx(kv_full, 2 * kTileBytes);
      tma_load_2d(sK, &tmK, kv_full, kvh * kHd, ky);
      tma_load_2d(sK + kChunk, &tmK, kv_full, kvh * kHd + 64, ky);
      tma_load_2d(sV, &tmV, kv_full, kvh * kHd, ky);
      tma_load_2d(sV + kChunk, &tmV, kv_full, kvh * kHd + 64, ky);
      for (int i = 0; i < nq; ++i) {
        if (!mbar_wait(q_empty, (i & 1) ^ 1u, p.status, kStatusTimeoutProducer)) break;
        const int qy = seq_start + (q_first + i) * kTile;
        mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
        tma_load_2d(sQ, &tmQ, q_full, head * kHd, qy);
        tma_load_2d(sQ + kChunk, &tmQ, q_full, head * kHd + 64, qy);
        tma_load_2d(sDO, &tmDO, q_full, head * kHd, qy);
        tma_load_2d(sDO + kChunk, &tmDO, q_full, head * kHd + 64, qy);
      }
      mbar_wait(kv_full, 0, nullptr, 0, 20000000ull);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc_kk = make_idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_kmn = make_idesc_bf16_f32(128, 128, false, true);
      constexpr uint32_t idesc_mnmn = make_idesc_bf16_f32(128, 128, true, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
      const uint32_t ds_addr = smem_u32(sDS);
      bool ok = mbar_wait(kv_full, 0, p.status, kStatusTimeoutMma);
      for (int i = 0; i < nq && ok; ++i) {
        if (!mbar_wait(q_full, i & 1, p.status, kStatusTimeoutMma)) break;
        if (!mbar_wait(dq_free, (i & 1) ^ 1u, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_bf16(tS, desc_kmajor(k_addr, kk), desc_kmajor(q_addr, kk), idesc_kk, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_bf16(tDP, desc_kmajor(v_addr, kk), desc_kmajor(do_addr, kk), idesc_kk, kk > 0);
        umma_commit(s_full);
        if (!mbar_wait(ps_full, i & 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        // dV += P^T dO with P^T read from TMEM (the elementwise warps wrote it over S^T)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts(tDV, tS + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8), desc_mnmajor(do_addr, kk), idesc_kmn,
                       (i > 0) || (kk > 0));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tDK, desc_kmajor(ds_addr, kk), desc_mnmajor(q_addr, kk), idesc_kmn, (i > 0) || (kk > 0));
        // dQ = dS K into the dP^T columns (read out by the elementwise warps before the next dP^T)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tDP, desc_mnmajor(ds_addr, kk), desc_mnmajor(k_addr, kk), idesc_mnmn, kk > 0);
        umma_commit(dq_full);
        umma_commit(q_empty);
      }
      umma_commit(acc_done);
    }
  } else {
    // Two warpgroups share every 128 x 128 tile: warp w reads TMEM lanes 32*(w%4).. (its rows) and
    // handles the column half w/4, so each thread does 64 columns of the elementwise work.
    const int quad = warp & 3;
    const int half = warp >> 2;
    const int r = quad * 32 + lane;  // key row for S^T/dP^T/dK/dV; query row for dQ
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int k_pos = kt * kTile + r;
    const bool key_valid = k_pos < len;
    const int ldacc = p.Hq * kHd;
    bool ok = true;
    // lse / delta of the query tile, loaded one iteration ahead so the load latency hides behind MMAs
    auto load_stats = [&](int qt, float& l2, float& dl) {
      const int q_pos_t = qt * kTile + r;
      if (q_pos_t < len) {
        const long long idx = static_cast<long long>(head) * p.T + seq_start + q_pos_t;
        l2 = p.lse[idx] * kLog2e;
        dl = p.delta[idx];
      } else {
        l2 = INFINITY;
        dl = 0.f;
      }
    };
    float nxt_lse = 0.f, nxt_delta = 0.f;
    if (half == 0) load_stats(q_first, nxt_lse, nxt_delta);
    for (int i = 0; i < nq; ++i) {
      const int qt = q_first + i;
      named_bar_sync(1, 256);
      if (half == 0) {
        s_lse[r] = nxt_lse;
        s_delta[r] = nxt_delta;
      }
      named_bar_sync(1, 256);
      if (half == 0 && i + 1 < nq) load_stats(qt + 1, nxt_lse, nxt_delta);
      if (!mbar_wait(s_full, i & 1, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * half + cc;
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + c * 32 + lane_off, sv);
        tmem_ld32(tDP + c * 32 + lane_off, dv);
        tmem_wait_ld();  // both loads in flight together
        uint32_t pw[16], dw[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pv[2], dsv[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ql = c * 32 + e + h;
            const int q_pos = qt * kTile + ql;
            const bool valid = key_valid && q_pos < len && (!p.causal || q_pos >= k_pos);
            const float pr = valid ? exp2f(__uint_as_float(sv[e + h]) * p.scale_log2 - s_lse[ql]) : 0.f;
            pv[h] = pr;
            dsv[h] = pr * (__uint_as_float(dv[e + h]) - s_delta[ql]) * p.scale;
          }
          pw[e >> 1] = pack_bf16x2(pv[0], pv[1]);
          dw[e >> 1] = pack_bf16x2(dsv[0], dsv[1]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint32_t off = swz_offset(r, c * 4 + u);
          *reinterpret_cast<uint4*>(sDS + off) = make_uint4(dw[4 * u], dw[4 * u + 1], dw[4 * u + 2], dw[4 * u + 3]);
        }
        // P^T as bf16 pairs into columns [64*half + 16*cc, +16): S^T of this warp's first chunk, already read
        tmem_st16(tS + half * 64 + cc * 16 + lane_off, pw);
      }
      tmem_wait_st();
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(ps_full);
      if (!mbar_wait(dq_full, i & 1, p.status, kStatusTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        // dQ rows of this warp (32 queries) x its 64 columns, added into dq_acc by two TMA reduce-adds
        // of 32 x 32 fp32 tiles staged in shared memory. Rows past the sequence carry zeros (their P and
        // dS are zero), so the tile may overlap the next sequence; rows past T are clipped by TMA.
        uint8_t* buf = sDQ + warp * 4096;
        const int y = seq_start + qt * kTile + quad * 32;
        uint32_t v[32], v2[32];
        tmem_ld32(tDP + half * 64 + lane_off, v);
        tmem_ld32(tDP + half * 64 + 32 + lane_off, v2);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(dq_free);  // the accumulator is in registers: the next dP^T may overwrite it
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const uint32_t* src = cc ? v2 : v;
          if (lane == 0) bulk_wait_read<0>();  // this warp's previous tile has left the buffer
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(buf + swz128(lane, j)) =
                make_float4(__uint_as_float(src[4 * j]), __uint_as_float(src[4 * j + 1]),
                            __uint_as_float(src[4 * j + 2]), __uint_as_float(src[4 * j + 3]));
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&tmDQ, buf, head * kHd + half * 64 + cc * 32, y);
            bulk_commit();
          }
        }
      }
    }
    if (lane == 0) bulk_wait<0>();  // dQ reductions complete before the CTA exits
    if (ok && mbar_wait(acc_done, 0, p.status, kStatusTimeoutEpilogue)) {
      tc_fence_after();
      const long long rowoff = static_cast<long long>(seq_start + k_pos) * ldacc + head * kHd;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t v[32], w[32];
        tmem_ld32(tDV + c * 32 + lane_off, v);
        tmem_ld32(tDK + c * 32 + lane_off, w);
        tmem_wait_ld();
        if (key_valid) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            *reinterpret_cast<float4*>(p.dv_part + rowoff + c * 32 + g * 4) =
                make_float4(__uint_as_float(v[g * 4]), __uint_as_float(v[g * 4 + 1]), __uint_as_float(v[g * 4 + 2]),
                            __uint_as_float(v[g * 4 + 3]));
            *reinterpret_cast<float4*>(p.dk_part + rowoff + c * 32 + g * 4) =
                make_float4(__uint_as_float(w[g * 4]), __uint_as_float(w[g * 4 + 1]), __uint_as_float(w[g * 4 + 2]),
                            __uint_as_float(w[g * 4 + 3]));
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------------------------
// backward, pipelined over 64-query tiles
// ------------------------------------------------------------------------------------------------
// Same work split as attn_bwd_kernel (one CTA per 128-key tile, q head and sequence; warps 0-7
// elementwise, warp 8 TMA, warp 9 MMA), but query tiles are 64 rows, so the scores of two tiles fit in
// TMEM next to the dK / dV accumulators:
//   [0,64) [64,128)     S^T of the tiles in buffers 0 / 1 (P^T written back over them as bf16 pairs)
//   [128,192) [192,256) dP^T of the same tiles, then dQ^T = K^T dS^T of that tile
//   [256,384) dV        [384,512) dK
// The MMA warp issues dV, dK, dQ^T of tile i and then S^T, dP^T of tile i + 2 while the elementwise
// warps work on tile i + 1, so the exponentials and the dQ drain overlap tensor-core work instead of
// alternating with it. dQ^T has the head dims on the TMEM lanes; each elementwise warp transposes its
// 32 x 32 block through shared memory and adds it into dq_acc with a TMA reduce-add.
constexpr int kBwdQ = 64;
constexpr int kQChunk = kBwdQ * 128;         // one [64 rows x 64 bf16] 128B-swizzled chunk (8 KB)
constexpr int kQTileBytes = 2 * kQChunk;     // [64 rows x 128] bf16
constexpr int kDsBytes = 128 * kBwdQ * 2;    // dS^T [128 keys x 64 queries] bf16, one chunk
constexpr int kBwdQ64Smem = 2 * kTileBytes + 4 * kQTileBytes + 2 * kDsBytes + 8 * 4096 + 1024 + 1024 + 256;

// K-major descriptor of a [64 rows x 128 elems] tile (two 8 KB chunks); kk = 16-element K step.
ACCERL_DEVINL uint64_t desc_kmajor64(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * kQChunk + (kk & 3) * 32, 16, 1024);
}
// MN-major descriptor of the same tile when its 64 rows are the K dimension.
ACCERL_DEVINL uint64_t desc_mnmajor64(uint32_t base, int kk) {
  return make_sw128_desc(base + kk * 16 * 128, kQChunk, 1024);
}

__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_q64_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                        const __grid_constant__ CUtensorMap tmDQ, const AttnBwdParams p) {
  const TileSeqHead at = tile_major(p.Hq);
  const int head = at.head;
  const int kt = at.tile;
  const int b = at.seq;
  const int seq_start = p.cu[b];
  const int len = p.cu[b + 1] - seq_start;
  if (kt * kTile >= len) return;
  const int ntiles = (len + kBwdQ - 1) / kBwdQ;
  const int q_first = p.causal ? kt * (kTile / kBwdQ) : 0;
  const int nq = ntiles - q_first;
  const int kvh = head / (p.Hq / p.Hkv);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + kTileBytes;
  uint8_t* sQ = sV + kTileBytes;          // [2] x kQTileBytes
  uint8_t* sDO = sQ + 2 * kQTileBytes;    // [2]
  uint8_t* sDS = sDO + 2 * kQTileBytes;   // [2] x kDsBytes
  uint8_t* sDQ = sDS + 2 * kDsBytes;      // 8 x 4 KB dQ staging
  float* s_lse = reinterpret_cast<float*>(sDQ + 8 * 4096);  // [2][64]
  float* s_delta = s_lse + 2 * kBwdQ;                        // [2][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(s_delta + 2 * kBwdQ);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;    // [2]
  uint64_t* q_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* ps_full = bars + 7;   // [2]
  uint64_t* dq_full = bars + 9;   // [2] dQ^T of the buffer's tile is in TMEM (its dS^T smem is free again)
  uint64_t* dq_free = bars + 11;  // [2]
  uint64_t* acc_done = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&q_full[x], 1);
      mbar_init(&q_empty[x], 1);
      mbar_init(&s_full[x], 1);
      mbar_init(&ps_full[x], 256);
      mbar_init(&dq_full[x], 1);
      mbar_init(&dq_free[x], 256);
    }
    mbar_init(acc_done, 1);
    fence_mbar_init();
  }
  if (warp == 9) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tS = tbase;          // + 64 * buffer
  const uint32_t tDP = tbase + 128;   // + 64 * buffer
  const uint32_t tDV = tbase + 256;
  const uint32_t tDK = tbase + 384;

  if (warp == 8) {
    if (lane == 0) {
      const int ky = seq_start + kt * kTile;
      mbar_arrive_expect_tx(kv_full, 2 * kTileBytes);
      tma_load_2d(sK, &tmK, kv_full, kvh * kHd, ky);
      tma_load_2d(sK + kChunk, &tmK, kv_full, kvh * kHd + 64, ky);
      tma_load_2d(sV, &tmV, kv_full, kvh * kHd, ky);
      tma_load_2d(sV + kChunk, &tmV, kv_full, kvh * kHd + 64, ky);
      for (int i = 0; i < nq; ++i) {
        const int qb = i & 1;
        if (!mbar_wait(&q_empty[qb], ((i >> 1) & 1) ^ 1u, p.status, kStatusTimeoutProducer)) break;
        const int qy = seq_start + (q_first + i) * kBwdQ;
        uint8_t* q_dst = sQ + qb * kQTileBytes;
        uint8_t* do_dst = sDO + qb * kQTileBytes;
        mbar_arrive_expect_tx(&q_full[qb], 2 * kQTileBytes);
        tma_load_2d(q_dst, &tmQ, &q_full[qb], head * kHd, qy);
        tma_load_2d(q_dst + kQChunk, &tmQ, &q_full[qb], head * kHd + 64, qy);
        tma_load_2d(do_dst, &tmDO, &q_full[qb], head * kHd, qy);
        tma_load_2d(do_dst + kQChunk, &tmDO, &q_full[qb], head * kHd + 64, qy);
      }
      mbar_wait(kv_full, 0, nullptr, 0, 20000000ull);
    }
  } else if (warp == 9) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, kBwdQ, false, false);  // S^T, dP^T
      constexpr uint32_t idesc_kmn = make_idesc_bf16_f32(128, 128, false, true);   // dV (TS), dK
      constexpr uint32_t idesc_q = make_idesc_bf16_f32(128, kBwdQ, true, true);    // dQ^T = K^T dS^T
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      bool ok = mbar_wait(kv_full, 0, p.status, kStatusTimeoutMma);
      // S^T = K Q^T and dP^T = V dO^T of tile i into buffer i & 1
      auto issue_scores = [&](int i) -> bool {
        const int qb = i & 1;
        if (!mbar_wait(&q_full[qb], (i >> 1) & 1, p.status, kStatusTimeoutMma)) return false;
        if (i >= 2 && !mbar_wait(&dq_free[qb], ((i - 2) >> 1) & 1, p.status, kStatusTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + qb * kQTileBytes), do_addr = smem_u32(sDO + qb * kQTileBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tS + qb * 64, desc_kmajor(k_addr, kk), desc_kmajor64(q_addr, kk), idesc_s, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tDP + qb * 64, desc_kmajor(v_addr, kk), desc_kmajor64(do_addr, kk), idesc_s, kk > 0);
        umma_commit(&s_full[qb]);
        return true;
      };
      if (ok) ok = issue_scores(0);
      if (ok && nq > 1) ok = issue_scores(1);
      for (int i = 0; i < nq && ok; ++i) {
        const int qb = i & 1;
        if (!mbar_wait(&ps_full[qb], (i >> 1) & 1, p.status, kStatusTimeoutMma)) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + qb * kQTileBytes), do_addr = smem_u32(sDO + qb * kQTileBytes);
        const uint32_t ds_addr = smem_u32(sDS + qb * kDsBytes);
        // dV += P^T dO with P^T from TMEM: queries 0-31 in columns [0,16), 32-63 in [32,48) of the buffer
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16_ts(tDV, tS + qb * 64 + (kk < 2 ? kk * 8 : 32 + (kk - 2) * 8), desc_mnmajor64(do_addr, kk),
                       idesc_kmn, (i > 0) || (kk > 0));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tDK, make_sw128_desc(ds_addr + kk * 32, 16, 1024), desc_mnmajor64(q_addr, kk), idesc_kmn,
                    (i > 0) || (kk > 0));
        umma_commit(&q_empty[qb]);
        // dQ^T = K^T dS^T over the dP^T columns of this buffer (drained before its next dP^T)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tDP + qb * 64, desc_mnmajor(k_addr, kk), make_sw128_desc(ds_addr + kk * 16 * 128, kChunk, 1024),
                    idesc_q, kk > 0);
        umma_commit(&dq_full[qb]);
        if (i + 2 < nq) ok = issue_scores(i + 2);
      }
      umma_commit(acc_done);
    }
  } else {
    const int quad = warp & 3;
    const int half = warp >> 2;      // query columns [32 * half, 32 * half + 32) of a tile
    const int r = quad * 32 + lane;  // key row of S^T / dP^T / dK / dV; head dim of dQ^T
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int k_pos = kt * kTile + r;
    const bool key_valid = k_pos < len;
    const int ldacc = p.Hq * kHd;
    const int tid = threadIdx.x;  // 0..255
    bool ok = true;
    auto load_stats = [&](int i) {  // lse (log2 units) / delta of tile i's queries into buffer i & 1
      if (tid < kBwdQ) {
        const int q_pos = (q_first + i) * kBwdQ + tid;
        float l2 = INFINITY, dl = 0.f;
        if (q_pos < len) {
          const long long idx = static_cast<long long>(head) * p.T + seq_start + q_pos;
          l2 = p.lse[idx] * kLog2e;
          dl = p.delta[idx];
        }
        s_lse[(i & 1) * kBwdQ + tid] = l2;
        s_delta[(i & 1) * kBwdQ + tid] = dl;
      }
    };
    // add dQ^T of tile j (TMEM lanes = head dims, columns = queries) into dq_acc
    auto drain_dq = [&](int j) -> bool {
      const int qb = j & 1;
      if (!mbar_wait(&dq_full[qb], (j >> 1) & 1, p.status, kStatusTimeoutEpilogue)) return false;
      tc_fence_after();
      uint32_t v[32];
      tmem_ld32(tDP + qb * 64 + half * 32 + lane_off, v);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&dq_free[qb]);  // the values are in registers: the next scores may overwrite them
      uint8_t* buf = sDQ + warp * 4096;
      if (lane == 0) bulk_wait_read<0>();  // this warp's previous tile has left the buffer
      __syncwarp();
      // transpose: row = query (32 of them), column = this lane's head dim
#pragma unroll
      for (int c = 0; c < 32; ++c)
        *reinterpret_cast<float*>(buf + c * 128 + ((((lane >> 2) ^ (c & 7)) & 7) << 4) + (lane & 3) * 4) =
            __uint_as_float(v[c]);
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tmDQ, buf, head * kHd + quad * 32, seq_start + (q_first + j) * kBwdQ + half * 32);
        bulk_commit();
      }
      return true;
    };
    load_stats(0);
    named_bar_sync(1, 256);
    // A failed (timed-out) wait clears ok; every thread still reaches the barrier at the end of the
    // iteration, whose AND-reduction makes all of them leave together.
    for (int i = 0; i < nq; ++i) {
      const int qb = i & 1;
      const int qt = q_first + i;
      if (i + 1 < nq) load_stats(i + 1);
      if (ok) ok = mbar_wait(&s_full[qb], (i >> 1) & 1, p.status, kStatusTimeoutEpilogue);
      if (ok) {
        tc_fence_after();
        uint32_t sv[32], dv[32];
        tmem_ld32(tS + qb * 64 + half * 32 + lane_off, sv);
        tmem_ld32(tDP + qb * 64 + half * 32 + lane_off, dv);
        tmem_wait_ld();
        const float* lse2 = s_lse + qb * kBwdQ + half * 32;
        const float* dlt = s_delta + qb * kBwdQ + half * 32;
        uint32_t pw[16], dw[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pv[2], dsv[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int q_pos = qt * kBwdQ + half * 32 + e + h;
            const bool valid = key_valid && q_pos < len && (!p.causal || q_pos >= k_pos);
            const float pr = valid ? exp2f(__uint_as_float(sv[e + h]) * p.scale_log2 - lse2[e + h]) : 0.f;
            pv[h] = pr;
            dsv[h] = pr * (__uint_as_float(dv[e + h]) - dlt[e + h]) * p.scale;
          }
          pw[e >> 1] = pack_bf16x2(pv[0], pv[1]);
          dw[e >> 1] = pack_bf16x2(dsv[0], dsv[1]);
        }
        // dS^T buffer qb was last read by the dK / dQ^T MMAs of tile i - 2
        if (i >= 2) ok = mbar_wait(&dq_full[qb], ((i - 2) >> 1) & 1, p.status, kStatusTimeoutEpilogue);
        if (ok) {
          uint8_t* ds = sDS + qb * kDsBytes;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint32_t off = r * 128 + ((((half * 4 + u) ^ (r & 7)) & 7) << 4);
            *reinterpret_cast<uint4*>(ds + off) = make_uint4(dw[4 * u], dw[4 * u + 1], dw[4 * u + 2], dw[4 * u + 3]);
          }
          tmem_st16(tS + qb * 64 + half * 32 + lane_off, pw);  // P^T over this thread's own S^T columns
          tmem_wait_st();
          fence_async_shared();
          tc_fence_before();
          mbar_arrive(&ps_full[qb]);
          if (i >= 1) ok = drain_dq(i - 1);
        }
      }
      // next tile's stats are in; this tile's stats buffer may be refilled
      if (!named_bar_and(1, 256, ok)) {
        ok = false;
        break;
      }
    }
    if (ok) ok = drain_dq(nq - 1);
    if (lane == 0) bulk_wait<0>();  // dQ reductions complete before the CTA exits
    if (ok && mbar_wait(acc_done, 0, p.status, kStatusTimeoutEpilogue)) {
      tc_fence_after();
      const long long rowoff = static_cast<long long>(seq_start + k_pos) * ldacc + head * kHd;
#pragma unroll 1
      for (int c = 2 * half; c < 2 * half + 2; ++c) {
        uint32_t v[32], w[32];
        tmem_ld32(tDV + c * 32 + lane_off, v);
        tmem_ld32(tDK + c * 32 + lane_off, w);
        tmem_wait_ld();
        if (key_valid) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            *reinterpret_cast<float4*>(p.dv_part + rowoff + c * 32 + g * 4) =
                make_float4(__uint_as_float(v[g * 4]), __uint_as_float(v[g * 4 + 1]), __uint_as_float(v[g * 4 + 2]),
                            __uint_as_float(v[g * 4 + 3]));
            *reinterpret_cast<float4*>(p.dk_part + rowoff + c * 32 + g * 4) =
                make_float4(__uint_as_float(w[g * 4]), __uint_as_float(w[g * 4 + 1]), __uint_as_float(w[g * 4 + 2]),
                            __uint_as_float(w[g * 4 + 3]));
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// delta[h, t] = sum_d dO[t, h, d] * O[t, h, d]; one warp per (t, h).
__global__ void attn_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                  float* __restrict__ delta, int T, int Hq, long long ldo, long long lddo) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<long long>(T) * Hq) return;
  const int t = static_cast<int>(w / Hq);
  const int h = static_cast<int>(w % Hq);
  const uint2 a = *reinterpret_cast<const uint2*>(o + t * ldo + h * kHd + lane * 4);
  const uint2 bb = *reinterpret_cast<const uint2*>(dout + t * lddo + h * kHd + lane * 4);
  const float2 a0 = unpack_bf16x2(a.x), a1 = unpack_bf16x2(a.y), b0 = unpack_bf16x2(bb.x), b1 = unpack_bf16x2(bb.y);
  float s = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
  s = warp_sum(s);
  if (lane == 0) delta[static_cast<long long>(h) * T + t] = s;
}

// dq (bf16, strided) from the fp32 accumulator; dk/dv from per-q-head partials summed over the GQA group.
// Store 4 dims of each half of a head (d and d + 64) as bf16, rotated by the inverse RoPE when asked
// (inputs rounded to bf16 first, as the separate RoPE kernel sees them).
ACCERL_DEVINL void store_rotated(float4 lo, float4 hi, const float (&c)[4], const float (&sn)[4], bool rotate,
                                 __nv_bfloat16* dst) {
  const float a[4] = {lo.x, lo.y, lo.z, lo.w}, b[4] = {hi.x, hi.y, hi.z, hi.w};
  float x[4], y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (rotate) {
      const float a16 = __bfloat162float(__float2bfloat16(a[i])), b16 = __bfloat162float(__float2bfloat16(b[i]));
      x[i] = a16 * c[i] - b16 * sn[i];
      y[i] = b16 * c[i] + a16 * sn[i];
    } else {
      x[i] = a[i];
      y[i] = b[i];
    }
  }
  uint2 o1, o2;
  o1.x = pack_bf16x2(x[0], x[1]);
  o1.y = pack_bf16x2(x[2], x[3]);
  o2.x = pack_bf16x2(y[0], y[1]);
  o2.y = pack_bf16x2(y[2], y[3]);
  *reinterpret_cast<uint2*>(dst) = o1;
  *reinterpret_cast<uint2*>(dst + kHd / 2) = o2;
}

// dq / dk / dv to bf16 (dk, dv summed over the query heads of each KV group), optionally with the
// inverse rotary rotation of dq and dk fused in (pos != nullptr). One thread per (token, 4 of the
// first 64 head dims): it computes the rotation coefficients once and walks every head, handling
// the 4 matching dims of the second half (d + 64), the pair that the rotate-half convention mixes.
__global__ void attn_bwd_finalize_kernel(const float* __restrict__ dq_acc, const float* __restrict__ dk_part,
                                         const float* __restrict__ dv_part, __nv_bfloat16* __restrict__ dq,
                                         __nv_bfloat16* __restrict__ dk, __nv_bfloat16* __restrict__ dv, int T, int Hq,
                                         int Hkv, long long lddq, long long lddk, long long lddv,
                                         const long long* __restrict__ pos, float log2_theta) {
  constexpr int kHalf = kHd / 2;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;  // over T * kHalf/4
  if (idx >= static_cast<long long>(T) * (kHalf / 4)) return;
  const int t = static_cast<int>(idx / (kHalf / 4));
  const int d = static_cast<int>(idx % (kHalf / 4)) * 4;  // 0..60
  float c[4] = {1.f, 1.f, 1.f, 1.f}, sn[4] = {0.f, 0.f, 0.f, 0.f};
  const bool rot = pos != nullptr;
  if (rot) {
    const float p = static_cast<float>(pos[t]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rope_cos_sin(p, d + i, kHd, log2_theta, c[i], sn[i]);
      sn[i] = -sn[i];  // inverse rotation
    }
  }
  const long long row = static_cast<long long>(t) * Hq * kHd;
  const int group = Hq / Hkv;
  for (int h = 0; h < Hq; ++h) {
    const float4 lo = *reinterpret_cast<const float4*>(dq_acc + row + h * kHd + d);
    const float4 hi = *reinterpret_cast<const float4*>(dq_acc + row + h * kHd + d + kHalf);
    store_rotated(lo, hi, c, sn, rot, dq + t * lddq + h * kHd + d);
  }
  for (int kvh = 0; kvh < Hkv; ++kvh) {
    float4 k0 = make_float4(0, 0, 0, 0), k1 = k0, v0 = k0, v1 = k0;
    for (int g = 0; g < group; ++g) {
      const long long off = row + (kvh * group + g) * kHd + d;
      const float4 a0 = *reinterpret_cast<const float4*>(dk_part + off);
      const float4 a1 = *reinterpret_cast<const float4*>(dk_part + off + kHalf);
      const float4 b0 = *reinterpret_cast<const float4*>(dv_part + off);
      const float4 b1 = *reinterpret_cast<const float4*>(dv_part + off + kHalf);
      k0.x += a0.x; k0.y += a0.y; k0.z += a0.z; k0.w += a0.w;
      k1.x += a1.x; k1.y += a1.y; k1.z += a1.z; k1.w += a1.w;
      v0.x += b0.x; v0.y += b0.y; v0.z += b0.z; v0.w += b0.w;
      v1.x += b1.x; v1.y += b1.y; v1.z += b1.z; v1.w += b1.w;
    }
    store_rotated(k0, k1, c, sn, rot, dk + t * lddk + kvh * kHd + d);
    store_rotated(v0, v1, c, sn, false, dv + t * lddv + kvh * kHd + d);
  }
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// Tile map over a [T, width] bf16 matrix with a 64-column x 128-row box, 128B swizzle.
// bf16 [T, width] map whose boxes are `rows` high (one page of a paged KV cache)
bool attn_map_rows(CUtensorMap* m, const void* ptr, int T, int width, long long ld, int rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(rows)};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool attn_map(CUtensorMap* m, const void* ptr, int T, int width, long long ld) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// fp32 [T, width] map with 32 x 32 boxes (128-byte rows, 128B swizzle) for the dQ reduce-adds
bool attn_map_f32(CUtensorMap* m, const float* ptr, int T, int width) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(width) * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kFwdSmem = 5 * kTileBytes + 1024 + 256;

// Which backward kernel runs: the 64-query pipelined one (default; 2-3 % faster on 2 x 8192 and
// 8 x 2048 tokens with 12 / 2 heads) or, with ACCERL_ATTN_BWD=q128, the 128-query one. Read once per
// process.
bool attn_bwd_q64_selected() {
  static const bool q64 = [] {
    const char* e = std::getenv("ACCERL_ATTN_BWD");
    return e == nullptr || std::string(e) != "q128";
  }();
  return q64;
}
constexpr int kBwdSmem = 6 * kTileBytes + 1024 + 1024 + 256;

}  // namespace
}  // namespace accerl

using namespace accerl;

// Paged keys: pass block_table ([num_seqs, max_blocks] int32) with k / v the layer's caches
// ([num_blocks, block_size, Hkv, 128], total_k = num_blocks * block_size rows); cu_seqlens_k then gives
// each sequence's key count (its keys are positions 0..len_k-1 of its pages).
extern "C" int accerl_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, const int* cu_seqlens,
                               const int* cu_seqlens_k, int num_seqs, int max_seqlen, int total_tokens, int total_k,
                               int Hq, int Hkv, long long ldq, long long ldk, long long ldv, long long ldo, float scale,
                               int causal, int* status, const int* block_table, int max_blocks, int block_size,
                               cudaStream_t s) {
  if (num_seqs <= 0 || total_tokens <= 0) return 0;
  if (Hq % Hkv) return -1;
  if ((ldq | ldk | ldv | ldo) & 7) return -2;
  if (block_table && (block_size < 8 || block_size > kTile || kTile % block_size || !cu_seqlens_k)) return -4;
  CUtensorMap mq, mk, mv;
  if (!attn_map(&mq, q, total_tokens, Hq * kHd, ldq)) return -3;
  if (block_table) {
    if (!attn_map_rows(&mk, k, total_k, Hkv * kHd, ldk, block_size) ||
        !attn_map_rows(&mv, v, total_k, Hkv * kHd, ldv, block_size))
      return -3;
  } else if (!attn_map(&mk, k, total_k, Hkv * kHd, ldk) || !attn_map(&mv, v, total_k, Hkv * kHd, ldv)) {
    return -3;
  }
  if (cudaError_t e = smem_attr_once<attn_fwd_kernel>(kFwdSmem); e != cudaSuccess) return (int)e;
  AttnFwdParams p;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  p.cu = cu_seqlens;
  p.cu_k = cu_seqlens_k ? cu_seqlens_k : cu_seqlens;
  p.max_tiles = (max_seqlen + kTile - 1) / kTile;
  p.T = total_tokens;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.ldo = ldo;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.status = status;
  p.block_table = block_table;
  p.max_blocks = max_blocks;
  p.block_size = block_size;
  dim3 grid(p.max_tiles * Hq, num_seqs);
  attn_fwd_kernel<<<grid, 192, kFwdSmem, s>>>(mq, mk, mv, p);
  return (int)cudaGetLastError();
}

extern "C" int accerl_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                               const float* lse, float* delta, float* dq_acc, void* dq, void* dk, void* dv,
                               const int* cu_seqlens, int num_seqs, int max_seqlen, int total_tokens, int Hq, int Hkv,
                               long long ldq, long long ldk, long long ldv, long long ldo, long long lddo,
                               long long lddq, long long lddk, long long lddv, float scale, int causal, int* status,
                               const long long* rope_pos, float rope_theta, cudaStream_t s) {
  if (num_seqs <= 0 || total_tokens <= 0) return 0;
  if (rope_pos && !(rope_theta > 0.f)) return -4;
  if (Hq % Hkv) return -1;
  if ((ldq | ldk | ldv | ldo | lddo | lddq | lddk | lddv) & 7) return -2;
  CUtensorMap mq, mk, mv, mdo;
  if (!attn_map(&mq, q, total_tokens, Hq * kHd, ldq) || !attn_map(&mk, k, total_tokens, Hkv * kHd, ldk) ||
      !attn_map(&mv, v, total_tokens, Hkv * kHd, ldv) || !attn_map(&mdo, dout, total_tokens, Hq * kHd, lddo))
    return -3;
  const bool q64 = attn_bwd_q64_selected();
  CUtensorMap mq64, mdo64;
  if (q64) {
    if (!attn_map_rows(&mq64, q, total_tokens, Hq * kHd, ldq, kBwdQ) ||
        !attn_map_rows(&mdo64, dout, total_tokens, Hq * kHd, lddo, kBwdQ))
      return -3;
    if (cudaError_t e = smem_attr_once<attn_bwd_q64_kernel>(kBwdQ64Smem); e != cudaSuccess) return (int)e;
  } else if (cudaError_t e = smem_attr_once<attn_bwd_kernel>(kBwdSmem); e != cudaSuccess) {
    return (int)e;
  }
  const long long nwarps = (long long)total_tokens * Hq;
  attn_delta_kernel<<<(unsigned)((nwarps * 32 + 255) / 256), 256, 0, s>>>(
      (const __nv_bfloat16*)o, (const __nv_bfloat16*)dout, delta, total_tokens, Hq, ldo, lddo);
  const long long acc_elems = (long long)total_tokens * Hq * kHd;
  // dq_acc holds [dq | dk_part | dv_part] contiguously (3 * acc_elems floats); only dq needs zeros.
  cudaMemsetAsync(dq_acc, 0, acc_elems * sizeof(float), s);
  CUtensorMap mdq;
  if (!attn_map_f32(&mdq, dq_acc, total_tokens, Hq * kHd)) return -3;
  AttnBwdParams p;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk_part = dq_acc + acc_elems;
  p.dv_part = dq_acc + 2 * acc_elems;
  p.cu = cu_seqlens;
  p.max_tiles = (max_seqlen + kTile - 1) / kTile;
  p.T = total_tokens;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.scale = scale;
  p.scale_log2 = scale * kLog2e;
  p.causal = causal;
  p.status = status;
  dim3 grid(p.max_tiles * Hq, num_seqs);
  if (q64)
    attn_bwd_q64_kernel<<<grid, kBwdThreads, kBwdQ64Smem, s>>>(mq64, mk, mv, mdo64, mdq, p);
  else
    attn_bwd_kernel<<<grid, kBwdThreads, kBwdSmem, s>>>(mq, mk, mv, mdo, mdq, p);
  const long long nthr = (long long)total_tokens * (kHd / 8);  // one thread per (token, 4 dims of a half)
  attn_bwd_finalize_kernel<<<(unsigned)((nthr + 255) / 256), 256, 0, s>>>(
      dq_acc, p.dk_part, p.dv_part, (__nv_bfloat16*)dq, (__nv_bfloat16*)dk, (__nv_bfloat16*)dv, total_tokens, Hq, Hkv,
      lddq, lddk, lddv, rope_pos, rope_theta > 0.f ? log2f(rope_theta) : 0.f);
  return (int)cudaGetLastError();
}

// Tensor-core paged decode (see paged_decode_tc_kernel). k_cache / v_cache: [num_blocks, block_size,
// Hkv, 128] bf16 of one layer. Writes the per-split partials that accerl_paged_decode_merge combines.
// Returns -2 when the shape is not supported by this kernel (the caller uses the CUDA-core kernel).
// Tensor maps and parameters shared by both tensor-core decode kernels; returns 0 or an error code
// (-1 bad head counts, -2 shape the kernels do not cover, -3 tensor-map failure).
static int decode_tc_setup(const void* q, long long ldq, const void* k_cache, const void* v_cache, int num_blocks,
                           const int* block_table, int max_blocks, const int* seq_lens, float* part_o,
                           float* part_ml, int num_seqs, int Hq, int Hkv, int block_size, int num_splits,
                           float scale, int* status, CUtensorMap* mk, CUtensorMap* mv, DecodeTcParams* p) {
  if (Hq % Hkv) return -1;
  const int G = Hq / Hkv;
  if (G > 32 || block_size < 8 || block_size > kTile || kTile % block_size || (ldq & 7)) return -2;
  auto fn = encode_fn();
  if (!fn) return -3;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(Hkv) * kHd, static_cast<cuuint64_t>(num_blocks) * block_size};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(Hkv) * kHd * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(block_size)};
  cuuint32_t es[2] = {1, 1};
  if (fn(mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(k_cache), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      fn(mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(v_cache), dims, strides, box, es,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -3;
  p->q = reinterpret_cast<const __nv_bfloat16*>(q);
  p->ldq = ldq;
  p->block_table = block_table;
  p->max_blocks = max_blocks;
  p->seq_lens = seq_lens;
  p->num_seqs = num_seqs;
  p->Hq = Hq;
  p->Hkv = Hkv;
  p->G = G;
  p->block_size = block_size;
  p->num_splits = num_splits;
  p->num_blocks = num_blocks;
  p->scale_log2 = scale * kLog2e;
  p->part_o = part_o;
  p->part_ml = part_ml;
  p->status = status;
  return 0;
}

static int num_sms() { return device_sm_count(); }

extern "C" int accerl_paged_decode_tc(const void* q, long long ldq, const void* k_cache, const void* v_cache,
                                      int num_blocks, const int* block_table, int max_blocks, const int* seq_lens,
                                      float* part_o, float* part_ml, int num_seqs, int Hq, int Hkv, int block_size,
                                      int num_splits, float scale, int* status, cudaStream_t s) {
  if (num_seqs == 0) return 0;
  CUtensorMap mk, mv;
  DecodeTcParams p;
  const int rc = decode_tc_setup(q, ldq, k_cache, v_cache, num_blocks, block_table, max_blocks, seq_lens, part_o,
                                 part_ml, num_seqs, Hq, Hkv, block_size, num_splits, scale, status, &mk, &mv, &p);
  if (rc) return rc;
  constexpr int smem = (1 + 2 * kDecStages) * kTileBytes + 1024 + 256;
  static_assert(smem <= 232448, "shared memory per CTA");
  if (cudaError_t e = smem_attr_once<paged_decode_tc_kernel>(smem); e != cudaSuccess) return (int)e;
  const int items = num_seqs * Hkv * num_splits;
  paged_decode_tc_kernel<<<std::min(items, num_sms()), 192, smem, s>>>(mk, mv, p);
  return (int)cudaGetLastError();
}

template <int NQ, int GM>
static int launch_decode_tq(const CUtensorMap& mk, const CUtensorMap& mv, const DecodeTcParams& p, int items,
                            cudaStream_t s) {
  // K/V ring + Q + two P buffers + per-warp maxima (two tiles) and sums + barriers, 1 KB alignment slack
  constexpr int smem = 2 * kDecStages * kTileBytes + 3 * NQ * 256 + 3 * 4 * NQ * 4 + 32 * 8 + 1024;
  static_assert(smem + 64 <= 232448, "shared memory per CTA");
  if (cudaError_t e = smem_attr_once<paged_decode_tq_kernel<NQ, GM>>(smem); e != cudaSuccess) return (int)e;
  paged_decode_tq_kernel<NQ, GM><<<std::min(items, num_sms()), 192, smem, s>>>(mk, mv, p);
  return (int)cudaGetLastError();
}

extern "C" int accerl_paged_decode_tq(const void* q, long long ldq, const void* k_cache, const void* v_cache,
                                      int num_blocks, const int* block_table, int max_blocks, const int* seq_lens,
                                      float* part_o, float* part_ml, int num_seqs, int Hq, int Hkv, int block_size,
                                      int num_splits, float scale, int* status, cudaStream_t s) {
  if (num_seqs == 0) return 0;
  CUtensorMap mk, mv;
  DecodeTcParams p;
  const int rc = decode_tc_setup(q, ldq, k_cache, v_cache, num_blocks, block_table, max_blocks, seq_lens, part_o,
                                 part_ml, num_seqs, Hq, Hkv, block_size, num_splits, scale, status, &mk, &mv, &p);
  if (rc) return rc;
  const int items = num_seqs * Hkv * num_splits;
  if (p.G == 1) return launch_decode_tq<16, 1>(mk, mv, p, items, s);
  if (p.G == 2) return launch_decode_tq<16, 2>(mk, mv, p, items, s);
  if (p.G <= 4) return launch_decode_tq<16, 4>(mk, mv, p, items, s);
  if (p.G <= 8) return launch_decode_tq<16, 8>(mk, mv, p, items, s);
  if (p.G <= 16) return launch_decode_tq<16, 16>(mk, mv, p, items, s);
  return launch_decode_tq<32, 32>(mk, mv, p, items, s);
}

ACCERL_DEBUG_EXPORT(attention)
