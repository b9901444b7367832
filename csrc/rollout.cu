// Rollout-engine kernels (sm_100a):
//  * paged-KV decode attention, split over the sequence ("flash decoding") and packed over the q
//    heads of one GQA group so each K/V row is read once per group; partial (o, m, l) per split are
//    merged by a second kernel.
//  * KV-cache write of freshly projected K/V rows into their paged slots.
// The token sampler is in sampler.cu.
// Cache layout: k_cache/v_cache [num_blocks, block_size, Hkv, 128] bf16.
#include "common.cuh"

namespace accerl {

constexpr int kDHead = 128;
constexpr int kMaxGroup = 16;

// out[s, h, :] = softmax(q . K^T * scale) V over the first seq_lens[s] cached tokens.
// grid (num_seqs, Hkv, num_splits), 4 warps; lanes map to tokens for Q.K and to head dims for P.V.
template <int G>
__global__ void __launch_bounds__(128) paged_decode_kernel(const __nv_bfloat16* __restrict__ q, long long ldq,
                                                          const __nv_bfloat16* __restrict__ k_cache,
                                                          const __nv_bfloat16* __restrict__ v_cache,
                                                          const int* __restrict__ block_table, int max_blocks,
                                                          const int* __restrict__ seq_lens, int block_size, int Hkv,
                                                          int num_splits, float scale, float* __restrict__ part_o,
                                                          float* __restrict__ part_ml) {
  const int s = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = seq_lens[s];
  const int per_split = (((len + num_splits - 1) / num_splits) + 31) & ~31;
  const int t0 = split * per_split;
  const int t1 = min(len, t0 + per_split);
  __shared__ float q_s[G][kDHead];
  __shared__ float p_s[4][G][32];
  __shared__ float red_m[4][G], red_l[4][G];
  __shared__ float red_o[4][G][kDHead];
  const int Hq = Hkv * G;
  for (int i = threadIdx.x; i < G * kDHead; i += blockDim.x) {
    const int h = i / kDHead, d = i % kDHead;
    q_s[h][d] = __bfloat162float(q[static_cast<long long>(s) * ldq + (kvh * G + h) * kDHead + d]) * scale;
  }
  __syncthreads();
  float m[G], l[G], acc[G][4];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[h][i] = 0.f;
  }
  const long long row_stride = static_cast<long long>(Hkv) * kDHead;
  for (int base = t0 + warp * 32; base < t1; base += 4 * 32) {
    const int tok = base + lane;
    const bool valid = tok < t1;
    long long off = 0;
    if (valid) {
      const int blk = block_table[static_cast<long long>(s) * max_blocks + tok / block_size];
      off = (static_cast<long long>(blk) * block_size + tok % block_size) * row_stride + kvh * kDHead;
    }
    float sc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) sc[h] = 0.f;
    if (valid) {
      const uint4* kr = reinterpret_cast<const uint4*>(k_cache + off);
      uint4 krow[kDHead / 8];  // the whole 256-byte K row in flight at once
#pragma unroll
      for (int c = 0; c < kDHead / 8; ++c) krow[c] = kr[c];
#pragma unroll
      for (int c = 0; c < kDHead / 8; ++c) {
        const uint4 kv = krow[c];
        const uint32_t kw[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = unpack_bf16x2(kw[i]);
#pragma unroll
          for (int h = 0; h < G; ++h) sc[h] += f.x * q_s[h][c * 8 + 2 * i] + f.y * q_s[h][c * 8 + 2 * i + 1];
        }
      }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const float x = valid ? sc[h] : -INFINITY;
      const float cm = warp_max(x);
      const float mn = fmaxf(m[h], cm);
      const float a = (m[h] == -INFINITY) ? 0.f : __expf(m[h] - mn);
      const float pv = valid ? __expf(x - mn) : 0.f;
      l[h] = l[h] * a + warp_sum(pv);
      m[h] = mn;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[h][i] *= a;
      p_s[warp][h][lane] = pv;
    }
    __syncwarp();
    // P.V: lanes own 4 head dims; 8 V rows are loaded before their FMAs so the loads overlap.
    // Invalid tokens have p = 0 and offset 0 (a valid row of the cache), so no guards are needed.
    const int nvalid = min(32, t1 - base);
#pragma unroll
    for (int tb = 0; tb < 32; tb += 8) {
      if (tb >= nvalid) break;
      uint2 vv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const long long o = __shfl_sync(0xffffffffu, off, tb + j);
        vv[j] = *reinterpret_cast<const uint2*>(v_cache + o + lane * 4);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float2 v0 = unpack_bf16x2(vv[j].x), v1 = unpack_bf16x2(vv[j].y);
#pragma unroll
        for (int h = 0; h < G; ++h) {
          const float pv = p_s[warp][h][tb + j];
          acc[h][0] += pv * v0.x;
          acc[h][1] += pv * v0.y;
          acc[h][2] += pv * v1.x;
          acc[h][3] += pv * v1.y;
        }
      }
    }
    __syncwarp();
  }
  // merge the 4 warps
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (lane == 0) {
      red_m[warp][h] = m[h];
      red_l[warp][h] = l[h];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) red_o[warp][h][lane * 4 + i] = acc[h][i];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * kDHead; i += blockDim.x) {
    const int h = i / kDHead, d = i % kDHead;
    float mm = -INFINITY;
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, red_m[w][h]);
    float ll = 0.f, oo = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float a = (red_m[w][h] == -INFINITY) ? 0.f : __expf(red_m[w][h] - mm);
      ll += red_l[w][h] * a;
      oo += red_o[w][h][d] * a;
    }
    const int hq = kvh * G + h;
    const long long pidx = (static_cast<long long>(s) * Hq + hq) * num_splits + split;
    part_o[pidx * kDHead + d] = oo;
    if (d == 0) {
      part_ml[pidx * 2] = mm;
      part_ml[pidx * 2 + 1] = ll;
    }
  }
}

__global__ void paged_decode_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                                          __nv_bfloat16* __restrict__ out, long long ldo, int Hq, int num_splits) {
  const int s = blockIdx.x, hq = blockIdx.y, d = threadIdx.x;
  const long long base = (static_cast<long long>(s) * Hq + hq) * num_splits;
  float mm = -INFINITY;
  for (int k = 0; k < num_splits; ++k) mm = fmaxf(mm, part_ml[(base + k) * 2]);
  float ll = 0.f, oo = 0.f;
  for (int k = 0; k < num_splits; ++k) {
    const float m = part_ml[(base + k) * 2];
    const float a = (m == -INFINITY) ? 0.f : __expf(m - mm);
    ll += part_ml[(base + k) * 2 + 1] * a;
    oo += part_o[(base + k) * kDHead + d] * a;
  }
  out[static_cast<long long>(s) * ldo + hq * kDHead + d] = __float2bfloat16(ll > 0.f ? oo / ll : 0.f);
}

__global__ void kv_cache_write_kernel(const __nv_bfloat16* __restrict__ k, const __nv_bfloat16* __restrict__ v,
                                      __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache,
                                      const int* __restrict__ slots, int T, int Hkv, long long ldk, long long ldv,
                                      long long num_slots) {
  const int t = blockIdx.x;
  const int slot = slots[t];
  if (slot < 0 || !ACCERL_DBG_OK(slot < num_slots, kDbgKvSlot, slot)) return;
  const int n16 = Hkv * kDHead / 8;
  const long long dst = static_cast<long long>(slot) * Hkv * kDHead;
  for (int i = threadIdx.x; i < n16; i += blockDim.x) {
    reinterpret_cast<uint4*>(k_cache + dst)[i] = reinterpret_cast<const uint4*>(k + t * ldk)[i];
    reinterpret_cast<uint4*>(v_cache + dst)[i] = reinterpret_cast<const uint4*>(v + t * ldv)[i];
  }
}

// Fused post-projection step of the engine's attention layers, one block per token row of the
// fused qkv projection [Hq*128 | Hkv*128 | Hkv*128]:
//   (Qwen3) per-head RMSNorm of the q and k heads, in place;
//   rotary embedding (rotate-half) of the q and k heads, in place;
//   the rotated k heads and the v heads into the paged caches at slots[t] (rows with slot < 0 skip).
// This replaces four launches (two RMSNorms, RoPE, cache write) and their round trips through
// memory. Every rounding matches the separate kernels: RMSNorm sums the squares in the order of
// rmsnorm_fwd_kernel (eight per lane, then a butterfly; the lanes it leaves idle add zeros) and
// rounds the normalised value before the weight; RoPE rounds cos/sin and its outputs to bf16.
// A half-warp owns one head: lane l holds elements [8l, 8l + 8), and its rotation partner
// (element d +- 64) sits on lane l +- 8.
__global__ void __launch_bounds__(256) qkv_rope_cache_kernel(
    __nv_bfloat16* __restrict__ qkv, long long ld, const long long* __restrict__ pos, const int* __restrict__ slots,
    int Hq, int Hkv, float log2_theta, const __nv_bfloat16* __restrict__ q_norm, const __nv_bfloat16* __restrict__ k_norm,
    float eps, __nv_bfloat16* __restrict__ k_cache, __nv_bfloat16* __restrict__ v_cache, long long num_slots) {
  __shared__ float cs[kDHead];  // [64] cos, [64] sin
  const int t = blockIdx.x;
  const float p = static_cast<float>(pos[t]);
  for (int i = threadIdx.x; i < kDHead / 2; i += blockDim.x) {
    float c, sn;
    rope_cos_sin(p, i, kDHead, log2_theta, c, sn);
    cs[i] = c;
    cs[kDHead / 2 + i] = sn;
  }
  __syncthreads();
  const int slot = slots[t];
  const bool cache = slot >= 0 && ACCERL_DBG_OK(slot < num_slots, kDbgKvSlot, slot);
  const int hl = threadIdx.x & 15;          // lane within the half-warp
  const int half_id = threadIdx.x >> 4;     // 16 half-warps per block
  const unsigned hmask = (threadIdx.x & 16) ? 0xffff0000u : 0x0000ffffu;
  __nv_bfloat16* row = qkv + t * ld;
  const int n_heads = Hq + 2 * Hkv;
  for (int h = half_id; h < n_heads; h += blockDim.x >> 4) {
    uint4* src = reinterpret_cast<uint4*>(row + h * kDHead) + hl;
    uint4 v = *src;
    if (h >= Hq + Hkv) {  // v head: to the cache only
      if (cache) reinterpret_cast<uint4*>(v_cache + (static_cast<long long>(slot) * Hkv + (h - Hq - Hkv)) * kDHead)[hl] = v;
      continue;
    }
    const __nv_bfloat16* nw = h < Hq ? q_norm : k_norm;
    uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(vw[i]);
        ss += f.x * f.x + f.y * f.y;
      }
      // rmsnorm_fwd_kernel's butterfly starts at offset 16, which only adds the zeros of its idle lanes
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(hmask, ss, o, 16);
      const float r = rsqrtf(ss / static_cast<float>(kDHead) + eps);
      const uint4 wv = reinterpret_cast<const uint4*>(nw)[hl];
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(vw[i]);
        const float2 g = unpack_bf16x2(ww[i]);
        const float2 n = unpack_bf16x2(pack_bf16x2(f.x * r, f.y * r));
        vw[i] = pack_bf16x2(n.x * g.x, n.y * g.y);
      }
    }
    // rotation: the partner lane holds the other half of every pair
    uint32_t pw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pw[i] = __shfl_xor_sync(hmask, vw[i], 8, 16);
    const bool first = hl < 8;
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 mine = unpack_bf16x2(vw[i]), other = unpack_bf16x2(pw[i]);
      const int d = (hl & 7) * 8 + 2 * i;  // frequency index of the pair's first element
      const float c0 = cs[d], c1 = cs[d + 1], s0 = cs[kDHead / 2 + d], s1 = cs[kDHead / 2 + d + 1];
      if (first) {  // x1 (mine) * c - x2 (other) * s
        o[i] = pack_bf16x2(mine.x * c0 - other.x * s0, mine.y * c1 - other.y * s1);
      } else {      // x2 (mine) * c + x1 (other) * s
        o[i] = pack_bf16x2(mine.x * c0 + other.x * s0, mine.y * c1 + other.y * s1);
      }
    }
    v = make_uint4(o[0], o[1], o[2], o[3]);
    *src = v;
    if (h >= Hq && cache) reinterpret_cast<uint4*>(k_cache + (static_cast<long long>(slot) * Hkv + (h - Hq)) * kDHead)[hl] = v;
  }
}

}  // namespace accerl

using namespace accerl;

extern "C" int accerl_paged_decode(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                                   const int* seq_lens, void* out, float* part_o, float* part_ml, int num_seqs, int Hq,
                                   int Hkv, int max_blocks_per_seq, int block_size, int num_splits, float scale,
                                   long long ldq, long long ldo, cudaStream_t s) {
  if (num_seqs == 0) return 0;
  if (Hq % Hkv) return -1;
  const int G = Hq / Hkv;
  dim3 grid(num_seqs, Hkv, num_splits);
#define LAUNCH_G(GV)                                                                                              \
  case GV:                                                                                                        \
    paged_decode_kernel<GV><<<grid, 128, 0, s>>>((const __nv_bfloat16*)q, ldq, (const __nv_bfloat16*)k_cache,   \
                                                 (const __nv_bfloat16*)v_cache, block_table, max_blocks_per_seq, \
                                                 seq_lens, block_size, Hkv, num_splits, scale, part_o, part_ml);  \
    break;
  switch (G) {
    LAUNCH_G(1)
    LAUNCH_G(2)
    LAUNCH_G(4)
    LAUNCH_G(6)
    LAUNCH_G(8)
    default:
      return -2;
  }
#undef LAUNCH_G
  paged_decode_merge_kernel<<<dim3(num_seqs, Hq), kDHead, 0, s>>>(part_o, part_ml, (__nv_bfloat16*)out, ldo, Hq,
                                                                  num_splits);
  return (int)cudaGetLastError();
}

// Combine the per-split partials of a paged decode into out ([num_seqs, Hq*128] bf16, row stride ldo).
extern "C" int accerl_paged_decode_merge(const float* part_o, const float* part_ml, void* out, long long ldo,
                                         int num_seqs, int Hq, int num_splits, cudaStream_t s) {
  if (num_seqs == 0) return 0;
  paged_decode_merge_kernel<<<dim3(num_seqs, Hq), kDHead, 0, s>>>(part_o, part_ml, (__nv_bfloat16*)out, ldo, Hq,
                                                                  num_splits);
  return (int)cudaGetLastError();
}

extern "C" int accerl_kv_cache_write(const void* k, const void* v, void* k_cache, void* v_cache, const int* slot_mapping,
                                     int T, int Hkv, long long ldk, long long ldv, long long num_slots, cudaStream_t s) {
  if (T == 0) return 0;
  if ((ldk | ldv) & 7) return -1;
  kv_cache_write_kernel<<<T, 128, 0, s>>>((const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (__nv_bfloat16*)k_cache,
                                          (__nv_bfloat16*)v_cache, slot_mapping, T, Hkv, ldk, ldv, num_slots);
  return (int)cudaGetLastError();
}

extern "C" int accerl_qkv_rope_cache(void* qkv, long long ld, const long long* pos, const int* slots, int T, int Hq,
                                     int Hkv, float theta, const void* q_norm, const void* k_norm, float eps,
                                     void* k_cache, void* v_cache, long long num_slots, cudaStream_t s) {
  if (T == 0) return 0;
  if ((ld & 7) || Hq < 1 || Hkv < 1 || ld < static_cast<long long>(Hq + 2 * Hkv) * kDHead || !(theta > 0.f) ||
      (!q_norm) != (!k_norm))
    return -1;
  qkv_rope_cache_kernel<<<T, 256, 0, s>>>((__nv_bfloat16*)qkv, ld, pos, slots, Hq, Hkv, log2f(theta),
                                          (const __nv_bfloat16*)q_norm, (const __nv_bfloat16*)k_norm, eps,
                                          (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, num_slots);
  return (int)cudaGetLastError();
}

ACCERL_DEBUG_EXPORT(rollout)
