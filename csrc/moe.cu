// MoE combine kernels (sm_100a), one block per token row:
//  combine_fwd  out[t] = residual[t] + sum_j w[t,j] * ys[pos[t,j]] + sg[t] * shared[t]
//               (fp32 accumulation, bf16 out; residual / shared expert optional)
//  combine_bwd  dys[pos[t,j]] = w[t,j] * dout[t]  (bf16 rows of the expert-output gradient)
//               dw[t,j] = <dout[t], ys[pos[t,j]]> (fp32 gradient of the routing weight)
// pos maps a (token, slot) pair to its row in the expert-ordered buffer (padded segments or the
// sorted order of an expert-parallel exchange). H must be a multiple of 8 and k <= 8.
#include "common.cuh"

namespace accerl {

constexpr int kMoeMaxK = 8;

__global__ void moe_combine_fwd_kernel(const __nv_bfloat16* __restrict__ ys, const long long* __restrict__ pos,
                                       const float* __restrict__ w, int k, int H,
                                       const __nv_bfloat16* __restrict__ residual,
                                       const __nv_bfloat16* __restrict__ shared, const float* __restrict__ sg,
                                       __nv_bfloat16* __restrict__ out, long long R) {
  const long long t = blockIdx.x;
  const int nv = H / 8;
  __shared__ long long rows[kMoeMaxK];
  __shared__ float ws[kMoeMaxK];
  if (threadIdx.x < k) {
    long long r = pos[t * k + threadIdx.x];
    float wr = w[t * k + threadIdx.x];
    if (!ACCERL_DBG_OK(r >= 0 && r < R, kDbgMoeRow, r)) {
      r = 0;
      wr = 0.f;
    }
    rows[threadIdx.x] = r;
    ws[threadIdx.x] = wr;
  }
  __syncthreads();
  const float g = sg ? sg[t] : 0.f;
  for (int c = threadIdx.x; c < nv; c += blockDim.x) {
    float acc[8];
    if (residual) {
      const uint4 r = reinterpret_cast<const uint4*>(residual + t * H)[c];
      const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(rw[i]);
        acc[2 * i] = f.x;
        acc[2 * i + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    }
    for (int j = 0; j < k; ++j) {
      const uint4 v = reinterpret_cast<const uint4*>(ys + rows[j] * H)[c];
      const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
      const float wj = ws[j];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(vw[i]);
        acc[2 * i] += wj * f.x;
        acc[2 * i + 1] += wj * f.y;
      }
    }
    if (shared) {
      const uint4 v = reinterpret_cast<const uint4*>(shared + t * H)[c];
      const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(vw[i]);
        acc[2 * i] += g * f.x;
        acc[2 * i + 1] += g * f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * H)[c] = o;
  }
}

__global__ void moe_combine_bwd_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ ys,
                                       const long long* __restrict__ pos, const float* __restrict__ w, int k, int H,
                                       __nv_bfloat16* __restrict__ dys, float* __restrict__ dw, long long R) {
  const long long t = blockIdx.x;
  const int nv = H / 8;
  __shared__ long long rows[kMoeMaxK];
  __shared__ float ws[kMoeMaxK];
  __shared__ float red[kMoeMaxK][8];
  if (threadIdx.x < k) {
    long long r = pos[t * k + threadIdx.x];
    float wr = w[t * k + threadIdx.x];
    if (!ACCERL_DBG_OK(r >= 0 && r < R, kDbgMoeRow, r)) {
      r = 0;
      wr = 0.f;
    }
    rows[threadIdx.x] = r;
    ws[threadIdx.x] = wr;
  }
  __syncthreads();
  float dot[kMoeMaxK];
#pragma unroll
  for (int j = 0; j < kMoeMaxK; ++j) dot[j] = 0.f;
  for (int c = threadIdx.x; c < nv; c += blockDim.x) {
    const uint4 d = reinterpret_cast<const uint4*>(dout + t * H)[c];
    const uint32_t dwd[4] = {d.x, d.y, d.z, d.w};
    float g[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(dwd[i]);
      g[2 * i] = f.x;
      g[2 * i + 1] = f.y;
    }
#pragma unroll
    for (int j = 0; j < kMoeMaxK; ++j) {
      if (j >= k) break;
      const uint4 v = reinterpret_cast<const uint4*>(ys + rows[j] * H)[c];
      const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(vw[i]);
        s += g[2 * i] * f.x + g[2 * i + 1] * f.y;
      }
      dot[j] += s;
      const float wj = ws[j];
      uint4 o;
      o.x = pack_bf16x2(wj * g[0], wj * g[1]);
      o.y = pack_bf16x2(wj * g[2], wj * g[3]);
      o.z = pack_bf16x2(wj * g[4], wj * g[5]);
      o.w = pack_bf16x2(wj * g[6], wj * g[7]);
      reinterpret_cast<uint4*>(dys + rows[j] * H)[c] = o;
    }
  }
  // block reduction of the k dot products (blockDim.x <= 256: 8 warps)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kMoeMaxK; ++j) {
    if (j >= k) break;
    const float v = warp_sum(dot[j]);
    if (lane == 0) red[j][warp] = v;
  }
  __syncthreads();
  if (threadIdx.x < k) {
    float s = 0.f;
    for (int i = 0; i < (blockDim.x >> 5); ++i) s += red[threadIdx.x][i];
    dw[t * k + threadIdx.x] = s;
  }
}

// Router of a mixture-of-experts layer, one warp per token: logits (fp32 GEMM output, rounded to
// bf16 as the reference's bf16 linear produces them) -> softmax over E experts -> top-k (largest
// first, lower expert id on ties) -> optional renormalisation of the k weights; per-expert routed
// row counts accumulate into `counts` (zeroed by the caller). E <= 128, k <= 8.
// With sg != null, column E of the logits is the shared-expert gate logit: sg[t] = sigmoid of it
// (rounded to bf16 first, as the reference's bf16 gate linear gives it).
__global__ void moe_router_kernel(const float* __restrict__ logits, long long ldl, int T, int E, int k, int norm_topk,
                                  float* __restrict__ probs, float* __restrict__ topw, long long* __restrict__ topi,
                                  int* __restrict__ counts, float* __restrict__ sg) {
  const int t = static_cast<int>((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  float v[4];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? __bfloat162float(__float2bfloat16(logits[static_cast<long long>(t) * ldl + e])) : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = lane + 32 * j < E ? expf(v[j] - mx) : 0.f;
    sum += v[j];
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    v[j] *= inv;
    if (e < E) probs[static_cast<long long>(t) * E + e] = v[j];
  }
  // top-k by repeated warp arg-max; a chosen value is set to -1 (probabilities are >= 0)
  float w_sel[kMoeMaxK];
  int i_sel[kMoeMaxK];
  float wsum = 0.f;
  for (int r = 0; r < k; ++r) {
    float best = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int e = lane + 32 * j;
      if (e < E && v[j] > best) {
        best = v[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    w_sel[r] = best;
    i_sel[r] = bi;
    wsum += best;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (lane + 32 * j == bi) v[j] = -1.f;
  }
  if (sg != nullptr && lane == 0) {
    const float z = __bfloat162float(__float2bfloat16(logits[static_cast<long long>(t) * ldl + E]));
    sg[t] = 1.f / (1.f + expf(-z));
  }
  if (lane == 0) {
    const float scale = norm_topk ? 1.f / wsum : 1.f;
    for (int r = 0; r < k; ++r) {
      topw[static_cast<long long>(t) * k + r] = w_sel[r] * scale;
      topi[static_cast<long long>(t) * k + r] = i_sel[r];
      atomicAdd(counts + i_sel[r], 1);
    }
  }
}

// Router backward, one warp per token (the reverse of moe_router_kernel plus the shared-expert gate):
//   d(top-k weights) dw -> (renormalised: (dw - <dw, topw>) / sum of the k probabilities) ->
//   scattered onto the k chosen experts -> softmax backward: dlogits = p * (dp - <dp, p>).
// With a shared expert (sy != null): dsg = <dout, sy> * sg * (1 - sg) is stored as column E of the
// gradient row, so that one GEMM against [gate weight; shared-gate weight] gives both input-gradient
// terms, and dsy = sg * dout (bf16), the shared expert's output gradient. Columns past E (+1) are
// zero. dgrad: [T, E_pad] bf16 with E_pad a multiple of 8 (>= E + 1 with a shared expert).
__global__ void moe_router_bwd_kernel(const float* __restrict__ probs, const long long* __restrict__ topi,
                                      const float* __restrict__ topw, const float* __restrict__ dw, int T, int E,
                                      int k, int norm_topk, const __nv_bfloat16* __restrict__ dout,
                                      const __nv_bfloat16* __restrict__ sy, const float* __restrict__ sg, int H,
                                      __nv_bfloat16* __restrict__ dgrad, int E_pad, __nv_bfloat16* __restrict__ dsy) {
  const int t = static_cast<int>((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  const long long tk = static_cast<long long>(t) * k;
  // gradient of the chosen probabilities
  float dpk = 0.f, wk = 0.f;
  int ek = -1;
  if (lane < k) {
    ek = static_cast<int>(topi[tk + lane]);
    dpk = dw[tk + lane];
    wk = topw[tk + lane];
  }
  if (norm_topk) {
    const float pk = lane < k ? probs[static_cast<long long>(t) * E + ek] : 0.f;
    const float S = warp_sum(pk);
    const float c = warp_sum(dpk * wk);
    dpk = S > 0.f ? (dpk - c) / S : 0.f;
  }
  // dp over all experts (zero outside the k chosen ones); lane holds experts lane + 32 j
  float p[4], dp[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    p[j] = e < E ? probs[static_cast<long long>(t) * E + e] : 0.f;
    dp[j] = 0.f;
  }
  for (int r = 0; r < k; ++r) {
    const int er = __shfl_sync(0xffffffffu, ek, r);
    const float gr = __shfl_sync(0xffffffffu, dpk, r);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (lane + 32 * j == er) dp[j] += gr;
  }
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) dot += dp[j] * p[j];
  dot = warp_sum(dot);
  __nv_bfloat16* row = dgrad + static_cast<long long>(t) * E_pad;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int e = lane + 32 * j;
    if (e < E) row[e] = __float2bfloat16(p[j] * (dp[j] - dot));
  }
  int first_pad = E;
  if (sy != nullptr) {
    const float g = sg[t];
    const __nv_bfloat16* drow = dout + static_cast<long long>(t) * H;
    const __nv_bfloat16* srow = sy + static_cast<long long>(t) * H;
    __nv_bfloat16* dsrow = dsy + static_cast<long long>(t) * H;
    float acc = 0.f;
    for (int c = lane * 8; c < H; c += 256) {
      const uint4 dv = *reinterpret_cast<const uint4*>(drow + c);
      const uint4 sv = *reinterpret_cast<const uint4*>(srow + c);
      const uint32_t dwv[4] = {dv.x, dv.y, dv.z, dv.w};
      const uint32_t swv[4] = {sv.x, sv.y, sv.z, sv.w};
      uint32_t ow[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = unpack_bf16x2(dwv[i]);
        const float2 b = unpack_bf16x2(swv[i]);
        acc += a.x * b.x + a.y * b.y;
        ow[i] = pack_bf16x2(a.x * g, a.y * g);
      }
      *reinterpret_cast<uint4*>(dsrow + c) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    acc = warp_sum(acc);
    if (lane == 0) row[E] = __float2bfloat16(acc * g * (1.f - g));
    first_pad = E + 1;
  }
  for (int e = first_pad + lane; e < E_pad; e += 32) row[e] = __float2bfloat16(0.f);
}

// Dispatch layout in two launches, with no host synchronisation and no sort.
// The (token, slot) pairs are numbered token-major, p = t * k + j. Block b owns pairs
// [b * 1024, (b + 1) * 1024). An expert's rows are its pairs in increasing p (a stable counting
// sort), so a pair's rank within its expert is
//   (its expert's pairs in earlier blocks) + (in earlier warps of its block) + (in lower lanes).
// Experts [lo, lo + El) own row segments padded to kLayoutSeg rows, back to back from row 0; a pair
// routed elsewhere (a tensor-parallel engine shard) gets row `total` and weight 0.
constexpr int kLayoutPairs = 1024;
constexpr int kLayoutSeg = 128;
constexpr int kLayoutMaxE = 256;

__global__ void __launch_bounds__(kLayoutPairs) moe_layout_hist_kernel(const long long* __restrict__ topi, long long n,
                                                                      int E, int* __restrict__ hist) {
  __shared__ int h[kLayoutMaxE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) h[e] = 0;
  __syncthreads();
  const long long p = static_cast<long long>(blockIdx.x) * kLayoutPairs + threadIdx.x;
  if (p < n) {
    const long long e = topi[p];
    if (e >= 0 && e < E) atomicAdd(&h[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[static_cast<long long>(blockIdx.x) * E + e] = h[e];
}

// Shared memory: before[E], tot[E], start[El], end[El], wrank[32][E] (ints).
__global__ void __launch_bounds__(kLayoutPairs) moe_layout_place_kernel(
    const long long* __restrict__ topi, const float* __restrict__ topw, long long n, int k, int E, int lo, int El,
    long long total, const int* __restrict__ hist, int nblocks, const __nv_bfloat16* __restrict__ h, int H,
    __nv_bfloat16* __restrict__ xs, int zero_pad, long long* __restrict__ pos, float* __restrict__ w,
    int* __restrict__ tile_expert, int* __restrict__ row_start, int* __restrict__ seg_rows, int* __restrict__ counts) {
  extern __shared__ int sm[];
  int* before = sm;
  int* tot = before + E;
  int* start = tot + E;
  int* end = start + El;
  int* wrank = end + El;  // [32][E]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 32 * E; i += blockDim.x) wrank[i] = 0;
  for (int e = tid; e < E; e += blockDim.x) {  // coalesced over e, one pass over the histogram rows
    int b4 = 0, s = 0;
    for (int b = 0; b < nblocks; ++b) {
      const int v = hist[static_cast<long long>(b) * E + e];
      b4 += b < static_cast<int>(blockIdx.x) ? v : 0;
      s += v;
    }
    before[e] = b4;
    tot[e] = s;
  }
  __syncthreads();
  if (warp == 0) {  // padded segment sizes and their exclusive prefix sum over the local experts
    const int per = (El + 31) / 32, a = min(El, lane * per), z = min(El, a + per);
    int run = 0;
    for (int i = a; i < z; ++i) run += (tot[lo + i] + kLayoutSeg - 1) / kLayoutSeg * kLayoutSeg;
    int incl = run;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int at = incl - run;
    for (int i = a; i < z; ++i) {
      const int pad = (tot[lo + i] + kLayoutSeg - 1) / kLayoutSeg * kLayoutSeg;
      start[i] = at;
      at += pad;
      end[i] = at;
    }
  }
  // this block's pairs: rank among the same expert's pairs of this warp, and per-warp counts
  const long long p = static_cast<long long>(blockIdx.x) * kLayoutPairs + tid;
  long long e = p < n ? topi[p] : -1;
  if (e < 0 || e >= E) e = -1;
  const unsigned same = __match_any_sync(0xffffffffu, static_cast<int>(e));
  const int lane_rank = __popc(same & ((1u << lane) - 1u));
  __syncthreads();  // wrank zeroed, start/end written
  if (e >= 0 && lane_rank == 0) wrank[warp * E + e] = __popc(same);
  __syncthreads();
  for (int x = tid; x < E; x += blockDim.x) {  // exclusive prefix over the warps
    int run = 0;
    for (int v = 0; v < 32; ++v) {
      const int c = wrank[v * E + x];
      wrank[v * E + x] = run;
      run += c;
    }
  }
  __syncthreads();
  long long row = total;
  if (e >= lo && e < lo + El) row = start[e - lo] + before[e] + wrank[warp * E + e] + lane_rank;
  if (p < n) {
    pos[p] = row;
    w[p] = row < total ? __bfloat162float(__float2bfloat16(topw[p])) : 0.f;
  }
  if (blockIdx.x == 0) {
    for (int i = tid; i < El; i += blockDim.x) {
      row_start[i] = start[i];
      seg_rows[i] = end[i] - start[i];
    }
    if (counts)
      for (int i = tid; i < E; i += blockDim.x) counts[i] = tot[i];
    const long long tiles = total / kLayoutSeg;
    for (long long t = tid; t < tiles; t += blockDim.x) {  // first segment whose end is past the tile
      const long long r = t * kLayoutSeg;
      int lo_i = 0, hi_i = El;
      while (lo_i < hi_i) {
        const int mid = (lo_i + hi_i) >> 1;
        if (end[mid] <= r) lo_i = mid + 1; else hi_i = mid;
      }
      tile_expert[t] = lo_i < El ? lo_i : -1;
    }
  }
  // gather: every pair of this warp copies its token's row of h into its row of xs (16 B per lane)
  const int vec = H / 8;
  for (int j = 0; j < 32; ++j) {
    const long long rj = __shfl_sync(0xffffffffu, row, j);
    const long long pj = static_cast<long long>(blockIdx.x) * kLayoutPairs + warp * 32 + j;
    if (pj >= n || rj >= total) continue;
    const uint4* src = reinterpret_cast<const uint4*>(h + (pj / k) * static_cast<long long>(H));
    uint4* dst = reinterpret_cast<uint4*>(xs + rj * static_cast<long long>(H));
    for (int c = lane; c < vec; c += 32) dst[c] = src[c];
  }
  if (!zero_pad) return;
  // training: rows of a segment past its expert's pairs, and the tiles past the last segment, are
  // zero (the weight-gradient contraction runs over them)
  const long long gw = static_cast<long long>(blockIdx.x) * 32 + warp, nw = static_cast<long long>(gridDim.x) * 32;
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  for (long long r = gw; r < total; r += nw) {
    int lo_i = 0, hi_i = El;
    while (lo_i < hi_i) {
      const int mid = (lo_i + hi_i) >> 1;
      if (end[mid] <= r) lo_i = mid + 1; else hi_i = mid;
    }
    if (lo_i < El && r - start[lo_i] < tot[lo + lo_i]) continue;
    uint4* dst = reinterpret_cast<uint4*>(xs + r * static_cast<long long>(H));
    for (int c = lane; c < vec; c += 32) dst[c] = z;
  }
}

}  // namespace accerl

using namespace accerl;

extern "C" int accerl_moe_router_bwd(const float* probs, const long long* topi, const float* topw, const float* dw,
                                     int T, int E, int k, int norm_topk, const void* dout, const void* sy,
                                     const float* sg, int H, void* dgrad, int E_pad, void* dsy, cudaStream_t s) {
  if (T <= 0) return 0;
  if (E < 1 || E > 128 || k < 1 || k > kMoeMaxK || k > 32 || E_pad % 8 || E_pad < E + (sy ? 1 : 0)) return -1;
  if (sy && (H % 8 || !dout || !sg || !dsy)) return -1;
  const long long threads = static_cast<long long>(T) * 32;
  moe_router_bwd_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
      probs, topi, topw, dw, T, E, k, norm_topk, (const __nv_bfloat16*)dout, (const __nv_bfloat16*)sy, sg, H,
      (__nv_bfloat16*)dgrad, E_pad, (__nv_bfloat16*)dsy);
  return (int)cudaGetLastError();
}

extern "C" int accerl_moe_combine_fwd(const void* ys, const long long* pos, const float* w, long long T, int k, int H,
                                      const void* residual, const void* shared, const float* sg, void* out,
                                      long long R, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 || k < 1 || k > kMoeMaxK) return -1;
  const int threads = min(256, max(32, ((H / 8 + 31) / 32) * 32));
  moe_combine_fwd_kernel<<<(unsigned)T, threads, 0, s>>>((const __nv_bfloat16*)ys, pos, w, k, H,
                                                         (const __nv_bfloat16*)residual, (const __nv_bfloat16*)shared,
                                                         sg, (__nv_bfloat16*)out, R);
  return (int)cudaGetLastError();
}

extern "C" int accerl_moe_combine_bwd(const void* dout, const void* ys, const long long* pos, const float* w, long long T,
                                      int k, int H, void* dys, float* dw, long long R, cudaStream_t s) {
  if (T <= 0) return 0;
  if (H % 8 || k < 1 || k > kMoeMaxK) return -1;
  const int threads = min(256, max(32, ((H / 8 + 31) / 32) * 32));
  moe_combine_bwd_kernel<<<(unsigned)T, threads, 0, s>>>((const __nv_bfloat16*)dout, (const __nv_bfloat16*)ys, pos, w,
                                                         k, H, (__nv_bfloat16*)dys, dw, R);
  return (int)cudaGetLastError();
}

extern "C" int accerl_moe_router(const float* logits, long long ldl, int T, int E, int k, int norm_topk, float* probs,
                                 float* topw, long long* topi, int* counts, float* sg, cudaStream_t s) {
  if (T <= 0) return 0;
  if (E < 1 || E > 128 || k < 1 || k > kMoeMaxK || k > E) return -1;
  const long long threads = static_cast<long long>(T) * 32;
  moe_router_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(logits, ldl, T, E, k, norm_topk, probs, topw,
                                                                       topi, counts, sg);
  return (int)cudaGetLastError();
}

// hist: [ceil(n / 1024), E] int32 scratch. total must be a multiple of 128 that holds every padded
// segment (n + El * 127 rounded up always does); tile_expert has total / 128 entries.
extern "C" int accerl_moe_layout(const long long* topi, const float* topw, long long n, int k, int E, int lo, int El,
                                 long long total, const void* h, int H, void* xs, int zero_pad, int* hist,
                                 long long* pos, float* w, int* tile_expert, int* row_start, int* seg_rows,
                                 int* counts, cudaStream_t s) {
  if (n <= 0) return 0;
  if (E < 1 || E > kLayoutMaxE || k < 1 || El < 1 || lo < 0 || lo + El > E || H % 8 || total % kLayoutSeg ||
      total < n + static_cast<long long>(El) * (kLayoutSeg - 1) || total > INT32_MAX)
    return -1;
  const long long blocks = (n + kLayoutPairs - 1) / kLayoutPairs;
  if (blocks > INT32_MAX) return -1;
  moe_layout_hist_kernel<<<(unsigned)blocks, kLayoutPairs, 0, s>>>(topi, n, E, hist);
  const int smem = (34 * E + 2 * El) * static_cast<int>(sizeof(int));
  moe_layout_place_kernel<<<(unsigned)blocks, kLayoutPairs, smem, s>>>(
      topi, topw, n, k, E, lo, El, total, hist, static_cast<int>(blocks), (const __nv_bfloat16*)h, H,
      (__nv_bfloat16*)xs, zero_pad, pos, w, tile_expert, row_start, seg_rows, counts);
  return (int)cudaGetLastError();
}

ACCERL_DEBUG_EXPORT(moe)
