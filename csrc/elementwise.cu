// Memory-bound fused ops of the decoder layer (sm_100a): RMSNorm fwd/bwd, rotary embedding,
// SwiGLU fwd/bwd, token embedding gather / scatter-add, bias-gradient column sums.
// All vector accesses are 16 bytes (8 bf16); the hidden sizes used here are multiples of 8.
#include <algorithm>

#include "common.cuh"

namespace accerl {

// ------------------------------------------------------------------------------------------------
// RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w ; one warp per row, rstd saved for backward.
// ------------------------------------------------------------------------------------------------
__global__ void rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                   __nv_bfloat16* __restrict__ y, float* __restrict__ rstd_out, int rows, int H,
                                   long long ldx, long long ldy, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const __nv_bfloat16* xr = x + row * ldx;
  float ss = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(vw[i]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / static_cast<float>(H) + eps);
  if (lane == 0 && rstd_out) rstd_out[row] = r;
  __nv_bfloat16* yr = y + row * ldy;
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(vw[i]);
      const float2 g = unpack_bf16x2(ww[i]);
      // Match the reference module: normalise in fp32, round to the activation dtype, then scale.
      const float2 n = unpack_bf16x2(pack_bf16x2(f.x * r, f.y * r));
      o[i] = pack_bf16x2(n.x * g.x, n.y * g.y);
    }
    *reinterpret_cast<uint4*>(yr + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// dx = rstd * (w*dy - xhat * mean(xhat * w * dy));  dx is added to `dx_accum` when given (the
// residual-stream gradient), written to dx otherwise.
__global__ void rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                   const __nv_bfloat16* __restrict__ w, const float* __restrict__ rstd,
                                   const __nv_bfloat16* dx_accum, __nv_bfloat16* dx, int rows, int H, long long ld) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float r = rstd[row];
  const __nv_bfloat16* dyr = dy + row * ld;
  const __nv_bfloat16* xr = x + row * ld;
  float dot = 0.f;
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(dyr + c);
    const uint4 b = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 g = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w}, gw[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = unpack_bf16x2(aw[i]), fb = unpack_bf16x2(bw[i]), fg = unpack_bf16x2(gw[i]);
      dot += fa.x * fg.x * fb.x * r + fa.y * fg.y * fb.y * r;
    }
  }
  dot = warp_sum(dot) / static_cast<float>(H);
  for (int c = lane * 8; c < H; c += 256) {
    const uint4 a = *reinterpret_cast<const uint4*>(dyr + c);
    const uint4 b = *reinterpret_cast<const uint4*>(xr + c);
    const uint4 g = *reinterpret_cast<const uint4*>(w + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t acc[4] = {0, 0, 0, 0};
    if (dx_accum) {
      const uint4 q = *reinterpret_cast<const uint4*>(dx_accum + row * ld + c);
      acc[0] = q.x; acc[1] = q.y; acc[2] = q.z; acc[3] = q.w;
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = unpack_bf16x2(aw[i]), fb = unpack_bf16x2(bw[i]), fg = unpack_bf16x2(gw[i]);
      float d0 = r * (fa.x * fg.x - fb.x * r * dot);
      float d1 = r * (fa.y * fg.y - fb.y * r * dot);
      if (dx_accum) {
        const float2 q = unpack_bf16x2(acc[i]);
        d0 += q.x;
        d1 += q.y;
      }
      o[i] = pack_bf16x2(d0, d1);
    }
    *reinterpret_cast<uint4*>(dx + row * ld + c) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Fused backward: dx as above plus the weight-gradient partial of the rows this warp visits, kept in
// registers (NC = H / 256 chunks of 8 columns per lane); the block's warps sum theirs in shared
// memory and each block writes one partial row.
template <int NC>
__global__ void __launch_bounds__(256) rmsnorm_bwd_fused_kernel(const __nv_bfloat16* __restrict__ dy,
                                                                const __nv_bfloat16* __restrict__ x,
                                                                const __nv_bfloat16* __restrict__ w,
                                                                const float* __restrict__ rstd,
                                                                const __nv_bfloat16* dx_accum, __nv_bfloat16* dx,
                                                                float* __restrict__ part, int rows, long long ld) {
  constexpr int H = NC * 256;
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  float wf[NC][8];
  float acc[NC][8];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const uint4 g = *reinterpret_cast<const uint4*>(w + c * 256 + lane * 8);
    const uint32_t gw4[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_bf16x2(gw4[i]);
      wf[c][2 * i] = f.x;
      wf[c][2 * i + 1] = f.y;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[c][i] = 0.f;
  }
  for (int row = gw; row < rows; row += nw) {
    // every load of the row is issued up front (dy, x and the incoming dx): one DRAM round trip per row.
    // Rows wider than 1536 keep only the incoming dx in registers and re-read dy, x from L1.
    constexpr bool kHold = NC <= 6;
    constexpr int NH = kHold ? NC : 1;
    uint4 av[NH], bv[NH], qv[NH];
    if constexpr (kHold) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        av[c] = *reinterpret_cast<const uint4*>(dy + row * ld + c * 256 + lane * 8);
        bv[c] = *reinterpret_cast<const uint4*>(x + row * ld + c * 256 + lane * 8);
        qv[c] = dx_accum ? *reinterpret_cast<const uint4*>(dx_accum + row * ld + c * 256 + lane * 8)
                         : make_uint4(0, 0, 0, 0);
      }
    }
    auto ld_q = [&](int c) -> uint4 {
      if constexpr (kHold) return qv[c];
      else
        return dx_accum ? *reinterpret_cast<const uint4*>(dx_accum + row * ld + c * 256 + lane * 8)
                        : make_uint4(0, 0, 0, 0);
    };
    auto ld_dy = [&](int c) -> uint4 {
      if constexpr (kHold) return av[c];
      else return *reinterpret_cast<const uint4*>(dy + row * ld + c * 256 + lane * 8);
    };
    auto ld_x = [&](int c) -> uint4 {
      if constexpr (kHold) return bv[c];
      else return *reinterpret_cast<const uint4*>(x + row * ld + c * 256 + lane * 8);
    };
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const uint4 a4 = ld_dy(c), b4 = ld_x(c);
      const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w}, bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fa = unpack_bf16x2(aw[i]), fb = unpack_bf16x2(bw[i]);
        dot += fa.x * wf[c][2 * i] * fb.x * r + fa.y * wf[c][2 * i + 1] * fb.y * r;
        // the module rounds x*rstd to bf16 before scaling by w; the weight gradient uses that value
        const float2 n = unpack_bf16x2(pack_bf16x2(fb.x * r, fb.y * r));
        acc[c][2 * i] += fa.x * n.x;
        acc[c][2 * i + 1] += fa.y * n.y;
      }
    }
    dot = warp_sum(dot) / static_cast<float>(H);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const uint4 a4 = ld_dy(c), b4 = ld_x(c);  // the second touch hits L1 when not held
      const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w}, bw[4] = {b4.x, b4.y, b4.z, b4.w};
      const uint4 q4 = ld_q(c);
      const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 fa = unpack_bf16x2(aw[i]), fb = unpack_bf16x2(bw[i]), q = unpack_bf16x2(qw[i]);
        const float d0 = r * (fa.x * wf[c][2 * i] - fb.x * r * dot) + q.x;
        const float d1 = r * (fa.y * wf[c][2 * i + 1] - fb.y * r * dot) + q.y;
        o[i] = pack_bf16x2(d0, d1);
      }
      *reinterpret_cast<uint4*>(dx + row * ld + c * 256 + lane * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // the block's 8 warps add their partials in fixed warp order (deterministic), one row per block
  __shared__ float red[H];
  const int warp = threadIdx.x >> 5;
  for (int wv = 0; wv < 8; ++wv) {
    if (warp == wv) {
#pragma unroll
      for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float* slot = red + c * 256 + lane * 8 + i;
          *slot = (wv == 0 ? 0.f : *slot) + acc[c][i];
        }
    }
    __syncthreads();
  }
  float* dst = part + static_cast<long long>(blockIdx.x) * H;
  for (int h = threadIdx.x; h < H; h += blockDim.x) dst[h] = red[h];
}

// Partial column sums for the RMSNorm weight gradient: part[b, h] = sum over this block's rows of
// dy * x * rstd. Each thread owns 8 consecutive columns.
__global__ void rmsnorm_dw_partial_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                          const float* __restrict__ rstd, float* __restrict__ part, int rows, int H,
                                          long long ld, int rows_per_block) {
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= H) return;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int r = r0; r < r1; ++r) {
    const float s = rstd[r];
    const uint4 a = *reinterpret_cast<const uint4*>(dy + r * ld + c);
    const uint4 b = *reinterpret_cast<const uint4*>(x + r * ld + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = unpack_bf16x2(aw[i]), fb = unpack_bf16x2(bw[i]);
      // The module rounds x*rstd to bf16 before scaling by w; the weight gradient uses that value.
      const float2 n = unpack_bf16x2(pack_bf16x2(fb.x * s, fb.y * s));
      acc[2 * i] += fa.x * n.x;
      acc[2 * i + 1] += fa.y * n.y;
    }
  }
  float* dst = part + static_cast<long long>(blockIdx.x) * H + c;
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = acc[i];
}

// out[h] (+)= sum_b part[b, h]: block (32 columns x 8 row groups); row group g sums rows g, g+8, ...
// and the 8 group sums are added in fixed order (deterministic).
__global__ void column_reduce_kernel(const float* __restrict__ part, float* __restrict__ out, int nblk, int H,
                                     int accumulate) {
  const int tx = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int h = blockIdx.x * 32 + tx;
  __shared__ float red[8][33];
  float s = 0.f;
  if (h < H)
    for (int b = g; b < nblk; b += 8) s += part[static_cast<long long>(b) * H + h];
  red[g][tx] = s;
  __syncthreads();
  if (g == 0 && h < H) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += red[i][tx];
    out[h] = accumulate ? out[h] + t : t;
  }
}

// Bias gradient partials: part[b, n] = sum of dy[r, n] over this block's rows.
__global__ void colsum_partial_kernel(const __nv_bfloat16* __restrict__ dy, float* __restrict__ part, int rows, int N,
                                      long long ld, int rows_per_block) {
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (c >= N) return;
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int r = r0; r < r1; ++r) {
    const uint4 a = *reinterpret_cast<const uint4*>(dy + r * ld + c);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = unpack_bf16x2(aw[i]);
      acc[2 * i] += fa.x;
      acc[2 * i + 1] += fa.y;
    }
  }
  float* dst = part + static_cast<long long>(blockIdx.x) * N + c;
#pragma unroll
  for (int i = 0; i < 8; ++i) dst[i] = acc[i];
}

// ------------------------------------------------------------------------------------------------
// Rotary embedding (rotate-half convention) applied in place to the q and k heads of a fused
// qkv row [Nq*D | Nkv*D | Nkv*D]. inv_freq[i] = theta^(-2i/D); sign=-1 applies the inverse rotation
// (backward). Angles are computed in fp32 and cos/sin are rounded to bf16 as the reference module does.
// ------------------------------------------------------------------------------------------------
__global__ void rope_kernel(__nv_bfloat16* __restrict__ qkv, const long long* __restrict__ pos, int T, int n_rot_heads,
                            int D, long long ld, float log2_theta, float sign) {
  // one block per token; cos/sin of the D/2 frequencies computed once and shared by all heads
  extern __shared__ float cs[];  // [D/2] cos, [D/2] sin
  const int t = blockIdx.x;
  const int half = D >> 1;
  const float p = static_cast<float>(pos[t]);
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    float c, s;
    rope_cos_sin(p, i, D, log2_theta, c, s);
    cs[i] = c;
    cs[half + i] = s * sign;
  }
  __syncthreads();
  __nv_bfloat16* row = qkv + t * ld;
  const int pairs = half >> 1;  // bf16x2 pairs per half
  for (int idx = threadIdx.x; idx < n_rot_heads * pairs; idx += blockDim.x) {
    const int h = idx / pairs;
    const int i = (idx % pairs) * 2;
    __nv_bfloat162* a = reinterpret_cast<__nv_bfloat162*>(row + h * D + i);
    __nv_bfloat162* b = reinterpret_cast<__nv_bfloat162*>(row + h * D + i + half);
    const float2 x1 = __bfloat1622float2(*a);
    const float2 x2 = __bfloat1622float2(*b);
    const float c0 = cs[i], c1 = cs[i + 1], s0 = cs[half + i], s1 = cs[half + i + 1];
    *a = __floats2bfloat162_rn(x1.x * c0 - x2.x * s0, x1.y * c1 - x2.y * s1);
    *b = __floats2bfloat162_rn(x2.x * c0 + x1.x * s0, x2.y * c1 + x1.y * s1);
  }
}

// ------------------------------------------------------------------------------------------------
// SwiGLU on a fused gate|up row: h = silu(g) * u ; backward gives d(gate|up).
// ------------------------------------------------------------------------------------------------
__global__ void swiglu_fwd_kernel(const __nv_bfloat16* __restrict__ gu, __nv_bfloat16* __restrict__ h, int T, int I) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const long long total = static_cast<long long>(T) * I;
  if (idx >= total) return;
  const long long t = idx / I;
  const int c = static_cast<int>(idx % I);
  const __nv_bfloat16* row = gu + t * 2 * I;
  const uint4 g = *reinterpret_cast<const uint4*>(row + c);
  const uint4 u = *reinterpret_cast<const uint4*>(row + I + c);
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fg = unpack_bf16x2(gw[i]), fu = unpack_bf16x2(uw[i]);
    // act(gate) is rounded to the activation dtype before the product, as in the reference module.
    o[i] = pack_bf16x2(swiglu_h(fg.x, fu.x), swiglu_h(fg.y, fu.y));
  }
  *reinterpret_cast<uint4*>(h + idx) = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void swiglu_bwd_kernel(const __nv_bfloat16* __restrict__ dh, const __nv_bfloat16* __restrict__ gu,
                                  __nv_bfloat16* __restrict__ dgu, int T, int I) {
  const long long idx = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const long long total = static_cast<long long>(T) * I;
  if (idx >= total) return;
  const long long t = idx / I;
  const int c = static_cast<int>(idx % I);
  const __nv_bfloat16* row = gu + t * 2 * I;
  const uint4 g = *reinterpret_cast<const uint4*>(row + c);
  const uint4 u = *reinterpret_cast<const uint4*>(row + I + c);
  const uint4 d = *reinterpret_cast<const uint4*>(dh + idx);
  const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w}, dw[4] = {d.x, d.y, d.z, d.w};
  uint32_t og[4], ou[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 fg = unpack_bf16x2(gw[i]), fu = unpack_bf16x2(uw[i]), fd = unpack_bf16x2(dw[i]);
    float r[2], s2[2];
    const float gg[2] = {fg.x, fg.y}, uu[2] = {fu.x, fu.y}, dd[2] = {fd.x, fd.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) swiglu_grads(gg[j], uu[j], dd[j], r[j], s2[j]);  // d gate, d up
    og[i] = pack_bf16x2(r[0], r[1]);
    ou[i] = pack_bf16x2(s2[0], s2[1]);
  }
  __nv_bfloat16* drow = dgu + t * 2 * I;
  *reinterpret_cast<uint4*>(drow + c) = make_uint4(og[0], og[1], og[2], og[3]);
  *reinterpret_cast<uint4*>(drow + I + c) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
}

// ------------------------------------------------------------------------------------------------
// Embedding
// ------------------------------------------------------------------------------------------------
__global__ void embedding_fwd_kernel(const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                     __nv_bfloat16* __restrict__ out, int T, int H, long long V) {
  const int t = blockIdx.x;
  const long long id = ids[t];
  if (!ACCERL_DBG_OK(id >= 0 && id < V, kDbgEmbeddingId, id)) return;
  const uint4* src = reinterpret_cast<const uint4*>(table + id * H);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<long long>(t) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

// grad[ids[t], :] += dout[t, :] in fp32 (atomic; rows of a packed batch rarely collide).
__global__ void embedding_bwd_kernel(const long long* __restrict__ ids, const __nv_bfloat16* __restrict__ dout,
                                     float* __restrict__ grad, int T, int H, long long V) {
  const int t = blockIdx.x;
  const long long id = ids[t];
  if (!ACCERL_DBG_OK(id >= 0 && id < V, kDbgEmbeddingId, id)) return;
  float* g = grad + id * H;
  const __nv_bfloat16* d = dout + static_cast<long long>(t) * H;
  for (int c = threadIdx.x * 2; c < H; c += blockDim.x * 2) {
    const float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(d + c));
    atomicAdd(g + c, v.x);
    atomicAdd(g + c + 1, v.y);
  }
}

}  // namespace accerl

using namespace accerl;

extern "C" int accerl_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int rows, int H, long long ldx,
                                  long long ldy, float eps, cudaStream_t s) {
  if (H % 8) return -1;
  const int warps = 8;
  rmsnorm_fwd_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, rstd, rows, H, ldx, ldy, eps);
  return (int)cudaGetLastError();
}

extern "C" int accerl_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, const void* dx_accum,
                                  void* dx, float* dw, float* workspace, int rows, int H, long long ld, int dw_accumulate,
                                  cudaStream_t s) {
  if (H % 8) return -1;
  if (dw && H % 256 == 0 && H <= 2048 && rows > 0) {
    // fused single pass: 8 warps per block, grid sized so every warp visits several rows
    const int nwarps_total = std::min((rows + 3) / 4, 148 * 16);
    const int blocks = (nwarps_total + 7) / 8;
#define RMS_BWD_CASE(NCV)                                                                                        \
  case NCV:                                                                                                      \
    rmsnorm_bwd_fused_kernel<NCV><<<blocks, 256, 0, s>>>(                                                        \
        (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, rstd,                        \
        (const __nv_bfloat16*)dx_accum, (__nv_bfloat16*)dx, workspace, rows, ld);                                \
    break;
    switch (H / 256) {
      RMS_BWD_CASE(1) RMS_BWD_CASE(2) RMS_BWD_CASE(4) RMS_BWD_CASE(6) RMS_BWD_CASE(8)
      default:
        goto generic;
    }
#undef RMS_BWD_CASE
    column_reduce_kernel<<<(H + 31) / 32, 256, 0, s>>>(workspace, dw, blocks, H, dw_accumulate);
    return (int)cudaGetLastError();
  }
generic:
  const int warps = 8;
  rmsnorm_bwd_kernel<<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, rstd, (const __nv_bfloat16*)dx_accum,
      (__nv_bfloat16*)dx, rows, H, ld);
  if (dw) {
    const int rpb = 64;
    const int nblk = (rows + rpb - 1) / rpb;
    dim3 grid(nblk, (H / 8 + 127) / 128);
    rmsnorm_dw_partial_kernel<<<grid, 128, 0, s>>>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, rstd, workspace,
                                                   rows, H, ld, rpb);
    column_reduce_kernel<<<(H + 31) / 32, 256, 0, s>>>(workspace, dw, nblk, H, dw_accumulate);
  }
  return (int)cudaGetLastError();
}

extern "C" int accerl_bias_grad(const void* dy, float* db, float* workspace, int rows, int N, long long ld,
                                int accumulate, cudaStream_t s) {
  if (N % 8) return -1;
  const int rpb = 64;
  const int nblk = (rows + rpb - 1) / rpb;
  dim3 grid(nblk, (N / 8 + 127) / 128);
  colsum_partial_kernel<<<grid, 128, 0, s>>>((const __nv_bfloat16*)dy, workspace, rows, N, ld, rpb);
  column_reduce_kernel<<<(N + 31) / 32, 256, 0, s>>>(workspace, db, nblk, N, accumulate);
  return (int)cudaGetLastError();
}

extern "C" int accerl_rope(void* qkv, const long long* pos, int T, int n_rot_heads, int D, long long ld, float theta,
                           int inverse, cudaStream_t s) {
  if (T == 0) return 0;
  if (D % 4) return -1;
  rope_kernel<<<T, 256, D * sizeof(float), s>>>((__nv_bfloat16*)qkv, pos, T, n_rot_heads, D, ld, log2f(theta),
                                                inverse ? -1.f : 1.f);
  return (int)cudaGetLastError();
}

extern "C" int accerl_swiglu_fwd(const void* gu, void* h, int T, int I, cudaStream_t s) {
  if (I % 8) return -1;
  const long long total = (long long)T * I / 8;
  if (total == 0) return 0;
  swiglu_fwd_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>((const __nv_bfloat16*)gu, (__nv_bfloat16*)h, T, I);
  return (int)cudaGetLastError();
}

extern "C" int accerl_swiglu_bwd(const void* dh, const void* gu, void* dgu, int T, int I, cudaStream_t s) {
  if (I % 8) return -1;
  const long long total = (long long)T * I / 8;
  if (total == 0) return 0;
  swiglu_bwd_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>((const __nv_bfloat16*)dh, (const __nv_bfloat16*)gu,
                                                                     (__nv_bfloat16*)dgu, T, I);
  return (int)cudaGetLastError();
}

extern "C" int accerl_embedding_fwd(const long long* ids, const void* table, void* out, int T, int H, long long V,
                                    cudaStream_t s) {
  if (H % 8 || T == 0) return T == 0 ? 0 : -1;
  embedding_fwd_kernel<<<T, 128, 0, s>>>(ids, (const __nv_bfloat16*)table, (__nv_bfloat16*)out, T, H, V);
  return (int)cudaGetLastError();
}

extern "C" int accerl_embedding_bwd(const long long* ids, const void* dout, float* grad, int T, int H, long long V,
                                    cudaStream_t s) {
  if (T == 0) return 0;
  embedding_bwd_kernel<<<T, 256, 0, s>>>(ids, (const __nv_bfloat16*)dout, grad, T, H, V);
  return (int)cudaGetLastError();
}

ACCERL_DEBUG_EXPORT(elementwise)
