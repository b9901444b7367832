// Loss-side kernels (sm_100a):
//  * LM-head log-softmax over bf16 logits rows: label log-probability, log-sum-exp and entropy;
//    backward writes d(logits) = g * (onehot - softmax) in place.
//  * Fused PPO / GIPO / SAPO objective with the k3 KL term: one pass produces d(loss)/d(logprob)
//    (already scaled by the caller's loss scale) and the float64 [policy_sum, k3_sum, clip_count]
//    statistics vector.
//  * Global gradient norm and the fused clip + AdamW update over a flat fp32 shard (fp32 master,
//    m, v), writing the bf16 compute copy and zeroing the gradient for the next accumulation.
#include "common.cuh"

namespace accerl {

template <int THREADS>
__device__ __forceinline__ void block_reduce_max_sum(float& m, float& s, float& t) {
  // combine (max, sumexp, sum(exp*logit)) triples across the block
  __shared__ float sm_m[THREADS / 32], sm_s[THREADS / 32], sm_t[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float t2 = __shfl_xor_sync(0xffffffffu, t, o);
    const float mn = fmaxf(m, m2);
    const float a = (m == -INFINITY) ? 0.f : __expf(m - mn);
    const float b = (m2 == -INFINITY) ? 0.f : __expf(m2 - mn);
    s = s * a + s2 * b;
    t = t * a + t2 * b;
    m = mn;
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sm_m[w] = m;
    sm_s[w] = s;
    sm_t[w] = t;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < THREADS / 32 ? sm_m[threadIdx.x] : -INFINITY;
    s = threadIdx.x < THREADS / 32 ? sm_s[threadIdx.x] : 0.f;
    t = threadIdx.x < THREADS / 32 ? sm_t[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float t2 = __shfl_xor_sync(0xffffffffu, t, o);
      const float mn = fmaxf(m, m2);
      const float a = (m == -INFINITY) ? 0.f : __expf(m - mn);
      const float b = (m2 == -INFINITY) ? 0.f : __expf(m2 - mn);
      s = s * a + s2 * b;
      t = t * a + t2 * b;
      m = mn;
    }
    if (threadIdx.x == 0) {
      sm_m[0] = m;
      sm_s[0] = s;
      sm_t[0] = t;
    }
  }
  __syncthreads();
  m = sm_m[0];
  s = sm_s[0];
  t = sm_t[0];
}

template <int THREADS>
__global__ void __launch_bounds__(THREADS) logsoftmax_label_fwd_kernel(const __nv_bfloat16* __restrict__ logits,
                                                                      long long ld, const long long* __restrict__ labels,
                                                                      float* __restrict__ logprob, float* __restrict__ lse_out,
                                                                      float* __restrict__ entropy, int V) {
  const int row = blockIdx.x;
  const __nv_bfloat16* l = logits + row * ld;
  float m = -INFINITY, s = 0.f, t = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += THREADS * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(l + c);
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = unpack_bf16x2(vw[i]);
      f[2 * i] = p.x;
      f[2 * i + 1] = p.y;
    }
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float mn = fmaxf(m, lm);
    const float a = (m == -INFINITY) ? 0.f : __expf(m - mn);
    s *= a;
    t *= a;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float e = __expf(f[i] - mn);
      s += e;
      t += e * f[i];
    }
    m = mn;
  }
  block_reduce_max_sum<THREADS>(m, s, t);
  if (threadIdx.x == 0) {
    const float lse = m + logf(s);
    const long long lab = labels[row];
    const float ll = (lab >= 0 && lab < V) ? __bfloat162float(l[lab]) : 0.f;
    logprob[row] = ll - lse;
    if (lse_out) lse_out[row] = lse;
    if (entropy) entropy[row] = lse - t / s;
  }
}

// dlogits = g[row] * (onehot(label) - softmax); written over the logits buffer.
// The logits may be one vocabulary chunk [label_offset, label_offset + V) of the full row: the label's
// one-hot term applies only when the label falls in the chunk.
__global__ void logsoftmax_label_bwd_kernel(__nv_bfloat16* __restrict__ logits, long long ld,
                                            const long long* __restrict__ labels, const float* __restrict__ lse,
                                            const float* __restrict__ grad, int V, long long label_offset) {
  const int row = blockIdx.x;
  __nv_bfloat16* l = logits + row * ld;
  const float z = lse[row];
  const float g = grad[row];
  const long long lab = labels[row] - label_offset;
  for (int c = threadIdx.x * 8; c < V; c += blockDim.x * 8) {
    uint4 v = *reinterpret_cast<const uint4*>(l + c);
    uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 p = unpack_bf16x2(vw[i]);
      float d0 = -g * __expf(p.x - z);
      float d1 = -g * __expf(p.y - z);
      if (lab == c + 2 * i) d0 += g;
      if (lab == c + 2 * i + 1) d1 += g;
      vw[i] = pack_bf16x2(d0, d1);
    }
    *reinterpret_cast<uint4*>(l + c) = make_uint4(vw[0], vw[1], vw[2], vw[3]);
  }
}

// One vocabulary chunk of the response-only LM head: logits [rows, V] of columns [c0, c0 + V). Folds
// the chunk into each row's running (max m, sum exp(x - m), sum exp(x - m) x, label logit); first
// chunk initialises the state. One CTA per row; the full [rows, vocab] logits never exist.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) lse_chunk_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                           const long long* __restrict__ labels, long long c0,
                                                           int V, int first, float* __restrict__ state) {
  const int row = blockIdx.x;
  const __nv_bfloat16* l = logits + row * ld;
  float m = -INFINITY, sum = 0.f, t = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += THREADS * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(l + c);
    const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 q = unpack_bf16x2(vw[i]);
      f[2 * i] = q.x;
      f[2 * i + 1] = q.y;
    }
    float lm = f[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) lm = fmaxf(lm, f[i]);
    const float mn = fmaxf(m, lm);
    const float a = (m == -INFINITY) ? 0.f : __expf(m - mn);
    sum *= a;
    t *= a;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float e = __expf(f[i] - mn);
      sum += e;
      t += e * f[i];
    }
    m = mn;
  }
  block_reduce_max_sum<THREADS>(m, sum, t);
  if (threadIdx.x == 0) {
    float* st = state + 4ll * row;  // [m, sum, t, label logit]
    const long long lab = labels[row] - c0;
    const bool has_label = lab >= 0 && lab < V;
    if (first) {
      st[0] = m;
      st[1] = sum;
      st[2] = t;
      st[3] = has_label ? __bfloat162float(l[lab]) : 0.f;
    } else {
      const float m0 = st[0];
      const float mn = fmaxf(m0, m);
      const float a0 = (m0 == -INFINITY) ? 0.f : __expf(m0 - mn);
      const float a1 = (m == -INFINITY) ? 0.f : __expf(m - mn);
      st[0] = mn;
      st[1] = st[1] * a0 + sum * a1;
      st[2] = st[2] * a0 + t * a1;
      if (has_label) st[3] = __bfloat162float(l[lab]);
    }
  }
}

// Row results from the folded state: label log-probability, log-sum-exp and (optionally) entropy.
__global__ void lse_finish_kernel(const float* __restrict__ state, int rows, float* __restrict__ logprob,
                                  float* __restrict__ lse_out, float* __restrict__ entropy) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* st = state + 4ll * row;
  const float lse = st[0] + logf(st[1]);
  logprob[row] = st[3] - lse;
  lse_out[row] = lse;
  if (entropy) entropy[row] = lse - st[2] / st[1];
}

// ------------------------------------------------------------------------------------------------
// Fused policy objective
// ------------------------------------------------------------------------------------------------
struct PolicyCfg {
  int mode;  // 0 ppo, 1 gipo, 2 sapo, 3 none (advantage x logprob, no ratio)
  float clip_eps, gipo_sigma, tau_pos, tau_neg, kl_coef, loss_scale;
};

__global__ void policy_loss_kernel(const float* __restrict__ lp, const float* __restrict__ old_lp,
                                   const float* __restrict__ adv, float* __restrict__ dlp, double* __restrict__ stats,
                                   int n, PolicyCfg cfg) {
  float obj_sum = 0.f, k3_sum = 0.f, clips = 0.f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float log_ratio = lp[i] - old_lp[i];
    const float r = expf(log_ratio);
    const float A = adv[i];
    float obj, dobj;
    if (cfg.mode == 0) {
      const float lo = 1.f - cfg.clip_eps, hi = 1.f + cfg.clip_eps;
      const float rc = fminf(fmaxf(r, lo), hi);
      const float s1 = r * A, s2 = rc * A;
      const float in_range = (r >= lo && r <= hi) ? 1.f : 0.f;
      if (s1 < s2) {
        obj = s1;
        dobj = A * r;
      } else if (s1 > s2) {
        obj = s2;
        dobj = A * r * in_range;
      } else {
        obj = s1;
        dobj = 0.5f * A * r + 0.5f * A * r * in_range;
      }
      if (r < lo || r > hi) clips += 1.f;
    } else if (cfg.mode == 1) {
      const float rd = fmaxf(r, 1e-9f);
      const float z = logf(rd) / cfg.gipo_sigma;
      const float coeff = expf(-0.5f * z * z);
      obj = r * A * coeff;
      dobj = A * coeff * r;
    } else if (cfg.mode == 3) {
      obj = A * lp[i];
      dobj = A;
    } else {
      const float rc = fminf(fmaxf(r, 1e-6f), 1e6f);
      const float tau = A > 0.f ? cfg.tau_pos : cfg.tau_neg;
      const float sig = 1.f / (1.f + expf(-tau * (rc - 1.f)));
      obj = sig * (4.f / tau) * A;
      const float in_range = (r >= 1e-6f && r <= 1e6f) ? 1.f : 0.f;
      dobj = 4.f * A * sig * (1.f - sig) * r * in_range;
    }
    const float k3 = r - 1.f - log_ratio;
    obj_sum += obj;
    k3_sum += k3;
    dlp[i] = cfg.loss_scale * (-dobj + cfg.kl_coef * (r - 1.f));
  }
  obj_sum = warp_sum(obj_sum);
  k3_sum = warp_sum(k3_sum);
  clips = warp_sum(clips);
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(&stats[0], static_cast<double>(-obj_sum));
    atomicAdd(&stats[1], static_cast<double>(k3_sum));
    atomicAdd(&stats[2], static_cast<double>(clips));
  }
}

// ------------------------------------------------------------------------------------------------
// Gradient norm and fused clip + AdamW on flat shards
// ------------------------------------------------------------------------------------------------
__global__ void sumsq_kernel(const float* __restrict__ g, long long n, double* __restrict__ out) {
  float acc = 0.f;
  const long long n4 = n / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = g4[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long long i = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    acc += g[i] * g[i];
  acc = warp_sum(acc);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(out, static_cast<double>(v));
  }
}

struct AdamCfg {
  float lr, beta1, beta2, eps, weight_decay, max_norm;
  float bc1, bc2_sqrt;  // 1 - beta1^t, sqrt(1 - beta2^t)
};

// sumsq points at the (already all-reduced) global sum of squared gradients. The clip coefficient
// follows torch.nn.utils.clip_grad_norm_: min(1, max_norm / (norm + 1e-6)).
__global__ void adamw_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                             float* __restrict__ grad, __nv_bfloat16* __restrict__ param, long long n,
                             const double* __restrict__ sumsq, AdamCfg c) {
  float coef = 1.f;
  if (c.max_norm > 0.f) {
    const float norm = static_cast<float>(sqrt(*sumsq));
    coef = fminf(1.f, c.max_norm / (norm + 1e-6f));
  }
  const float step = c.lr / c.bc1;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float g = grad[i] * coef;
    float p = master[i];
    p -= c.lr * c.weight_decay * p;
    const float mi = c.beta1 * m[i] + (1.f - c.beta1) * g;
    const float vi = c.beta2 * v[i] + (1.f - c.beta2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi) / c.bc2_sqrt + c.eps;
    p -= step * mi / denom;
    master[i] = p;
    param[i] = __float2bfloat16(p);
    grad[i] = 0.f;
  }
}

}  // namespace accerl

using namespace accerl;

extern "C" int accerl_logsoftmax_label_fwd(const void* logits, long long ld, const long long* labels, float* logprob,
                                           float* lse, float* entropy, int rows, int V, cudaStream_t s) {
  if (V % 8 || ld % 8) return -1;
  if (rows == 0) return 0;
  logsoftmax_label_fwd_kernel<512><<<rows, 512, 0, s>>>((const __nv_bfloat16*)logits, ld, labels, logprob, lse, entropy, V);
  return (int)cudaGetLastError();
}

extern "C" int accerl_logsoftmax_label_bwd(void* logits, long long ld, const long long* labels, const float* lse,
                                           const float* grad, int rows, int V, long long label_offset,
                                           cudaStream_t s) {
  if (V % 8 || ld % 8) return -1;
  if (rows == 0) return 0;
  logsoftmax_label_bwd_kernel<<<rows, 512, 0, s>>>((__nv_bfloat16*)logits, ld, labels, lse, grad, V, label_offset);
  return (int)cudaGetLastError();
}

// Fold the vocabulary chunk [c0, c0 + V) held in logits into the per-row state (4 floats per row).
extern "C" int accerl_lse_chunk(const void* logits, long long ld, const long long* labels, long long c0, int rows,
                                int V, int first, float* state, cudaStream_t s) {
  if (V % 8 || ld % 8) return -1;
  if (rows == 0) return 0;
  lse_chunk_kernel<512><<<rows, 512, 0, s>>>((const __nv_bfloat16*)logits, ld, labels, c0, V, first, state);
  return (int)cudaGetLastError();
}

extern "C" int accerl_lse_finish(const float* state, int rows, float* logprob, float* lse, float* entropy,
                                 cudaStream_t s) {
  if (rows == 0) return 0;
  lse_finish_kernel<<<(rows + 255) / 256, 256, 0, s>>>(state, rows, logprob, lse, entropy);
  return (int)cudaGetLastError();
}

extern "C" int accerl_policy_loss(const float* lp, const float* old_lp, const float* adv, float* dlp, double* stats,
                                  int n, int mode, float clip_eps, float gipo_sigma, float tau_pos, float tau_neg,
                                  float kl_coef, float loss_scale, cudaStream_t s) {
  if (n == 0) return 0;
  PolicyCfg cfg{mode, clip_eps, gipo_sigma, tau_pos, tau_neg, kl_coef, loss_scale};
  const int blocks = (n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024;
  policy_loss_kernel<<<blocks, 256, 0, s>>>(lp, old_lp, adv, dlp, stats, n, cfg);
  return (int)cudaGetLastError();
}

extern "C" int accerl_sumsq(const float* g, long long n, double* out, cudaStream_t s) {
  if (n == 0) return 0;
  long long blocks = (n / 4 + 255) / 256;
  if (blocks > 2048) blocks = 2048;
  if (blocks < 1) blocks = 1;
  sumsq_kernel<<<(unsigned)blocks, 256, 0, s>>>(g, n, out);
  return (int)cudaGetLastError();
}

extern "C" int accerl_adamw(float* master, float* m, float* v, float* grad, void* param, long long n,
                            const double* sumsq, float lr, float beta1, float beta2, float eps, float weight_decay,
                            float max_norm, float bc1, float bc2_sqrt, cudaStream_t s) {
  if (n == 0) return 0;
  AdamCfg c{lr, beta1, beta2, eps, weight_decay, max_norm, bc1, bc2_sqrt};
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  adamw_kernel<<<(unsigned)blocks, 256, 0, s>>>(master, m, v, grad, (__nv_bfloat16*)param, n, sumsq, c);
  return (int)cudaGetLastError();
}
