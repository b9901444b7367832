// Token sampler of the rollout engine (sm_100a), replacing the sampling stage of the reference's
// inference engine (vLLM SamplingParams with temperature / top_p / top_k and logprobs=1,
// accerl_agent/agent_textworld.py:1831-1839).
//
// A row of bf16 logits x is sampled from softmax(x / T) by inverse-CDF with one uniform per draw
// (counter-based SplitMix64 stream keyed by the row's (seed, offset)); T <= 0 takes the argmax
// (lowest index among equal maxima). The reported log-probability is that of the sampled token
// under the untempered softmax, log_softmax(x)[token]. Logits may be -inf (masked); a row with no
// finite logit returns token 0 with log-probability -inf.
//
// Plain rows (no top-k / top-p) take two kernels:
//   sample_partial_kernel  grid (rows, chunks): per chunk, max / argmax, then sum exp(x - max) and
//                          sum exp((x - max) / T). One exp per element (two when T != 1), no per-element
//                          random numbers, so the pass runs at memory speed.
//   sample_final_kernel    one CTA per row: merges the chunk partials, finds the chunk that holds
//                          u * sum, and scans only that chunk (1/chunks of the row) for the element.
// Rows with top_k > 0 (and < V) or top_p < 1 take sample_filtered_kernel, one 1024-thread CTA per row:
//   1. row max; 2. the top-k threshold on the order-preserving 16-bit key of bf16 by bisection over
//   counts (ties at the k-th value are kept, as a value threshold does); 3. sums over the kept set;
//   4. top-p by pivoted rejection: draw j from the kept set restricted to keys >= pivot; j belongs to
//   the nucleus iff the tempered mass of strictly larger keys is below top_p of the kept mass (the
//   "cumulative mass before the token < top_p" rule of a sorted implementation); otherwise every key
//   <= key(j) is outside the nucleus too, so the pivot moves above key(j) and the draw repeats on the
//   remaining mass, which is the same distribution conditioned on the nucleus. The row stays in L2
//   between passes.
#include <climits>

#include "sampler.cuh"

namespace accerl {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {  // SplitMix64 output function (Steele, Lea, Flood 2014)
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// Uniform in (0, 1) for draw `k` of a row.
__device__ __forceinline__ float row_uniform(uint64_t seed, uint64_t offset, uint32_t k) {
  const uint64_t h = mix64(seed ^ mix64(offset * 0x100000001b3ull + k));
  return (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

// Order-preserving 16-bit key of a bf16 bit pattern: larger value <=> larger key.
__device__ __forceinline__ uint32_t bf16_key(uint32_t bits) {
  return (bits & 0x8000u) ? (~bits & 0xFFFFu) : (bits | 0x8000u);
}

__device__ __forceinline__ bool row_filtered(int row, int V, float T, const int* top_k, const float* top_p) {
  if (T <= 0.f) return false;
  const int k = top_k ? top_k[row] : 0;
  const float p = top_p ? top_p[row] : 1.f;
  return (k > 0 && k < V) || p < 1.f;
}

// 8 consecutive bf16 values (16-byte aligned) as floats and as raw 16-bit patterns.
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&x)[8], uint32_t (&b)[8]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    b[2 * i] = w[i] & 0xFFFFu;
    b[2 * i + 1] = w[i] >> 16;
    x[2 * i] = __uint_as_float(b[2 * i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// ---- block-wide reductions (every thread gets the same result) ----
template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red may still be read by a previous call
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < NW; ++i) t += red[i];
  return t;
}

template <int NW>
__device__ __forceinline__ int block_sum_int(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) t += red[i];
  return t;
}

template <int NW>
__device__ __forceinline__ int block_max_int(int v, int* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = INT_MIN;
#pragma unroll
  for (int i = 0; i < NW; ++i) t = max(t, red[i]);
  return t;
}

// (max value, lowest index holding it)
template <int NW>
__device__ __forceinline__ void block_argmax(float& m, int& mi, float* redf, int* redi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, mi, o);
    if (m2 > m || (m2 == m && i2 < mi)) {
      m = m2;
      mi = i2;
    }
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    redf[threadIdx.x >> 5] = m;
    redi[threadIdx.x >> 5] = mi;
  }
  __syncthreads();
  m = -INFINITY;
  mi = INT_MAX;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    if (redf[i] > m || (redf[i] == m && redi[i] < mi)) {
      m = redf[i];
      mi = redi[i];
    }
  }
}

// Exclusive / inclusive prefix sums of v over the block in thread order, and the block total. The
// interval [excl, incl) of thread t+1 starts exactly (bit for bit) where thread t's ends, so the
// intervals partition [0, total) and exactly one thread owns any r in that range.
template <int NW>
__device__ __forceinline__ void block_scan(float v, float* wsum, float& excl, float& incl, float& total) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  float prev = __shfl_up_sync(0xffffffffu, x, 1);
  if (lane == 0) prev = 0.f;
  __syncthreads();
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = 0.f;
    for (int i = 0; i < NW; ++i) {
      const float t = wsum[i];
      wsum[i] = acc;
      acc += t;
    }
    wsum[NW] = acc;
  }
  __syncthreads();
  const float off = wsum[w];
  incl = off + x;
  excl = off + prev;
  total = wsum[NW];
}

// Inverse CDF over elements [c0, c1) of a row in element order: the first element whose cumulative
// weight exp((x - M) * invT) (0 for keys below min_key) exceeds r. Falls back to the last element of
// positive weight when rounding leaves r at or past the total; -1 if every weight is 0.
template <int NT>
__device__ int block_icdf(const __nv_bfloat16* l, int c0, int c1, float M, float invT, uint32_t min_key, float r,
                          float* wsum, int* redi, int* found) {
  constexpr int NW = NT / 32;
  if (threadIdx.x == 0) *found = -1;
  __syncthreads();
  float running = 0.f;
  int last_pos = -1;
  for (int base = c0; base < c1; base += NT * 8) {
    const int c = base + threadIdx.x * 8;
    float e[8];
    float tsum = 0.f;
    if (c < c1) {
      float x[8];
      uint32_t b[8];
      load8(l + c, x, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        e[j] = (bf16_key(b[j]) >= min_key) ? __expf((x[j] - M) * invT) : 0.f;
        tsum += e[j];
        if (e[j] > 0.f) last_pos = c + j;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = 0.f;
    }
    float excl, incl, total;
    block_scan<NW>(tsum, wsum, excl, incl, total);
    if (tsum > 0.f && running + excl <= r && r < running + incl) {
      float acc = running + excl;
      int pick = -1;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (e[j] > 0.f && pick < 0) {
          acc += e[j];
          if (r < acc) pick = c + j;
        }
      }
      if (pick < 0) {  // the in-thread sum rounded below r: take the thread's last positive element
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (e[j] > 0.f) pick = c + j;
      }
      *found = pick;
    }
    __syncthreads();
    if (*found >= 0) break;
    running += total;
  }
  const int f = *found;
  const int fallback = block_max_int<NW>(last_pos, redi);
  return f >= 0 ? f : fallback;
}

constexpr int kMaxPivotRounds = 64;

}  // namespace

__global__ void __launch_bounds__(256) sample_partial_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                            int V, const float* __restrict__ temperature,
                                                            const int* __restrict__ top_k,
                                                            const float* __restrict__ top_p, float* __restrict__ part,
                                                            int num_chunks) {
  constexpr int NT = 256, NW = NT / 32;
  __shared__ float redf[NW];
  __shared__ int redi[NW];
  const int row = blockIdx.x, chunk = blockIdx.y;
  const float T = temperature[row];
  if (row_filtered(row, V, T, top_k, top_p)) return;
  const float invT = T > 0.f ? 1.f / T : 1.f;
  const int per = (((V + num_chunks - 1) / num_chunks) + 7) & ~7;
  const int c0 = min(V, chunk * per), c1 = min(V, c0 + per);
  const __nv_bfloat16* l = logits + static_cast<long long>(row) * ld;
  float m = -INFINITY;
  int mi = INT_MAX;
  for (int c = c0 + threadIdx.x * 8; c < c1; c += NT * 8) {
    float x[8];
    uint32_t b[8];
    load8(l + c, x, b);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (x[j] > m) {
        m = x[j];
        mi = c + j;
      }
  }
  block_argmax<NW>(m, mi, redf, redi);
  float s = 0.f, st = 0.f;
  if (m != -INFINITY) {  // m is finite here, so x = -inf contributes exp(-inf) = 0, never NaN
    for (int c = c0 + threadIdx.x * 8; c < c1; c += NT * 8) {
      float x[8];
      uint32_t b[8];
      load8(l + c, x, b);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s += __expf(x[j] - m);
        if (invT != 1.f) st += __expf((x[j] - m) * invT);
      }
    }
  }
  s = block_sum<NW>(s, redf);
  st = (invT != 1.f) ? block_sum<NW>(st, redf) : s;
  if (threadIdx.x == 0) {
    float* dst = part + (static_cast<long long>(row) * num_chunks + chunk) * kSamplePartFloats;
    dst[0] = m;
    dst[1] = s;
    dst[2] = st;
    dst[3] = __int_as_float(mi);
  }
}

__global__ void __launch_bounds__(256) sample_final_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                          int V, const float* __restrict__ temperature,
                                                          const int* __restrict__ top_k,
                                                          const float* __restrict__ top_p,
                                                          const unsigned long long* __restrict__ seeds,
                                                          const long long* __restrict__ offsets,
                                                          const float* __restrict__ part, int num_chunks,
                                                          long long* __restrict__ out_tokens,
                                                          float* __restrict__ out_logprobs) {
  constexpr int NT = 256, NW = NT / 32;
  __shared__ float wsum[NW + 1];
  __shared__ int redi[NW];
  __shared__ int found;
  __shared__ float sh_f[3];  // row max, untempered sum, residual within the chosen chunk
  __shared__ int sh_i[2];    // argmax index, chosen chunk
  const int row = blockIdx.x;
  const float T = temperature[row];
  if (row_filtered(row, V, T, top_k, top_p)) return;
  const bool greedy = T <= 0.f;
  const float invT = greedy ? 1.f : 1.f / T;
  if (threadIdx.x == 0) {
    const float* p = part + static_cast<long long>(row) * num_chunks * kSamplePartFloats;
    float M = -INFINITY;
    int I = INT_MAX;
    for (int c = 0; c < num_chunks; ++c) {
      const float m = p[c * kSamplePartFloats];
      const int mi = __float_as_int(p[c * kSamplePartFloats + 3]);
      if (m > M || (m == M && mi < I)) {
        M = m;
        I = mi;
      }
    }
    float S = 0.f;
    int chunk = -1;
    float r = 0.f;
    if (M != -INFINITY) {
      float ST = 0.f;
      for (int c = 0; c < num_chunks; ++c) {
        const float m = p[c * kSamplePartFloats];
        if (m == -INFINITY) continue;
        S += p[c * kSamplePartFloats + 1] * __expf(m - M);
        ST += p[c * kSamplePartFloats + 2] * __expf((m - M) * invT);
      }
      if (!greedy) {
        const float target = row_uniform(seeds[row], static_cast<uint64_t>(offsets[row]), 0) * ST;
        float acc = 0.f;
        int last = -1;
        for (int c = 0; c < num_chunks; ++c) {
          const float m = p[c * kSamplePartFloats];
          if (m == -INFINITY) continue;
          const float w = p[c * kSamplePartFloats + 2] * __expf((m - M) * invT);
          if (w <= 0.f) continue;
          last = c;
          if (target < acc + w) {
            chunk = c;
            r = target - acc;
            break;
          }
          acc += w;
        }
        if (chunk < 0 && last >= 0) {  // rounding left the target past the last chunk
          chunk = last;
          r = INFINITY;
        }
      }
    }
    sh_f[0] = M;
    sh_f[1] = S;
    sh_f[2] = r;
    sh_i[0] = I;
    sh_i[1] = chunk;
  }
  __syncthreads();
  const float M = sh_f[0], S = sh_f[1], r = sh_f[2];
  const int I = sh_i[0], chunk = sh_i[1];
  const __nv_bfloat16* l = logits + static_cast<long long>(row) * ld;
  int tok;
  if (M == -INFINITY) {
    tok = 0;
  } else if (greedy || chunk < 0) {
    tok = I;
  } else {
    const int per = (((V + num_chunks - 1) / num_chunks) + 7) & ~7;
    const int c0 = min(V, chunk * per), c1 = min(V, c0 + per);
    tok = block_icdf<NT>(l, c0, c1, M, invT, 0u, r, wsum, redi, &found);
    if (tok < 0) tok = I;
  }
  if (threadIdx.x == 0) {
    out_tokens[row] = tok;
    out_logprobs[row] =
        (M == -INFINITY || !(S > 0.f)) ? -INFINITY : __bfloat162float(l[tok]) - (M + __logf(S));
  }
}

__global__ void __launch_bounds__(1024) sample_filtered_kernel(const __nv_bfloat16* __restrict__ logits, long long ld,
                                                              int V, const float* __restrict__ temperature,
                                                              const int* __restrict__ top_k,
                                                              const float* __restrict__ top_p,
                                                              const unsigned long long* __restrict__ seeds,
                                                              const long long* __restrict__ offsets,
                                                              long long* __restrict__ out_tokens,
                                                              float* __restrict__ out_logprobs) {
  constexpr int NT = 1024, NW = NT / 32;
  __shared__ float wsum[NW + 1];
  __shared__ float redf[NW];
  __shared__ int redi[NW];
  __shared__ int found;
  const int row = blockIdx.x;
  const float T = temperature[row];
  if (!row_filtered(row, V, T, top_k, top_p)) return;
  const float invT = 1.f / T;
  const int k = top_k ? top_k[row] : 0;
  const float pp = top_p ? top_p[row] : 1.f;
  const uint64_t seed = seeds[row];
  const uint64_t offset = static_cast<uint64_t>(offsets[row]);
  const __nv_bfloat16* l = logits + static_cast<long long>(row) * ld;

  // 1. row max and its index
  float M = -INFINITY;
  int mi = INT_MAX;
  for (int c = threadIdx.x * 8; c < V; c += NT * 8) {
    float x[8];
    uint32_t b[8];
    load8(l + c, x, b);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (x[j] > M) {
        M = x[j];
        mi = c + j;
      }
  }
  block_argmax<NW>(M, mi, redf, redi);
  if (M == -INFINITY) {
    if (threadIdx.x == 0) {
      out_tokens[row] = 0;
      out_logprobs[row] = -INFINITY;
    }
    return;
  }
  const uint32_t key_max = bf16_key(__bfloat16_as_ushort(l[mi]));

  // 2. top-k threshold: the largest key t with count(key >= t) >= k
  uint32_t tk = 0;
  if (k > 0 && k < V) {
    uint32_t lo = 0, hi = key_max;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) >> 1;
      int cnt = 0;
      for (int c = threadIdx.x * 8; c < V; c += NT * 8) {
        float x[8];
        uint32_t b[8];
        load8(l + c, x, b);
#pragma unroll
        for (int j = 0; j < 8; ++j) cnt += bf16_key(b[j]) >= mid;
      }
      cnt = block_sum_int<NW>(cnt, redi);
      if (cnt >= k) lo = mid;
      else hi = mid - 1;
    }
    tk = lo;
  }

  // 3. untempered sum over the row and tempered mass of the kept set
  float s = 0.f, sk = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += NT * 8) {
    float x[8];
    uint32_t b[8];
    load8(l + c, x, b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s += __expf(x[j] - M);
      if (bf16_key(b[j]) >= tk) sk += __expf((x[j] - M) * invT);
    }
  }
  const float S = block_sum<NW>(s, redf);
  const float SK = block_sum<NW>(sk, redf);

  // 4. draw from the kept set; top-p by pivoted rejection
  int tok = mi;
  uint32_t pivot = tk;
  float spiv = SK;
  const float bound = pp * SK;
  for (int round = 0; round < kMaxPivotRounds; ++round) {
    const float target = row_uniform(seed, offset, static_cast<uint32_t>(round)) * spiv;
    const int j = block_icdf<NT>(l, 0, V, M, invT, pivot, target, wsum, redi, &found);
    if (j < 0) break;  // nothing of positive weight left: keep the argmax, which is always kept
    if (pp >= 1.f) {
      tok = j;
      break;
    }
    const uint32_t kj = bf16_key(__bfloat16_as_ushort(l[j]));
    float g = 0.f;
    for (int c = threadIdx.x * 8; c < V; c += NT * 8) {
      float x[8];
      uint32_t b[8];
      load8(l + c, x, b);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (bf16_key(b[q]) > kj) g += __expf((x[q] - M) * invT);
    }
    const float G = block_sum<NW>(g, redf);
    if (G < bound) {
      tok = j;
      break;
    }
    pivot = kj + 1;
    spiv = G;
    if (!(spiv > 0.f)) break;
  }
  if (threadIdx.x == 0) {
    out_tokens[row] = tok;
    out_logprobs[row] = __bfloat162float(l[tok]) - (M + __logf(S));
  }
}

}  // namespace accerl

using namespace accerl;

// logits [rows, V] bf16 (row stride ld), temperature [rows] f32, top_k [rows] i32 (0 = off) and
// top_p [rows] f32 (1 = off) may be null, seeds / offsets [rows] 64-bit, part: rows * num_chunks * 4
// floats of workspace. Returns 0, -1 for a bad shape / alignment, or a cudaError_t code.
extern "C" int accerl_sample_logits(const void* logits, long long ld, int rows, int V, const float* temperature,
                                    const int* top_k, const float* top_p, const unsigned long long* seeds,
                                    const long long* offsets, long long* out_tokens, float* out_logprobs,
                                    float* part, int num_chunks, cudaStream_t s) {
  if (rows == 0) return 0;
  if (rows < 0 || V <= 0 || num_chunks < 1 || num_chunks > 64) return -1;
  if (V % 8 || ld % 8 || (reinterpret_cast<uintptr_t>(logits) & 15)) return -1;
  const auto* lg = static_cast<const __nv_bfloat16*>(logits);
  sample_partial_kernel<<<dim3(rows, num_chunks), 256, 0, s>>>(lg, ld, V, temperature, top_k, top_p, part,
                                                               num_chunks);
  sample_final_kernel<<<rows, 256, 0, s>>>(lg, ld, V, temperature, top_k, top_p, seeds, offsets, part, num_chunks,
                                           out_tokens, out_logprobs);
  if (top_k != nullptr || top_p != nullptr)
    sample_filtered_kernel<<<rows, 1024, 0, s>>>(lg, ld, V, temperature, top_k, top_p, seeds, offsets, out_tokens,
                                                 out_logprobs);
  return static_cast<int>(cudaGetLastError());
}
