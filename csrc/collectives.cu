// Optimizer-step collectives over NVLink peer memory, fused with their compute (sm_100a).
//
//  rs_sumsq     reduce-scatter fused with the global-norm partial: rank r reads its shard range
//               [r*S, (r+1)*S) of every peer's full fp32 gradient buffer with vectorised P2P loads,
//               writes the fp32 sum to its gradient shard and accumulates sum(g^2) into one double.
//  adamw_push   clip (by the all-reduced norm) + AdamW on the fp32 shard, then the all-gather half:
//               the updated bf16 parameter shard is stored into the same range of every peer's full
//               bf16 parameter buffer (P2P stores), so no separate all-gather runs.
// Peer buffers are mapped once (CUDA IPC) and passed as device arrays of base pointers. Plain loads
// and stores only: no TMA, no multicast.
#include "common.cuh"

namespace accerl {

__global__ void rs_sumsq_kernel(const float* const* __restrict__ peers, int world, int rank, long long shard,
                                float* __restrict__ out, double* __restrict__ sumsq) {
  const long long base = static_cast<long long>(rank) * shard;
  const long long n4 = shard / 4;
  float acc2 = 0.f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const int peer = (rank + r) % world;  // stagger the start so ranks hit different peers first
      const float4 v = reinterpret_cast<const float4*>(peers[peer] + base)[i];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    reinterpret_cast<float4*>(out)[i] = s;
    acc2 += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
  }
  for (long long i = n4 * 4 + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < shard;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += peers[r][base + i];
    out[i] = s;
    acc2 += s * s;
  }
  acc2 = warp_sum(acc2);
  __shared__ float red[32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc2;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(sumsq, static_cast<double>(v));
  }
}

struct PushCfg {
  float lr, beta1, beta2, eps, weight_decay, max_norm, bc1, bc2_sqrt;
};

__global__ void adamw_push_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                                  const float* __restrict__ grad, __nv_bfloat16* const* __restrict__ peer_params,
                                  int world, int rank, long long shard, const double* __restrict__ sumsq, PushCfg c) {
  float coef = 1.f;
  if (c.max_norm > 0.f) coef = fminf(1.f, c.max_norm / (static_cast<float>(sqrt(*sumsq)) + 1e-6f));
  const float step = c.lr / c.bc1;
  const long long base = static_cast<long long>(rank) * shard;
  const long long n2 = shard / 2;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n2;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float out[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const long long j = 2 * i + h;
      const float g = grad[j] * coef;
      float p = master[j];
      p -= c.lr * c.weight_decay * p;
      const float mi = c.beta1 * m[j] + (1.f - c.beta1) * g;
      const float vi = c.beta2 * v[j] + (1.f - c.beta2) * g * g;
      m[j] = mi;
      v[j] = vi;
      p -= step * mi / (sqrtf(vi) / c.bc2_sqrt + c.eps);
      master[j] = p;
      out[h] = p;
    }
    const __nv_bfloat162 b = __floats2bfloat162_rn(out[0], out[1]);
    for (int r = 0; r < world; ++r) {
      const int peer = (rank + r) % world;
      reinterpret_cast<__nv_bfloat162*>(peer_params[peer] + base)[i] = b;
    }
  }
  if ((shard & 1) && blockIdx.x == 0 && threadIdx.x == 0) {
    const long long j = shard - 1;
    const float g = grad[j] * coef;
    float p = master[j] * (1.f - c.lr * c.weight_decay);
    const float mi = c.beta1 * m[j] + (1.f - c.beta1) * g;
    const float vi = c.beta2 * v[j] + (1.f - c.beta2) * g * g;
    m[j] = mi;
    v[j] = vi;
    p -= step * mi / (sqrtf(vi) / c.bc2_sqrt + c.eps);
    master[j] = p;
    for (int r = 0; r < world; ++r) peer_params[r][base + j] = __float2bfloat16(p);
  }
  __threadfence_system();
}

// Row copy to arbitrary (local or peer) addresses: row i of the source (src_row[i], or i when null) is
// stored at dst_addr[i] (0 = skip). One warp per row, 16-byte P2P stores. Used for the expert-parallel
// dispatch of tokens (and of their gradients) into the owning rank's receive buffer.
__global__ void row_scatter_kernel(const __nv_bfloat16* __restrict__ src, long long ld, const long long* __restrict__ src_row,
                                   const long long* __restrict__ dst_addr, long long n, int H) {
  const long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= n) return;
  const long long dst = dst_addr[w];
  if (dst == 0) return;
  const long long r = src_row ? src_row[w] : w;
  const uint4* s = reinterpret_cast<const uint4*>(src + r * ld);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int c = lane; c < H / 8; c += 32) d[c] = s[c];
}

// Trainer -> engine weight pull: a list of 2-D copies desc[i] = {src_off, src_ld, dst_off, dst_ld,
// rows, cols} (elements) from a source buffer (the trainer's flat parameters, normally another GPU's
// memory mapped by CUDA IPC) into the local flat parameter buffer. Work is split into units of one
// row chunk of at most kPullChunk elements; unit_start[i] is the first unit of descriptor i. One warp
// per unit, 16-byte loads and stores where both addresses allow, element copies otherwise.
constexpr int kPullChunk = 4096;

__global__ void weight_pull_kernel(const long long* __restrict__ desc, const long long* __restrict__ unit_start,
                                   int n_desc, const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst) {
  const long long n_units = unit_start[n_desc];
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (long long u = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; u < n_units; u += warps) {
    int lo = 0, hi = n_desc;  // unit_start[lo] <= u < unit_start[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (unit_start[mid] <= u) lo = mid;
      else hi = mid;
    }
    const long long* d = desc + 6 * lo;
    const long long cols = d[5];
    const long long per_row = (cols + kPullChunk - 1) / kPullChunk;
    const long long local = u - unit_start[lo];
    const long long row = local / per_row;
    const long long c0 = (local % per_row) * kPullChunk;
    const long long c1 = min(cols, c0 + kPullChunk);
    const __nv_bfloat16* s = src + d[0] + row * d[1];
    __nv_bfloat16* t = dst + d[2] + row * d[3];
    const bool vec = (((reinterpret_cast<uintptr_t>(s + c0) | reinterpret_cast<uintptr_t>(t + c0)) & 15) == 0);
    long long c = c0;
    if (vec) {
      const long long nv = (c1 - c0) / 8;
      const uint4* sv = reinterpret_cast<const uint4*>(s + c0);
      uint4* tv = reinterpret_cast<uint4*>(t + c0);
      for (long long i = lane; i < nv; i += 32) tv[i] = sv[i];
      c = c0 + nv * 8;
    }
    for (long long i = c + lane; i < c1; i += 32) t[i] = s[i];
  }
}

// One-shot all-reduce of bf16 partial sums for tensor-parallel (row-parallel) layers, over NVLink
// peer memory. Every rank's partial for this call sits in slot `slot` of its symmetric buffer
// (element offset slot * slot_elems). Block 0 publishes `epoch` into flags_r[slot][rank] of every
// rank r (system-scope release); every block then waits (bounded) until this rank's flags[slot][src]
// equal `epoch` for all src, sums all ranks' partials in rank order (identical result on every rank)
// plus the optional residual, and writes `out`. epoch = *ctr + 1; the last block to finish stores it
// back into *ctr, so the count lives on the device and CUDA-graph replays advance it. Ranks issue the
// same calls in the same order, alternating slots, so a rank can be at most one call ahead and a
// slot is never overwritten while a peer still reads it. On timeout the status word is set and the
// kernel returns without writing.
__global__ void tp_allreduce_kernel(const long long* __restrict__ peer_data, const long long* __restrict__ peer_flags,
                                    int world, int rank, int slot, long long slot_elems, long long n,
                                    const __nv_bfloat16* __restrict__ residual, __nv_bfloat16* __restrict__ out,
                                    int* ctr, int* done, int* status) {
  __shared__ int epoch_s, ok_s;
  if (threadIdx.x == 0) {
    const int epoch = *reinterpret_cast<volatile int*>(ctr) + 1;
    epoch_s = epoch;
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int r = 0; r < world; ++r)
        st_release_sys(reinterpret_cast<int*>(peer_flags[r]) + slot * world + rank, epoch);
    }
    const int* mine = reinterpret_cast<const int*>(peer_flags[rank]) + slot * world;
    int ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int r = 0; r < world && ok; ++r) {
      while (ld_acquire_sys(mine + r) != epoch) {
        if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
          atomicExch(status, kStatusTimeoutPeer);
          ok = 0;
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  if (ok_s) {
    const long long base = static_cast<long long>(slot) * slot_elems;
    const long long n8 = n / 8;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += static_cast<long long>(gridDim.x) * blockDim.x) {
      float acc[8];
      if (residual) {
        const uint4 r = *reinterpret_cast<const uint4*>(residual + 8 * i);
        const uint32_t rw[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(rw[j]);
          acc[2 * j] = f.x;
          acc[2 * j + 1] = f.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      }
      for (int r = 0; r < world; ++r) {
        const uint4 v = ld_cg_v4(reinterpret_cast<const __nv_bfloat16*>(peer_data[r]) + base + 8 * i);
        const uint32_t vw[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(vw[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16x2(acc[0], acc[1]);
      o.y = pack_bf16x2(acc[2], acc[3]);
      o.z = pack_bf16x2(acc[4], acc[5]);
      o.w = pack_bf16x2(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(out + 8 * i) = o;
    }
    if (blockIdx.x == 0) {
      for (long long i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) {
        float a = residual ? __bfloat162float(residual[i]) : 0.f;
        for (int r = 0; r < world; ++r)
          a += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(peer_data[r])[base + i]);
        out[i] = __float2bfloat16(a);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1) == static_cast<int>(gridDim.x) - 1) {
      *done = 0;
      *ctr = epoch_s;
      __threadfence();
    }
  }
}

}  // namespace accerl

using namespace accerl;

extern "C" int accerl_tp_allreduce(const long long* peer_data, const long long* peer_flags, int world, int rank, int slot,
                                   long long slot_elems, long long n, const void* residual, void* out, int* ctr,
                                   int* status, cudaStream_t s) {
  if (n <= 0) return 0;
  if (world < 1 || world > 8 || slot < 0 || slot > 1 || n > slot_elems) return -1;
  long long blocks = (n / 8 + 255) / 256;
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  tp_allreduce_kernel<<<(unsigned)blocks, 256, 0, s>>>(peer_data, peer_flags, world, rank, slot, slot_elems, n,
                                                       (const __nv_bfloat16*)residual, (__nv_bfloat16*)out, ctr,
                                                       ctr + 1, status);
  return (int)cudaGetLastError();
}

extern "C" int accerl_weight_pull(const long long* desc, const long long* unit_start, int n_desc, long long n_units,
                                  const void* src, void* dst, cudaStream_t s) {
  if (n_desc <= 0 || n_units <= 0) return 0;
  long long blocks = (n_units + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  weight_pull_kernel<<<(unsigned)blocks, 256, 0, s>>>(desc, unit_start, n_desc, (const __nv_bfloat16*)src,
                                                      (__nv_bfloat16*)dst);
  return (int)cudaGetLastError();
}

extern "C" int accerl_row_scatter(const void* src, long long ld, const long long* src_row, const long long* dst_addr,
                                  long long n, int H, cudaStream_t s) {
  if (n <= 0) return 0;
  if (H % 8 || ld % 8) return -1;
  const long long threads = n * 32;
  row_scatter_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>((const __nv_bfloat16*)src, ld, src_row, dst_addr,
                                                                        n, H);
  return (int)cudaGetLastError();
}

extern "C" int accerl_enable_peer_access(int peer) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (peer == dev) return 0;
  int can = 0;
  cudaDeviceCanAccessPeer(&can, dev, peer);
  if (!can) return -1;
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return 0;
  }
  return (int)e;
}

extern "C" int accerl_rs_sumsq(const float* const* peers, int world, int rank, long long shard, float* out,
                               double* sumsq, cudaStream_t s) {
  if (shard <= 0) return 0;
  long long blocks = (shard / 4 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  rs_sumsq_kernel<<<(unsigned)blocks, 256, 0, s>>>(peers, world, rank, shard, out, sumsq);
  return (int)cudaGetLastError();
}

extern "C" int accerl_adamw_push(float* master, float* m, float* v, const float* grad, void* const* peer_params,
                                 int world, int rank, long long shard, const double* sumsq, float lr, float beta1,
                                 float beta2, float eps, float weight_decay, float max_norm, float bc1, float bc2_sqrt,
                                 cudaStream_t s) {
  if (shard <= 0) return 0;
  PushCfg c{lr, beta1, beta2, eps, weight_decay, max_norm, bc1, bc2_sqrt};
  long long blocks = (shard / 2 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  adamw_push_kernel<<<(unsigned)blocks, 256, 0, s>>>(master, m, v, grad, (__nv_bfloat16* const*)peer_params, world,
                                                     rank, shard, sumsq, c);
  return (int)cudaGetLastError();
}
