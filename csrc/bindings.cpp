// Python bindings of the sm_100a kernels. Kernels live in .cu files without torch headers and
// expose extern "C" launchers; this file validates tensors and forwards raw pointers together with
// the current CUDA stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDACachingAllocator.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <tuple>
#include <vector>
#include <torch/extension.h>

extern "C" {
int accerl_gemm_bf16(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn, void* C,
                     long long ldc, int c_f32, int M, int N, int K, float alpha, float beta, const void* bias,
                     const void* residual, long long ldr, int* status, int block_n, int max_ctas, int splits,
                     cudaStream_t stream);
int accerl_gemm_rope_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M,
                          int N, int K, const void* bias, const long long* pos, int rope_cols, float theta, int* status,
                          int block_n, int max_ctas, cudaStream_t stream);
int accerl_gemm_glu_bf16(const void* X, long long ldx, const void* W, long long ldw, void* gu, long long ldgu, void* h,
                         long long ldh, int M, int I, int K, int* status, int block_n, int max_ctas,
                         cudaStream_t stream);
int accerl_gemm_dglu_bf16(const void* dY, long long lddy, const void* Wd, long long ldwd, const void* gu,
                          long long ldgu, void* dgu, long long lddgu, int M, int I, int K, int* status, int block_n,
                          int max_ctas, cudaStream_t stream);
int accerl_grouped_gemm_bf16(const void* A, long long lda, int a_mn, const void* B, long long ldb, int b_mn, void* C,
                             long long ldc, int c_f32, int M, int N, int K, long long b_rows_total, float beta, int mode,
                             const int* tile_expert, const int* group_row_start, const int* group_rows, int num_groups,
                             int b_group_stride, long long c_group_stride, const long long* row_dst, int* status,
                             cudaStream_t stream);
int accerl_row_scatter(const void* src, long long ld, const long long* src_row, const long long* dst_addr, long long n,
                       int H, cudaStream_t s);
int accerl_tp_allreduce(const long long* peer_data, const long long* peer_flags, int world, int rank, int slot,
                        long long slot_elems, long long n, const void* residual, void* out, int* ctr, int* status,
                        cudaStream_t s);
int accerl_moe_combine_fwd(const void* ys, const long long* pos, const float* w, long long T, int k, int H,
                           const void* residual, const void* shared, const float* sg, void* out, long long R,
                           cudaStream_t s);
int accerl_moe_combine_bwd(const void* dout, const void* ys, const long long* pos, const float* w, long long T, int k,
                           int H, void* dys, float* dw, long long R, cudaStream_t s);
int accerl_moe_router(const float* logits, long long ldl, int T, int E, int k, int norm_topk, float* probs, float* topw,
                      long long* topi, int* counts, float* sg, cudaStream_t s);
int accerl_moe_layout(const long long* topi, const float* topw, long long n, int k, int E, int lo, int El,
                      long long total, const void* h, int H, void* xs, int zero_pad, int* hist, long long* pos, float* w,
                      int* tile_expert, int* row_start, int* seg_rows, int* counts, cudaStream_t s);
int accerl_moe_router_bwd(const float* probs, const long long* topi, const float* topw, const float* dw, int T, int E,
                          int k, int norm_topk, const void* dout, const void* sy, const float* sg, int H, void* dgrad,
                          int E_pad, void* dsy, cudaStream_t s);
int accerl_weight_pull(const long long* desc, const long long* unit_start, int n_desc, long long n_units,
                       const void* src, void* dst, cudaStream_t s);
int accerl_splitk_finish(const float* acc, long long lda, const void* bias, const void* residual, long long ldr,
                         void* out, long long ldo, int M, int N, cudaStream_t stream);
int accerl_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int rows, int H, long long ldx,
                       long long ldy, float eps, cudaStream_t s);
int accerl_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, const void* dx_accum, void* dx,
                       float* dw, float* workspace, int rows, int H, long long ld, int dw_accumulate, cudaStream_t s);
int accerl_bias_grad(const void* dy, float* db, float* workspace, int rows, int N, long long ld, int accumulate,
                     cudaStream_t s);
int accerl_rope(void* qkv, const long long* pos, int T, int n_rot_heads, int D, long long ld, float theta, int inverse,
                cudaStream_t s);
int accerl_swiglu_fwd(const void* gu, void* h, int T, int I, cudaStream_t s);
int accerl_swiglu_bwd(const void* dh, const void* gu, void* dgu, int T, int I, cudaStream_t s);
int accerl_embedding_fwd(const long long* ids, const void* table, void* out, int T, int H, long long V, cudaStream_t s);
int accerl_embedding_bwd(const long long* ids, const void* dout, float* grad, int T, int H, long long V,
                         cudaStream_t s);
int accerl_logsoftmax_label_fwd(const void* logits, long long ld, const long long* labels, float* logprob, float* lse,
                                float* entropy, int rows, int V, cudaStream_t s);
int accerl_logsoftmax_label_bwd(void* logits, long long ld, const long long* labels, const float* lse,
                                const float* grad, int rows, int V, long long label_offset, cudaStream_t s);
int accerl_lse_chunk(const void* logits, long long ld, const long long* labels, long long c0, int rows, int V,
                     int first, float* state, cudaStream_t s);
int accerl_lse_finish(const float* state, int rows, float* logprob, float* lse, float* entropy, cudaStream_t s);
int accerl_policy_loss(const float* lp, const float* old_lp, const float* adv, float* dlp, double* stats, int n,
                       int mode, float clip_eps, float gipo_sigma, float tau_pos, float tau_neg, float kl_coef,
                       float loss_scale, cudaStream_t s);
int accerl_sumsq(const float* g, long long n, double* out, cudaStream_t s);
int accerl_adamw(float* master, float* m, float* v, float* grad, void* param, long long n, const double* sumsq,
                 float lr, float beta1, float beta2, float eps, float weight_decay, float max_norm, float bc1,
                 float bc2_sqrt, cudaStream_t s);
int accerl_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, const int* cu_seqlens,
                    const int* cu_seqlens_k, int num_seqs, int max_seqlen, int total_tokens, int total_k, int Hq,
                    int Hkv, long long ldq, long long ldk, long long ldv, long long ldo, float scale, int causal,
                    int* status, const int* block_table, int max_blocks, int block_size, cudaStream_t s);
int accerl_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                    float* delta, float* dq_acc, void* dq, void* dk, void* dv, const int* cu_seqlens, int num_seqs,
                    int max_seqlen, int total_tokens, int Hq, int Hkv, long long ldq, long long ldk, long long ldv,
                    long long ldo, long long lddo, long long lddq, long long lddk, long long lddv, float scale,
                    int causal, int* status, const long long* rope_pos, float rope_theta, cudaStream_t s);
int accerl_paged_decode_tc(const void* q, long long ldq, const void* k_cache, const void* v_cache, int num_blocks,
                           const int* block_table, int max_blocks, const int* seq_lens, float* part_o, float* part_ml,
                           int num_seqs, int Hq, int Hkv, int block_size, int num_splits, float scale, int* status,
                           cudaStream_t s);
int accerl_paged_decode_tq(const void* q, long long ldq, const void* k_cache, const void* v_cache, int num_blocks,
                           const int* block_table, int max_blocks, const int* seq_lens, float* part_o, float* part_ml,
                           int num_seqs, int Hq, int Hkv, int block_size, int num_splits, float scale, int* status,
                           cudaStream_t s);
int accerl_paged_decode_merge(const float* part_o, const float* part_ml, void* out, long long ldo, int num_seqs, int Hq,
                              int num_splits, cudaStream_t s);
int accerl_paged_decode(const void* q, const void* k_cache, const void* v_cache, const int* block_table,
                        const int* seq_lens, void* out, float* part_o, float* part_ml, int num_seqs, int Hq, int Hkv,
                        int max_blocks_per_seq, int block_size, int num_splits, float scale, long long ldq,
                        long long ldo, cudaStream_t s);
int accerl_enable_peer_access(int peer);
int accerl_debug_status_attention(long long* out, int reset);
int accerl_debug_status_elementwise(long long* out, int reset);
int accerl_debug_status_moe(long long* out, int reset);
int accerl_debug_status_rollout(long long* out, int reset);
int accerl_rs_sumsq(const float* const* peers, int world, int rank, long long shard, float* out, double* sumsq,
                    cudaStream_t s);
int accerl_adamw_push(float* master, float* m, float* v, const float* grad, void* const* peer_params, int world,
                      int rank, long long shard, const double* sumsq, float lr, float beta1, float beta2, float eps,
                      float weight_decay, float max_norm, float bc1, float bc2_sqrt, cudaStream_t s);
int accerl_qkv_rope_cache(void* qkv, long long ld, const long long* pos, const int* slots, int T, int Hq, int Hkv,
                          float theta, const void* q_norm, const void* k_norm, float eps, void* k_cache, void* v_cache,
                          long long num_slots, cudaStream_t s);
int accerl_kv_cache_write(const void* k, const void* v, void* k_cache, void* v_cache, const int* slot_mapping, int T,
                          int Hkv, long long ldk, long long ldv, long long num_slots, cudaStream_t s);
int accerl_sample_logits(const void* logits, long long ld, int rows, int V, const float* temperature,
                         const int* top_k, const float* top_p, const unsigned long long* seeds,
                         const long long* offsets, long long* out_tokens, float* out_logprobs, float* part,
                         int num_chunks, cudaStream_t s);
}

namespace {

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// Launch status of the most recent call on this thread; Python reads it through last_error() and
// raises there, so no C++ exception ever crosses the kernel-launch path.
thread_local int g_last_rc = 0;
thread_local const char* g_last_what = "";

void check(int rc, const char* what) {
  g_last_rc = rc;
  g_last_what = what;
}

std::tuple<int64_t, std::string> last_error() {
  const int rc = g_last_rc;
  std::string msg = g_last_what;
  if (rc > 0) msg += std::string(": ") + cudaGetErrorString(static_cast<cudaError_t>(rc));
  g_last_rc = 0;
  g_last_what = "";
  return {rc, msg};
}

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bfloat16")
#define CHECK_F32(x) TORCH_CHECK((x).scalar_type() == at::kFloat, #x " must be float32")
#define CHECK_I64(x) TORCH_CHECK((x).scalar_type() == at::kLong, #x " must be int64")
#define CHECK_I32(x) TORCH_CHECK((x).scalar_type() == at::kInt, #x " must be int32")

const void* opt_ptr(const c10::optional<at::Tensor>& t) { return t.has_value() ? t->data_ptr() : nullptr; }

int* status_ptr(const c10::optional<at::Tensor>& t) {
  return t.has_value() ? t->data_ptr<int>() : nullptr;
}

// Row-major 2-D view helpers: leading dimension = stride(0), last dim contiguous.
long long ld_of(const at::Tensor& t) {
  TORCH_CHECK(t.dim() == 2, "expected a 2-D tensor");
  TORCH_CHECK(t.stride(1) == 1, "last dimension must be contiguous");
  return t.stride(0);
}

// out = alpha * op(a) op(b) + beta*out (+bias)(+residual)
// a: [M,K] (a_mn=false) or [K,M] (a_mn=true); b: [N,K] (b_mn=false) or [K,N] (b_mn=true)
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, double alpha, double beta,
          const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& status, int64_t block_n, int64_t max_ctas, int64_t splits) {
  CHECK_CUDA(a);
  CHECK_CUDA(b);
  CHECK_CUDA(out);
  CHECK_BF16(a);
  CHECK_BF16(b);
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat, "out must be bf16 or f32");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  const int Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm: inner dimensions differ (", K, " vs ", Kb, ")");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: output shape mismatch");
  long long ldr = 0;
  if (residual.has_value()) {
    CHECK_BF16(*residual);
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N, "gemm: residual shape mismatch");
    ldr = ld_of(*residual);
  }
  if (bias.has_value()) {
    CHECK_BF16(*bias);
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous(), "gemm: bias must be contiguous [N]");
  }
  const c10::cuda::CUDAGuard guard(a.device());
  check(accerl_gemm_bf16(a.data_ptr(), ld_of(a), a_mn, b.data_ptr(), ld_of(b), b_mn, out.data_ptr(), ld_of(out),
                         out.scalar_type() == at::kFloat, M, N, K, static_cast<float>(alpha), static_cast<float>(beta),
                         opt_ptr(bias), opt_ptr(residual), ldr, status_ptr(status), static_cast<int>(block_n),
                         static_cast<int>(max_ctas), static_cast<int>(splits), cur_stream()),
        "gemm");
}

// out = x w^T (+ bias) with the rotary embedding applied to the first rope_cols columns (heads of 128)
// at positions pos (int64 [M]) in the epilogue.
void gemm_rope(const at::Tensor& x, const at::Tensor& w, at::Tensor& out, const c10::optional<at::Tensor>& bias,
               const at::Tensor& pos, int64_t rope_cols, double theta, const c10::optional<at::Tensor>& status,
               int64_t block_n, int64_t max_ctas) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(x));
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(out);
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.numel() == x.size(0), "gemm_rope: pos int64 [M]");
  TORCH_CHECK(w.size(1) == x.size(1) && out.size(0) == x.size(0) && out.size(1) == w.size(0), "gemm_rope: shapes");
  if (bias.has_value()) CHECK_BF16(*bias);
  check(accerl_gemm_rope_bf16(x.data_ptr(), ld_of(x), w.data_ptr(), ld_of(w), out.data_ptr(), ld_of(out), x.size(0),
                              w.size(0), x.size(1), opt_ptr(bias), reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()),
                              static_cast<int>(rope_cols), static_cast<float>(theta), status_ptr(status),
                              static_cast<int>(block_n), static_cast<int>(max_ctas), cur_stream()),
        "gemm_rope");
}

// h = silu(x Wg^T) * (x Wu^T) for w = [Wg; Wu] ([2I, K]); gu (optional, [M, 2I]) keeps the gate|up outputs.
void gemm_glu(const at::Tensor& x, const at::Tensor& w, const c10::optional<at::Tensor>& gu, at::Tensor& h,
              const c10::optional<at::Tensor>& status, int64_t block_n, int64_t max_ctas) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(x));
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(h);
  const int M = x.size(0), K = x.size(1), I = h.size(1);
  TORCH_CHECK(w.size(0) == 2 * I && w.size(1) == K, "gemm_glu: weight must be [2I, K]");
  TORCH_CHECK(h.size(0) == M, "gemm_glu: output rows");
  if (gu.has_value()) {
    CHECK_BF16(*gu);
    TORCH_CHECK(gu->size(0) == M && gu->size(1) == 2 * I, "gemm_glu: gu must be [M, 2I]");
  }
  check(accerl_gemm_glu_bf16(x.data_ptr(), ld_of(x), w.data_ptr(), ld_of(w), gu.has_value() ? gu->data_ptr() : nullptr,
                             gu.has_value() ? ld_of(*gu) : 0, h.data_ptr(), ld_of(h), M, I, K, status_ptr(status),
                             static_cast<int>(block_n), static_cast<int>(max_ctas), cur_stream()),
        "gemm_glu");
}

// dgu = SwiGLU backward of (dy Wd) given gu; dy [M, K], wd [K, I] (the down projection), gu/dgu [M, 2I].
void gemm_dglu(const at::Tensor& dy, const at::Tensor& wd, const at::Tensor& gu, at::Tensor& dgu,
               const c10::optional<at::Tensor>& status, int64_t block_n, int64_t max_ctas) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(dy));
  CHECK_CUDA(dy);
  CHECK_BF16(dy);
  CHECK_BF16(wd);
  CHECK_BF16(gu);
  CHECK_BF16(dgu);
  const int M = dy.size(0), K = dy.size(1), I = wd.size(1);
  TORCH_CHECK(wd.size(0) == K, "gemm_dglu: down weight must be [K, I]");
  TORCH_CHECK(gu.size(0) == M && gu.size(1) == 2 * I && dgu.size(0) == M && dgu.size(1) == 2 * I,
              "gemm_dglu: gu / dgu must be [M, 2I]");
  check(accerl_gemm_dglu_bf16(dy.data_ptr(), ld_of(dy), wd.data_ptr(), ld_of(wd), gu.data_ptr(), ld_of(gu),
                              dgu.data_ptr(), ld_of(dgu), M, I, K, status_ptr(status), static_cast<int>(block_n),
                              static_cast<int>(max_ctas), cur_stream()),
        "gemm_dglu");
}

// Grouped expert GEMM. mode 1: a [M, K] (or [K, M] if a_mn), b stacked [E*Nb, K] K-major / [E*Kb, N]
// MN-major, out [M, N]. mode 2: a [R, M], b [R, N] (MN-major), out stacked [E*c_stride, N] fp32.
void grouped_gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t M,
                  int64_t N, int64_t K, double beta, int64_t mode, const c10::optional<at::Tensor>& tile_expert,
                  const c10::optional<at::Tensor>& row_start, const c10::optional<at::Tensor>& rows,
                  int64_t num_groups, int64_t b_group_stride, int64_t c_group_stride,
                  const c10::optional<at::Tensor>& status, const c10::optional<at::Tensor>& row_dst) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(a));
  CHECK_BF16(a);
  CHECK_BF16(b);
  auto iptr = [](const c10::optional<at::Tensor>& t) -> const int* {
    return t.has_value() ? t->data_ptr<int>() : nullptr;
  };
  check(accerl_grouped_gemm_bf16(a.data_ptr(), ld_of(a), a_mn, b.data_ptr(), ld_of(b), b_mn, out.data_ptr(), ld_of(out),
                                 out.scalar_type() == at::kFloat, M, N, K, b.size(0), static_cast<float>(beta), mode,
                                 iptr(tile_expert), iptr(row_start), iptr(rows), num_groups, b_group_stride,
                                 c_group_stride,
                                 row_dst.has_value() ? reinterpret_cast<const long long*>(row_dst->data_ptr<int64_t>())
                                                     : nullptr,
                                 status_ptr(status), cur_stream()),
        "grouped_gemm");
}

void weight_pull(const at::Tensor& desc, const at::Tensor& unit_start, int64_t n_units, int64_t src_addr,
                 at::Tensor& dst) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(desc));
  CHECK_BF16(dst);
  TORCH_CHECK(desc.scalar_type() == at::kLong && unit_start.scalar_type() == at::kLong, "weight_pull: int64 plans");
  check(accerl_weight_pull(reinterpret_cast<const long long*>(desc.data_ptr<int64_t>()),
                           reinterpret_cast<const long long*>(unit_start.data_ptr<int64_t>()),
                           static_cast<int>(desc.size(0)), n_units, reinterpret_cast<const void*>(src_addr),
                           dst.data_ptr(), cur_stream()),
        "weight_pull");
}

void tp_allreduce(const at::Tensor& peer_data, const at::Tensor& peer_flags, int64_t rank, int64_t slot,
                  int64_t slot_elems, int64_t n, const c10::optional<at::Tensor>& residual, at::Tensor& out,
                  at::Tensor& ctr, at::Tensor& status) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(peer_data));
  CHECK_BF16(out);
  TORCH_CHECK(ctr.scalar_type() == at::kInt && ctr.numel() >= 2, "tp_allreduce: int32 counter pair");
  if (residual.has_value()) CHECK_BF16(*residual);
  check(accerl_tp_allreduce(reinterpret_cast<const long long*>(peer_data.data_ptr<int64_t>()),
                            reinterpret_cast<const long long*>(peer_flags.data_ptr<int64_t>()),
                            static_cast<int>(peer_data.numel()), static_cast<int>(rank), static_cast<int>(slot),
                            slot_elems, n, residual.has_value() ? residual->data_ptr() : nullptr, out.data_ptr(),
                            ctr.data_ptr<int>(), status.data_ptr<int>(), cur_stream()),
        "tp_allreduce");
}

// Router: logits fp32 [T, >=E] -> probs [T, E], topw [T, k], topi int64 [T, k]; counts int32 [E] += rows.
void moe_router(const at::Tensor& logits, int64_t E, int64_t k, bool norm_topk, at::Tensor& probs, at::Tensor& topw,
                at::Tensor& topi, at::Tensor& counts, const c10::optional<at::Tensor>& sg) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(logits));
  CHECK_F32(logits);
  CHECK_F32(probs);
  CHECK_F32(topw);
  TORCH_CHECK(topi.scalar_type() == at::kLong && counts.scalar_type() == at::kInt, "moe_router: topi int64, counts int32");
  float* sgp = nullptr;
  if (sg.has_value()) {
    CHECK_F32(*sg);
    TORCH_CHECK(logits.size(1) > E, "moe_router: the shared-gate logit is column E of the logits");
    sgp = sg->data_ptr<float>();
  }
  check(accerl_moe_router(logits.data_ptr<float>(), ld_of(logits), logits.size(0), E, k, norm_topk,
                          probs.data_ptr<float>(), topw.data_ptr<float>(),
                          reinterpret_cast<long long*>(topi.data_ptr<int64_t>()), counts.data_ptr<int>(), sgp,
                          cur_stream()),
        "moe_router");
}

void moe_combine_fwd(const at::Tensor& ys, const at::Tensor& pos, const at::Tensor& w, int64_t k,
                     const c10::optional<at::Tensor>& residual, const c10::optional<at::Tensor>& shared,
                     const c10::optional<at::Tensor>& sg, at::Tensor& out) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(ys));
  CHECK_BF16(ys);
  CHECK_BF16(out);
  CHECK_F32(w);
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.is_contiguous() && w.is_contiguous(), "moe_combine: pos/w");
  TORCH_CHECK(ys.is_contiguous() && out.is_contiguous(), "moe_combine: contiguous rows");
  if (residual.has_value()) TORCH_CHECK(residual->is_contiguous() && residual->scalar_type() == at::kBFloat16);
  if (shared.has_value()) TORCH_CHECK(shared->is_contiguous() && shared->scalar_type() == at::kBFloat16);
  check(accerl_moe_combine_fwd(ys.data_ptr(), reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()),
                               w.data_ptr<float>(), pos.numel() / k, static_cast<int>(k), static_cast<int>(ys.size(1)),
                               residual.has_value() ? residual->data_ptr() : nullptr,
                               shared.has_value() ? shared->data_ptr() : nullptr,
                               sg.has_value() ? sg->data_ptr<float>() : nullptr, out.data_ptr(), ys.size(0),
                               cur_stream()),
        "moe_combine_fwd");
}

void moe_combine_bwd(const at::Tensor& dout, const at::Tensor& ys, const at::Tensor& pos, const at::Tensor& w,
                     int64_t k, at::Tensor& dys, at::Tensor& dw) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(dout));
  CHECK_BF16(dout);
  CHECK_BF16(ys);
  CHECK_BF16(dys);
  CHECK_F32(w);
  CHECK_F32(dw);
  TORCH_CHECK(pos.scalar_type() == at::kLong && dout.is_contiguous() && ys.is_contiguous() && dys.is_contiguous(),
              "moe_combine_bwd: layouts");
  check(accerl_moe_combine_bwd(dout.data_ptr(), ys.data_ptr(), reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()),
                               w.data_ptr<float>(), pos.numel() / k, static_cast<int>(k), static_cast<int>(ys.size(1)),
                               dys.data_ptr(), dw.data_ptr<float>(), std::min(ys.size(0), dys.size(0)), cur_stream()),
        "moe_combine_bwd");
}

void row_scatter(const at::Tensor& src, const c10::optional<at::Tensor>& src_row, const at::Tensor& dst_addr) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(src));
  CHECK_BF16(src);
  check(accerl_row_scatter(src.data_ptr(), ld_of(src),
                           src_row.has_value() ? reinterpret_cast<const long long*>(src_row->data_ptr<int64_t>())
                                               : nullptr,
                           reinterpret_cast<const long long*>(dst_addr.data_ptr<int64_t>()), dst_addr.numel(),
                           src.size(1), cur_stream()),
        "row_scatter");
}

void splitk_finish(const at::Tensor& acc, const c10::optional<at::Tensor>& bias,
                   const c10::optional<at::Tensor>& residual, at::Tensor& out) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(acc));
  CHECK_F32(acc);
  CHECK_BF16(out);
  check(accerl_splitk_finish(acc.data_ptr<float>(), ld_of(acc), opt_ptr(bias), opt_ptr(residual),
                             residual.has_value() ? ld_of(*residual) : 0, out.data_ptr(), ld_of(out), out.size(0),
                             out.size(1), cur_stream()),
        "splitk_finish");
}

at::Tensor rmsnorm_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, const c10::optional<at::Tensor>& rstd,
                       double eps) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(x));
  CHECK_CUDA(x);
  CHECK_BF16(x);
  CHECK_BF16(w);
  CHECK_BF16(y);
  const int rows = x.size(0), H = x.size(1);
  float* r = rstd.has_value() ? rstd->data_ptr<float>() : nullptr;
  check(accerl_rmsnorm_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), r, rows, H, ld_of(x), ld_of(y),
                           static_cast<float>(eps), cur_stream()),
        "rmsnorm_fwd");
  return y;
}

void rmsnorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                 const c10::optional<at::Tensor>& dx_accum, at::Tensor& dx, const c10::optional<at::Tensor>& dw,
                 const c10::optional<at::Tensor>& workspace, bool dw_accumulate) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(dy));
  CHECK_BF16(dy);
  CHECK_BF16(x);
  CHECK_F32(rstd);
  const int rows = x.size(0), H = x.size(1);
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dx.is_contiguous(), "rmsnorm_bwd: contiguous inputs");
  float* dwp = nullptr;
  float* ws = nullptr;
  if (dw.has_value()) {
    CHECK_F32(*dw);
    const long long fused_warps = 8LL * ((std::min((rows + 3) / 4, 148 * 16) + 7) / 8);
    TORCH_CHECK(workspace.has_value() &&
                    workspace->numel() >= std::max<long long>((rows + 63) / 64, fused_warps) * (long long)H,
                "rmsnorm_bwd: workspace too small");
    dwp = dw->data_ptr<float>();
    ws = workspace->data_ptr<float>();
  }
  check(accerl_rmsnorm_bwd(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr<float>(), opt_ptr(dx_accum),
                           dx.data_ptr(), dwp, ws, rows, H, H, dw_accumulate, cur_stream()),
        "rmsnorm_bwd");
}

void bias_grad(const at::Tensor& dy, at::Tensor& db, at::Tensor& workspace, bool accumulate) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(dy));
  CHECK_BF16(dy);
  CHECK_F32(db);
  const int rows = dy.size(0), N = dy.size(1);
  TORCH_CHECK(workspace.numel() >= ((rows + 63) / 64) * (long long)N, "bias_grad: workspace too small");
  check(accerl_bias_grad(dy.data_ptr(), db.data_ptr<float>(), workspace.data_ptr<float>(), rows, N, ld_of(dy),
                         accumulate, cur_stream()),
        "bias_grad");
}

void rope(at::Tensor& qkv, const at::Tensor& pos, int64_t n_rot_heads, int64_t head_dim, double theta, bool inverse) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(qkv));
  CHECK_BF16(qkv);
  CHECK_I64(pos);
  TORCH_CHECK(pos.is_contiguous() && pos.numel() == qkv.size(0), "rope: positions must be [T]");
  check(accerl_rope(qkv.data_ptr(), reinterpret_cast<long long*>(pos.data_ptr<int64_t>()), qkv.size(0), n_rot_heads, head_dim, ld_of(qkv),
                    static_cast<float>(theta), inverse, cur_stream()),
        "rope");
}

void swiglu_fwd(const at::Tensor& gu, at::Tensor& h) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(gu));
  CHECK_BF16(gu);
  TORCH_CHECK(gu.is_contiguous() && h.is_contiguous(), "swiglu: contiguous");
  check(accerl_swiglu_fwd(gu.data_ptr(), h.data_ptr(), gu.size(0), h.size(1), cur_stream()), "swiglu_fwd");
}

void swiglu_bwd(const at::Tensor& dh, const at::Tensor& gu, at::Tensor& dgu) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(dh));
  TORCH_CHECK(dh.is_contiguous() && gu.is_contiguous() && dgu.is_contiguous(), "swiglu_bwd: contiguous");
  check(accerl_swiglu_bwd(dh.data_ptr(), gu.data_ptr(), dgu.data_ptr(), gu.size(0), dh.size(1), cur_stream()),
        "swiglu_bwd");
}

void embedding_fwd(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(ids));
  CHECK_I64(ids);
  CHECK_BF16(table);
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && ids.is_contiguous(), "embedding: contiguous");
  check(accerl_embedding_fwd(reinterpret_cast<long long*>(ids.data_ptr<int64_t>()), table.data_ptr(), out.data_ptr(), ids.numel(), table.size(1),
                             table.size(0), cur_stream()),
        "embedding_fwd");
}

void embedding_bwd(const at::Tensor& ids, const at::Tensor& dout, at::Tensor& grad) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(ids));
  CHECK_I64(ids);
  CHECK_F32(grad);
  check(accerl_embedding_bwd(reinterpret_cast<long long*>(ids.data_ptr<int64_t>()), dout.data_ptr(), grad.data_ptr<float>(), ids.numel(),
                             grad.size(1), grad.size(0), cur_stream()),
        "embedding_bwd");
}

void logsoftmax_label_fwd(const at::Tensor& logits, const at::Tensor& labels, at::Tensor& logprob, at::Tensor& lse,
                          const c10::optional<at::Tensor>& entropy) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(logits));
  CHECK_BF16(logits);
  CHECK_I64(labels);
  float* ent = entropy.has_value() ? entropy->data_ptr<float>() : nullptr;
  check(accerl_logsoftmax_label_fwd(logits.data_ptr(), ld_of(logits), reinterpret_cast<long long*>(labels.data_ptr<int64_t>()),
                                    logprob.data_ptr<float>(), lse.data_ptr<float>(), ent, logits.size(0),
                                    logits.size(1), cur_stream()),
        "logsoftmax_label_fwd");
}

void logsoftmax_label_bwd(at::Tensor& logits, const at::Tensor& labels, const at::Tensor& lse, const at::Tensor& grad,
                          int64_t label_offset) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(logits));
  CHECK_BF16(logits);
  check(accerl_logsoftmax_label_bwd(logits.data_ptr(), ld_of(logits), reinterpret_cast<long long*>(labels.data_ptr<int64_t>()),
                                    lse.data_ptr<float>(), grad.data_ptr<float>(), logits.size(0), logits.size(1),
                                    label_offset, cur_stream()),
        "logsoftmax_label_bwd");
}

void lse_chunk(const at::Tensor& logits, const at::Tensor& labels, int64_t c0, bool first, at::Tensor& state) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(logits));
  CHECK_BF16(logits);
  CHECK_F32(state);
  check(accerl_lse_chunk(logits.data_ptr(), ld_of(logits), reinterpret_cast<const long long*>(labels.data_ptr<int64_t>()),
                         c0, logits.size(0), logits.size(1), first ? 1 : 0, state.data_ptr<float>(), cur_stream()),
        "lse_chunk");
}

void lse_finish(const at::Tensor& state, at::Tensor& logprob, at::Tensor& lse, const c10::optional<at::Tensor>& entropy) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(state));
  CHECK_F32(state);
  check(accerl_lse_finish(state.data_ptr<float>(), logprob.size(0), logprob.data_ptr<float>(), lse.data_ptr<float>(),
                          entropy.has_value() ? entropy->data_ptr<float>() : nullptr, cur_stream()),
        "lse_finish");
}

void policy_loss(const at::Tensor& lp, const at::Tensor& old_lp, const at::Tensor& adv, at::Tensor& dlp,
                 at::Tensor& stats, int64_t mode, double clip_eps, double gipo_sigma, double tau_pos, double tau_neg,
                 double kl_coef, double loss_scale) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(lp));
  CHECK_F32(lp);
  CHECK_F32(old_lp);
  CHECK_F32(adv);
  TORCH_CHECK(stats.scalar_type() == at::kDouble && stats.numel() >= 3, "stats must be float64[3]");
  check(accerl_policy_loss(lp.data_ptr<float>(), old_lp.data_ptr<float>(), adv.data_ptr<float>(),
                           dlp.data_ptr<float>(), stats.data_ptr<double>(), lp.numel(), mode, clip_eps, gipo_sigma,
                           tau_pos, tau_neg, kl_coef, loss_scale, cur_stream()),
        "policy_loss");
}

void sumsq(const at::Tensor& g, at::Tensor& out) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(g));
  CHECK_F32(g);
  TORCH_CHECK(out.scalar_type() == at::kDouble, "sumsq: out must be float64");
  check(accerl_sumsq(g.data_ptr<float>(), g.numel(), out.data_ptr<double>(), cur_stream()), "sumsq");
}

void adamw(at::Tensor& master, at::Tensor& m, at::Tensor& v, at::Tensor& grad, at::Tensor& param,
           const at::Tensor& sumsq_t, double lr, double beta1, double beta2, double eps, double weight_decay,
           double max_norm, double bc1, double bc2_sqrt) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(master));
  CHECK_F32(master);
  CHECK_BF16(param);
  TORCH_CHECK(master.numel() == param.numel() && grad.numel() == param.numel(), "adamw: size mismatch");
  check(accerl_adamw(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr<float>(),
                     param.data_ptr(), master.numel(), sumsq_t.data_ptr<double>(), lr, beta1, beta2, eps, weight_decay,
                     max_norm, bc1, bc2_sqrt, cur_stream()),
        "adamw");
}

// q: [T, Hq*D] view (row stride ldq), k/v: [T, Hkv*D], o: [T, Hq*D]; lse: [Hq, T] fp32
void attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
              const at::Tensor& cu_seqlens, const c10::optional<at::Tensor>& cu_seqlens_k, int64_t max_seqlen,
              int64_t Hq, int64_t Hkv, double scale, bool causal, const c10::optional<at::Tensor>& status,
              const c10::optional<at::Tensor>& block_table) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(q));
  CHECK_BF16(q);
  CHECK_BF16(k);
  CHECK_BF16(v);
  CHECK_BF16(o);
  CHECK_F32(lse);
  CHECK_I32(cu_seqlens);
  const int* cuk = cu_seqlens_k.has_value() ? cu_seqlens_k->data_ptr<int>() : nullptr;
  if (block_table.has_value()) {
    // k / v: the layer's paged caches [num_blocks, block_size, Hkv, 128]
    CHECK_I32(*block_table);
    TORCH_CHECK(k.dim() == 4 && k.is_contiguous() && v.is_contiguous(), "attn_fwd: paged caches must be contiguous");
    check(accerl_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(),
                          cu_seqlens.data_ptr<int>(), cuk, cu_seqlens.numel() - 1, max_seqlen, q.size(0),
                          k.size(0) * k.size(1), Hq, Hkv, ld_of(q), Hkv * 128, Hkv * 128, ld_of(o),
                          static_cast<float>(scale), causal, status_ptr(status), block_table->data_ptr<int>(),
                          block_table->size(1), k.size(1), cur_stream()),
          "attn_fwd");
    return;
  }
  check(accerl_attn_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(),
                        cu_seqlens.data_ptr<int>(), cuk, cu_seqlens.numel() - 1, max_seqlen, q.size(0), k.size(0), Hq,
                        Hkv, ld_of(q), ld_of(k), ld_of(v), ld_of(o), static_cast<float>(scale), causal,
                        status_ptr(status), nullptr, 0, 0, cur_stream()),
        "attn_fwd");
}

void attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& o,
              const at::Tensor& dout, const at::Tensor& lse, at::Tensor& delta, at::Tensor& dq_acc, at::Tensor& dq,
              at::Tensor& dk, at::Tensor& dv, const at::Tensor& cu_seqlens, int64_t max_seqlen, int64_t Hq, int64_t Hkv,
              double scale, bool causal, const c10::optional<at::Tensor>& status,
              const c10::optional<at::Tensor>& rope_pos, double rope_theta) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(q));
  CHECK_F32(delta);
  if (rope_pos.has_value())
    TORCH_CHECK(rope_pos->scalar_type() == at::kLong && rope_pos->numel() == q.size(0), "attn_bwd: rope_pos int64 [T]");
  CHECK_F32(dq_acc);
  check(accerl_attn_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(), lse.data_ptr<float>(),
                        delta.data_ptr<float>(), dq_acc.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                        cu_seqlens.data_ptr<int>(), cu_seqlens.numel() - 1, max_seqlen, q.size(0), Hq, Hkv, ld_of(q),
                        ld_of(k), ld_of(v), ld_of(o), ld_of(dout), ld_of(dq), ld_of(dk), ld_of(dv),
                        static_cast<float>(scale), causal, status_ptr(status),
                        rope_pos.has_value() ? reinterpret_cast<const long long*>(rope_pos->data_ptr<int64_t>()) : nullptr,
                        static_cast<float>(rope_theta), cur_stream()),
        "attn_bwd");
}

// impl: 0 = the keys-on-lanes tensor-core kernel when the shape allows it, else the CUDA-core kernel;
// 1 = CUDA-core; 2 = tensor-core with the query heads as MMA rows; 3 = tensor-core with the keys as
// MMA rows (2 and 3: error if unsupported).
void paged_decode(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                  const at::Tensor& block_table, const at::Tensor& seq_lens, at::Tensor& out, at::Tensor& part_o,
                  at::Tensor& part_ml, int64_t Hq, int64_t Hkv, int64_t num_splits, double scale, int64_t impl,
                  const c10::optional<at::Tensor>& status) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(q));
  CHECK_BF16(q);
  CHECK_I32(block_table);
  CHECK_I32(seq_lens);
  if (impl != 1 && k_cache.size(-1) == 128) {
    auto* launch = impl == 2 ? accerl_paged_decode_tc : accerl_paged_decode_tq;
    const int rc = launch(q.data_ptr(), ld_of(q), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.size(0),
                          block_table.data_ptr<int>(), block_table.size(1), seq_lens.data_ptr<int>(),
                          part_o.data_ptr<float>(), part_ml.data_ptr<float>(), q.size(0), Hq, Hkv, k_cache.size(1),
                          num_splits, static_cast<float>(scale), status_ptr(status), cur_stream());
    if (rc != -2 || impl >= 2) {
      check(rc, "paged_decode_tc");
      check(accerl_paged_decode_merge(part_o.data_ptr<float>(), part_ml.data_ptr<float>(), out.data_ptr(), ld_of(out),
                                      q.size(0), Hq, num_splits, cur_stream()),
            "paged_decode_merge");
      return;
    }
  }
  check(accerl_paged_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), block_table.data_ptr<int>(),
                            seq_lens.data_ptr<int>(), out.data_ptr(), part_o.data_ptr<float>(),
                            part_ml.data_ptr<float>(), q.size(0), Hq, Hkv, block_table.size(1), k_cache.size(1),
                            num_splits, static_cast<float>(scale), ld_of(q), ld_of(out), cur_stream()),
        "paged_decode");
}

void kv_cache_write(const at::Tensor& k, const at::Tensor& v, at::Tensor& k_cache, at::Tensor& v_cache,
                    const at::Tensor& slot_mapping, int64_t Hkv) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(k));
  CHECK_I32(slot_mapping);
  check(accerl_kv_cache_write(k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                              slot_mapping.data_ptr<int>(), k.size(0), Hkv, ld_of(k), ld_of(v),
                              k_cache.size(0) * k_cache.size(1), cur_stream()),
        "kv_cache_write");
}

void qkv_rope_cache(at::Tensor& qkv, const at::Tensor& pos, const at::Tensor& slot_mapping, at::Tensor& k_cache,
                    at::Tensor& v_cache, int64_t Hq, int64_t Hkv, double theta, const c10::optional<at::Tensor>& q_norm,
                    const c10::optional<at::Tensor>& k_norm, double eps) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(qkv));
  CHECK_BF16(qkv);
  CHECK_BF16(k_cache);
  CHECK_BF16(v_cache);
  CHECK_I64(pos);
  CHECK_I32(slot_mapping);
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) == (Hq + 2 * Hkv) * 128,
              "qkv_rope_cache: qkv rows [Hq | Hkv | Hkv] heads of 128");
  TORCH_CHECK(pos.numel() == qkv.size(0) && slot_mapping.numel() == qkv.size(0) && pos.is_contiguous() &&
                  slot_mapping.is_contiguous(), "qkv_rope_cache: one position and slot per row");
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous() && k_cache.size(-1) == 128 &&
                  k_cache.size(-2) == Hkv && k_cache.sizes() == v_cache.sizes(),
              "qkv_rope_cache: caches [blocks, block_size, Hkv, 128]");
  TORCH_CHECK(q_norm.has_value() == k_norm.has_value(), "qkv_rope_cache: both or neither qk-norm weights");
  if (q_norm.has_value()) {
    CHECK_BF16(*q_norm);
    CHECK_BF16(*k_norm);
    TORCH_CHECK(q_norm->numel() == 128 && k_norm->numel() == 128 && q_norm->is_contiguous() && k_norm->is_contiguous(),
                "qkv_rope_cache: qk-norm weights of 128");
  }
  check(accerl_qkv_rope_cache(qkv.data_ptr(), ld_of(qkv), reinterpret_cast<const long long*>(pos.data_ptr<int64_t>()),
                              slot_mapping.data_ptr<int>(), qkv.size(0), Hq, Hkv, static_cast<float>(theta),
                              q_norm.has_value() ? q_norm->data_ptr() : nullptr,
                              k_norm.has_value() ? k_norm->data_ptr() : nullptr, static_cast<float>(eps),
                              k_cache.data_ptr(), v_cache.data_ptr(), k_cache.numel() / (Hkv * 128), cur_stream()),
        "qkv_rope_cache");
}

// CUDA IPC of a tensor's allocation. The handle covers the caching-allocator segment that holds the
// tensor; the tensor's byte offset inside it travels with the handle. Peers open it on THEIR current
// device with lazy peer access, so the mapping lives in the context their kernels run in. Errors are
// returned as codes (no exceptions across the binding).
std::tuple<int64_t, py::bytes, int64_t> ipc_export(const at::Tensor& t) {
  TORCH_CHECK(t.is_cuda(), "ipc_export: cuda tensor");
  size_t seg = 0;
  void* base = c10::cuda::CUDACachingAllocator::getBaseAllocation(t.data_ptr(), &seg);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, base);
  const int64_t off = static_cast<const char*>(t.data_ptr()) - static_cast<const char*>(base);
  return {static_cast<int64_t>(e), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)), off};
}

std::tuple<int64_t, int64_t> ipc_open(const py::bytes& handle) {
  const std::string raw = handle;
  if (raw.size() != sizeof(cudaIpcMemHandle_t)) return {-1, 0};
  cudaIpcMemHandle_t h;
  std::memcpy(&h, raw.data(), sizeof(h));
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) cudaGetLastError();
  return {static_cast<int64_t>(e), reinterpret_cast<int64_t>(base)};
}

int64_t ipc_close(int64_t base) {
  const cudaError_t e = cudaIpcCloseMemHandle(reinterpret_cast<void*>(base));
  if (e != cudaSuccess) cudaGetLastError();
  return static_cast<int64_t>(e);
}

// Synchronous copy of n bytes from a (peer) device address into host memory: a host-side check that
// a mapping is readable and holds what its owner reports, before any kernel dereferences it.
std::tuple<int64_t, py::bytes> peer_read(int64_t addr, int64_t n) {
  std::string out(static_cast<size_t>(n), '\0');
  const cudaError_t e = cudaMemcpy(out.data(), reinterpret_cast<const void*>(addr), n, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) cudaGetLastError();
  return {static_cast<int64_t>(e), py::bytes(out)};
}

void enable_peer_access(int64_t peer) { check(accerl_enable_peer_access(static_cast<int>(peer)), "enable_peer_access"); }

// peer_ptrs: int64 device tensor [world] of base addresses (fp32 full gradient buffers)
void rs_sumsq(const at::Tensor& peer_ptrs, int64_t rank, int64_t shard, at::Tensor& out, at::Tensor& sumsq) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(peer_ptrs));
  CHECK_F32(out);
  TORCH_CHECK(peer_ptrs.scalar_type() == at::kLong && peer_ptrs.is_cuda(), "peer_ptrs: int64 cuda tensor");
  check(accerl_rs_sumsq(reinterpret_cast<const float* const*>(peer_ptrs.data_ptr<int64_t>()), peer_ptrs.numel(),
                        rank, shard, out.data_ptr<float>(), sumsq.data_ptr<double>(), cur_stream()),
        "rs_sumsq");
}

void adamw_push(at::Tensor& master, at::Tensor& m, at::Tensor& v, const at::Tensor& grad, const at::Tensor& peer_ptrs,
                int64_t rank, const at::Tensor& sumsq_t, double lr, double beta1, double beta2, double eps,
                double weight_decay, double max_norm, double bc1, double bc2_sqrt) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(master));
  CHECK_F32(master);
  check(accerl_adamw_push(master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr<float>(),
                          reinterpret_cast<void* const*>(peer_ptrs.data_ptr<int64_t>()), peer_ptrs.numel(), rank,
                          master.numel(), sumsq_t.data_ptr<double>(), lr, beta1, beta2, eps, weight_decay, max_norm,
                          bc1, bc2_sqrt, cur_stream()),
        "adamw_push");
}

void sample_logits(const at::Tensor& logits, const at::Tensor& temperature, const at::Tensor& seeds,
                   const at::Tensor& offsets, at::Tensor& out_tokens, at::Tensor& out_logprobs, at::Tensor& part,
                   int64_t num_chunks, const c10::optional<at::Tensor>& top_k,
                   const c10::optional<at::Tensor>& top_p) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(logits));
  CHECK_BF16(logits);
  CHECK_F32(temperature);
  const int* tk = nullptr;
  const float* tp = nullptr;
  if (top_k.has_value()) {
    TORCH_CHECK(top_k->scalar_type() == at::kInt && top_k->is_contiguous(), "top_k must be contiguous int32");
    tk = top_k->data_ptr<int>();
  }
  if (top_p.has_value()) {
    CHECK_F32(*top_p);
    tp = top_p->data_ptr<float>();
  }
  check(accerl_sample_logits(logits.data_ptr(), ld_of(logits), logits.size(0), logits.size(1),
                             temperature.data_ptr<float>(), tk, tp,
                             reinterpret_cast<const unsigned long long*>(seeds.data_ptr<int64_t>()),
                             reinterpret_cast<long long*>(offsets.data_ptr<int64_t>()),
                             reinterpret_cast<long long*>(out_tokens.data_ptr<int64_t>()),
                             out_logprobs.data_ptr<float>(), part.data_ptr<float>(), num_chunks, cur_stream()),
        "sample_logits");
}

}  // namespace

// Debug-checks build records, one (code, index) pair per kernel source file (code 0: no failed check).
// Returns an empty list in a release build.
std::vector<std::tuple<std::string, int64_t, int64_t>> debug_status(bool reset) {
  using Reader = int (*)(long long*, int);
  const std::pair<const char*, Reader> units[] = {{"attention", accerl_debug_status_attention},
                                                  {"elementwise", accerl_debug_status_elementwise},
                                                  {"moe", accerl_debug_status_moe},
                                                  {"rollout", accerl_debug_status_rollout}};
  std::vector<std::tuple<std::string, int64_t, int64_t>> out;
  for (const auto& u : units) {
    long long rec[2] = {0, 0};
    const int rc = u.second(rec, reset ? 1 : 0);
    TORCH_CHECK(rc >= 0, "debug_status: reading the record of ", u.first, " failed");
    if (rc == 1) out.emplace_back(u.first, rec[0], rec[1]);
  }
  return out;
}

void moe_router_bwd(const at::Tensor& probs, const at::Tensor& topi, const at::Tensor& topw, const at::Tensor& dw,
                    bool norm_topk, const c10::optional<at::Tensor>& dout, const c10::optional<at::Tensor>& sy,
                    const c10::optional<at::Tensor>& sg, at::Tensor& dgrad, const c10::optional<at::Tensor>& dsy) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(probs));
  CHECK_F32(probs);
  CHECK_F32(topw);
  CHECK_F32(dw);
  CHECK_BF16(dgrad);
  const int T = probs.size(0), E = probs.size(1), k = topi.size(1);
  const bool shared = sy.has_value();
  check(accerl_moe_router_bwd(probs.data_ptr<float>(), reinterpret_cast<const long long*>(topi.data_ptr<int64_t>()),
                              topw.data_ptr<float>(), dw.data_ptr<float>(), T, E, k, norm_topk ? 1 : 0,
                              shared ? dout->data_ptr() : nullptr, shared ? sy->data_ptr() : nullptr,
                              shared ? sg->data_ptr<float>() : nullptr, shared ? sy->size(1) : 0, dgrad.data_ptr(),
                              dgrad.size(1), shared ? dsy->data_ptr() : nullptr, cur_stream()),
        "moe_router_bwd");
}

void moe_layout(const at::Tensor& topi, const at::Tensor& topw, const at::Tensor& h, int64_t E, int64_t lo, int64_t El,
                int64_t total, at::Tensor& xs, bool zero_pad, at::Tensor& hist, at::Tensor& pos, at::Tensor& w,
                at::Tensor& tile_expert, at::Tensor& row_start, at::Tensor& seg_rows,
                const c10::optional<at::Tensor>& counts) {
  const c10::cuda::OptionalCUDAGuard device_guard(at::device_of(topi));
  CHECK_F32(topw);
  CHECK_BF16(h);
  CHECK_BF16(xs);
  TORCH_CHECK(topi.scalar_type() == at::kLong && topi.is_contiguous() && topw.is_contiguous() &&
                  topi.numel() == topw.numel() && topi.dim() == 2,
              "moe_layout: topi [T, k] int64 and topw [T, k] fp32, contiguous");
  const int64_t n = topi.numel(), k = topi.size(1), H = h.size(1);
  TORCH_CHECK(h.is_contiguous() && h.size(0) * k == n && xs.is_contiguous() && xs.size(1) == H && xs.size(0) >= total,
              "moe_layout: h [T, H] and xs [>= total, H] contiguous");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(h.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(xs.data_ptr()) % 16 == 0,
              "moe_layout: 16-byte aligned rows");
  TORCH_CHECK(hist.scalar_type() == at::kInt && hist.numel() >= ((n + 1023) / 1024) * E, "moe_layout: hist scratch");
  TORCH_CHECK(pos.scalar_type() == at::kLong && pos.numel() == n && w.scalar_type() == at::kFloat && w.numel() == n,
              "moe_layout: pos int64 / w fp32 per pair");
  TORCH_CHECK(tile_expert.scalar_type() == at::kInt && tile_expert.numel() >= total / 128 &&
                  row_start.scalar_type() == at::kInt && row_start.numel() >= El &&
                  seg_rows.scalar_type() == at::kInt && seg_rows.numel() >= El,
              "moe_layout: int32 layout outputs");
  int* cp = nullptr;
  if (counts.has_value()) {
    TORCH_CHECK(counts->scalar_type() == at::kInt && counts->numel() >= E, "moe_layout: counts int32 [E]");
    cp = counts->data_ptr<int>();
  }
  check(accerl_moe_layout(reinterpret_cast<const long long*>(topi.data_ptr<int64_t>()), topw.data_ptr<float>(), n,
                          static_cast<int>(k), static_cast<int>(E), static_cast<int>(lo), static_cast<int>(El), total,
                          h.data_ptr(), static_cast<int>(H), xs.data_ptr(), zero_pad ? 1 : 0, hist.data_ptr<int>(),
                          reinterpret_cast<long long*>(pos.data_ptr<int64_t>()), w.data_ptr<float>(),
                          tile_expert.data_ptr<int>(), row_start.data_ptr<int>(), seg_rows.data_ptr<int>(), cp,
                          cur_stream()),
        "moe_layout");
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("debug_status", &debug_status, "debug-checks build: (unit, code, index) per kernel file");
  m.doc() = "accerl_agent_b200 sm_100a kernels";
  m.def("last_error", &last_error, "(code, message) of the most recent launch; resets it");
  m.def("gemm", &gemm, "tcgen05 bf16 GEMM");
  m.def("gemm_glu", &gemm_glu, "gate/up GEMM with the SwiGLU epilogue");
  m.def("gemm_rope", &gemm_rope, "projection GEMM with the rotary-embedding epilogue");
  m.def("gemm_dglu", &gemm_dglu, "down-projection dgrad GEMM with the SwiGLU backward epilogue");
  m.def("splitk_finish", &splitk_finish);
  m.def("grouped_gemm", &grouped_gemm);
  m.def("row_scatter", &row_scatter);
  m.def("weight_pull", &weight_pull);
  m.def("moe_router_bwd", &moe_router_bwd);
  m.def("moe_layout", &moe_layout);
  m.def("qkv_rope_cache", &qkv_rope_cache);
  m.def("moe_router", &moe_router);
  m.def("moe_combine_fwd", &moe_combine_fwd);
  m.def("moe_combine_bwd", &moe_combine_bwd);
  m.def("tp_allreduce", &tp_allreduce);
  m.def("ipc_export", &ipc_export);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("peer_read", &peer_read);
  m.def("rmsnorm_fwd", &rmsnorm_fwd);
  m.def("rmsnorm_bwd", &rmsnorm_bwd);
  m.def("bias_grad", &bias_grad);
  m.def("rope", &rope);
  m.def("swiglu_fwd", &swiglu_fwd);
  m.def("swiglu_bwd", &swiglu_bwd);
  m.def("embedding_fwd", &embedding_fwd);
  m.def("embedding_bwd", &embedding_bwd);
  m.def("logsoftmax_label_fwd", &logsoftmax_label_fwd);
  m.def("logsoftmax_label_bwd", &logsoftmax_label_bwd);
  m.def("lse_chunk", &lse_chunk);
  m.def("lse_finish", &lse_finish);
  m.def("policy_loss", &policy_loss);
  m.def("sumsq", &sumsq);
  m.def("adamw", &adamw);
  m.def("attn_fwd", &attn_fwd);
  m.def("attn_bwd", &attn_bwd);
  m.def("paged_decode", &paged_decode);
  m.def("kv_cache_write", &kv_cache_write);
  m.def("sample_logits", &sample_logits);
  m.def("enable_peer_access", &enable_peer_access);
  m.def("rs_sumsq", &rs_sumsq);
  m.def("adamw_push", &adamw_push);
}
