"""Public op surface. CUDA tensors run the sm_100a kernels of ``csrc/``; CPU tensors run the fp32
PyTorch implementations in ``reference.py``.

Shapes follow the packed-varlen convention: activations are ``[T, features]`` row-major matrices,
weights keep the HF ``[out_features, in_features]`` layout.
"""

from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from . import reference
from ._ext import available, check_status, debug_checks_enabled, debug_status, native as _native_module, status_tensor


# Kernels launched by one call of each binding (the benchmark reports launches per timed step).
KERNELS_PER_CALL = {
    "rmsnorm_bwd": 3, "bias_grad": 2, "attn_bwd": 4, "paged_decode": 2, "sample_logits": 2,
}
LAUNCHES = [0]


class _Checked:
    """Proxy over the extension: every kernel launch is followed by a check of its launch code
    (argument validation or cudaError) so failures raise here with the op name."""

    def __init__(self, ext):
        self._ext = ext

    def __getattr__(self, name):
        fn = getattr(self._ext, name)
        per_call = KERNELS_PER_CALL.get(name, 1)
        last_error = self._ext.last_error

        def call(*args):
            fn(*args)
            LAUNCHES[0] += per_call
            rc, msg = last_error()
            if rc != 0:
                raise RuntimeError(f"native op {name} failed (code {rc}): {msg}")

        self.__dict__[name] = call  # later lookups find the wrapper without __getattr__
        return call


_CHECKED = None


def native():
    global _CHECKED
    if _CHECKED is None:
        _CHECKED = _Checked(_native_module())
    return _CHECKED

__all__ = [
    "available",
    "check_status",
    "gemm",
    "linear",
    "linear_dgrad",
    "linear_wgrad",
    "bias_grad",
    "rmsnorm",
    "rmsnorm_backward",
    "rope_",
    "swiglu",
    "swiglu_backward",
    "linear_swiglu",
    "linear_rope",
    "linear_dgrad_swiglu",
    "embedding",
    "embedding_backward",
    "attention_varlen",
    "attention_varlen_backward",
    "logsoftmax_label",
    "logsoftmax_label_backward",
    "lm_head_logprobs",
    "lm_head_backward",
    "policy_loss",
    "grad_sumsq",
    "adamw_step",
    "paged_decode",
    "kv_cache_write",
    "qkv_rope_cache",
    "sample",
    "workspace",
]

_WORKSPACE: Dict[Tuple[int, str], torch.Tensor] = {}
_RETIRED: list = []  # outgrown workspaces stay alive: captured CUDA graphs may still point at them


def workspace(device: torch.device, name: str, numel: int, dtype=torch.float32) -> torch.Tensor:
    """Grow-only scratch buffers, one per (device, name). Callers use them within one stream."""
    key = (device.index if device.index is not None else -1, name)
    buf = _WORKSPACE.get(key)
    if buf is None or buf.numel() < numel or buf.dtype != dtype:
        size = numel
        if buf is not None:
            _RETIRED.append(buf)
            if buf.dtype == dtype:
                size = max(numel, int(buf.numel() * 1.5))  # grow geometrically: few reallocations
        buf = torch.empty(max(size, 1), dtype=dtype, device=device)
        _WORKSPACE[key] = buf
    return buf[:numel]


# ------------------------------------------------------------------------------------------------
# GEMM / linear
# ------------------------------------------------------------------------------------------------
def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: Optional[torch.Tensor] = None,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    alpha: float = 1.0,
    beta: float = 0.0,
    bias: Optional[torch.Tensor] = None,
    residual: Optional[torch.Tensor] = None,
    out_dtype: torch.dtype = torch.bfloat16,
    block_n: int = 0,
    max_ctas: int = 0,
    splits: int = 0,
) -> torch.Tensor:
    """``out = alpha * A @ B^T + beta*out (+bias) (+residual)`` with A given as [M,K] (or [K,M] if
    ``a_mn``) and B as [N,K] (or [K,N] if ``b_mn``).

    ``splits`` > 1 splits K across CTAs (fp32 output accumulated with ``beta=1`` only); 0 lets the
    launcher choose for fp32 accumulation, 1 disables it."""
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    if a.is_cuda:
        native().gemm(a, a_mn, b, b_mn, out, alpha, beta, bias, residual, status_tensor(a.device), block_n, max_ctas,
                      splits)
        return out
    af = a.float().t() if a_mn else a.float()
    bf = b.float() if b_mn else b.float().t()
    acc = alpha * (af @ bf)
    if beta != 0.0:
        acc = acc + beta * out.float()
    if bias is not None:
        acc = acc + bias.float()
    if residual is not None:
        acc = acc + residual.float()
    out.copy_(acc.to(out.dtype))
    return out


def linear(x: torch.Tensor, w: torch.Tensor, bias=None, residual=None, out=None) -> torch.Tensor:
    """``y = x w^T (+b) (+residual)``; x [T, in], w [out, in]. Skinny products (few rows, e.g. decode
    steps) run split-K into an fp32 scratch and a finishing pass, so the whole GPU streams weights."""
    if x.is_cuda and x.shape[0] <= 256 and x.dtype == torch.bfloat16:
        M, N, K = x.shape[0], w.shape[0], w.shape[1]
        tiles = (N + 127) // 128
        splits = 1
        while tiles * splits * 2 <= 148 and (K // 64) // (splits * 2) >= 2:
            splits *= 2
        if splits > 1:
            acc = workspace(x.device, "splitk_acc", M * N).view(M, N)
            acc.zero_()
            gemm(x, w, acc, beta=1.0, out_dtype=torch.float32, block_n=128, splits=splits)
            out = out if out is not None else torch.empty(M, N, dtype=x.dtype, device=x.device)
            native().splitk_finish(acc, bias, residual, out)
            return out
    return gemm(x, w, out, bias=bias, residual=residual, out_dtype=x.dtype)


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out=None, accumulate: bool = False) -> torch.Tensor:
    """``dx = dy w`` (``+= `` into ``out`` when ``accumulate``); dy [T, out], w [out, in]."""
    return gemm(dy, w, out, b_mn=True, beta=1.0 if accumulate else 0.0, out_dtype=dy.dtype)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, grad: torch.Tensor, accumulate: bool = True) -> torch.Tensor:
    """``grad (+)= dy^T x`` in fp32; dy [T, out], x [T, in], grad [out, in] fp32. Accumulating calls
    split the token dimension across CTAs when the weight alone would not fill the GPU."""
    return gemm(dy, x, grad, a_mn=True, b_mn=True, beta=1.0 if accumulate else 0.0, out_dtype=torch.float32,
                splits=0 if accumulate else 1)


def bias_grad(dy: torch.Tensor, grad: torch.Tensor, accumulate: bool = True) -> torch.Tensor:
    if dy.is_cuda:
        ws = workspace(dy.device, "colsum", ((dy.shape[0] + 63) // 64) * dy.shape[1])
        native().bias_grad(dy, grad, ws, accumulate)
        return grad
    s = dy.float().sum(0)
    if accumulate:
        grad.add_(s)
    else:
        grad.copy_(s)
    return grad


# ------------------------------------------------------------------------------------------------
# normalisation / positional / activation / embedding
# ------------------------------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out=None) -> Tuple[torch.Tensor, torch.Tensor]:
    if x.is_cuda:
        y = out if out is not None else torch.empty_like(x)
        rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
        native().rmsnorm_fwd(x, w, y, rstd, eps)
        return y, rstd
    return reference.rmsnorm(x, w, eps)


def rmsnorm_backward(dy, x, w, rstd, dx_accum=None, dw_grad=None, dw_accumulate: bool = True) -> torch.Tensor:
    """Returns ``dx (+ dx_accum)``; adds the weight gradient into ``dw_grad`` (fp32) when given."""
    if x.is_cuda:
        dx = torch.empty_like(x)
        ws = None
        if dw_grad is not None:
            rows, H = x.shape
            ws = workspace(x.device, "rmsnorm_dw", max((rows + 63) // 64, 8 * ((min((rows + 3) // 4, 148 * 16) + 7) // 8)) * H)
        native().rmsnorm_bwd(dy, x, w, rstd, dx_accum, dx, dw_grad, ws, dw_accumulate)
        return dx
    dx, dw = reference.rmsnorm_backward(dy, x, w, rstd)
    if dw_grad is not None:
        if dw_accumulate:
            dw_grad.add_(dw)
        else:
            dw_grad.copy_(dw)
    if dx_accum is not None:
        dx = dx + dx_accum.float()
    return dx.to(x.dtype)


def rope_(qkv: torch.Tensor, pos: torch.Tensor, n_rot_heads: int, head_dim: int, theta: float, inverse: bool = False):
    """Rotate the first ``n_rot_heads`` heads of each ``qkv`` row in place (q heads then k heads)."""
    if qkv.is_cuda:
        native().rope(qkv, pos, n_rot_heads, head_dim, theta, inverse)
        return qkv
    T = qkv.shape[0]
    view = qkv[:, : n_rot_heads * head_dim].reshape(T, n_rot_heads, head_dim)
    view.copy_(reference.apply_rope(view, pos.view(-1), theta, inverse))
    return qkv


def linear_rope(x: torch.Tensor, w: torch.Tensor, bias, pos: torch.Tensor, n_rot_heads: int, head_dim: int,
                theta: float) -> torch.Tensor:
    """``qkv = x w^T (+bias)`` with the rotary embedding applied to its first ``n_rot_heads`` heads at
    positions ``pos``. On the GPU the rotation runs in the GEMM's epilogue (head dim 128, more than 256
    rows); otherwise the projection is followed by the RoPE kernel."""
    if (x.is_cuda and x.dtype == torch.bfloat16 and head_dim == 128 and x.shape[0] > 256
            and (n_rot_heads * head_dim) % 128 == 0):
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        native().gemm_rope(x, w, out, bias, pos.reshape(-1), n_rot_heads * head_dim, float(theta),
                           status_tensor(x.device), 0, 0)
        return out
    out = linear(x, w, bias=bias)
    rope_(out, pos, n_rot_heads, head_dim, theta)
    return out


def linear_swiglu(x: torch.Tensor, w: torch.Tensor, keep_gu: bool = False):
    """``h = silu(x Wg^T) * (x Wu^T)`` for ``w = [Wg; Wu]`` ([2I, in]). Returns ``(h, gu)`` where
    ``gu = x w^T`` is materialised only when ``keep_gu`` (the backward needs it). On the GPU the
    SwiGLU runs in the GEMM epilogue (one kernel; I a multiple of 128); skinny products (decode
    steps) keep the split-K GEMM and the separate SwiGLU kernel."""
    inter = w.shape[0] // 2
    if x.is_cuda and x.dtype == torch.bfloat16 and inter % 128 == 0 and x.shape[0] > 256:
        h = torch.empty(x.shape[0], inter, dtype=x.dtype, device=x.device)
        gu = torch.empty(x.shape[0], 2 * inter, dtype=x.dtype, device=x.device) if keep_gu else None
        native().gemm_glu(x, w, gu, h, status_tensor(x.device), 0, 0)
        return h, gu
    gu = linear(x, w)
    return swiglu(gu), (gu if keep_gu else None)


def linear_dgrad_swiglu(dy: torch.Tensor, wd: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    """``d(gate|up)`` of a SwiGLU MLP from the down projection's output gradient: the SwiGLU backward
    of ``dy wd`` (wd [out, I]) given the saved ``gu``, fused into the dgrad GEMM's epilogue on the GPU."""
    if dy.is_cuda and dy.dtype == torch.bfloat16:
        dgu = torch.empty_like(gu)
        native().gemm_dglu(dy, wd, gu, dgu, status_tensor(dy.device), 0, 0)
        return dgu
    return swiglu_backward(linear_dgrad(dy, wd), gu)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    if gu.is_cuda:
        h = torch.empty(gu.shape[0], gu.shape[1] // 2, dtype=gu.dtype, device=gu.device)
        native().swiglu_fwd(gu, h)
        return h
    return reference.swiglu(gu)


def swiglu_backward(dh: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    if gu.is_cuda:
        dgu = torch.empty_like(gu)
        native().swiglu_bwd(dh, gu, dgu)
        return dgu
    return reference.swiglu_backward(dh, gu)


def embedding(ids: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    if table.is_cuda:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
        native().embedding_fwd(ids.reshape(-1), table, out)
        return out
    return table[ids.reshape(-1)]


def embedding_backward(ids: torch.Tensor, dout: torch.Tensor, grad: torch.Tensor) -> torch.Tensor:
    if grad.is_cuda:
        native().embedding_bwd(ids.reshape(-1), dout, grad)
        return grad
    grad.index_add_(0, ids.reshape(-1), dout.float())
    return grad


# ------------------------------------------------------------------------------------------------
# attention
# ------------------------------------------------------------------------------------------------
def attention_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    n_heads: int,
    n_kv_heads: int,
    head_dim: int,
    scale: Optional[float] = None,
    causal: bool = True,
    out: Optional[torch.Tensor] = None,
    cu_seqlens_k: Optional[torch.Tensor] = None,
    block_table: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """q: [T, Hq*D] (may be a strided view), k/v: [Tk, Hkv*D]. Returns (o [T, Hq*D], lse [Hq, T]).

    ``cu_seqlens_k`` (default: ``cu_seqlens``) lets every sequence have more keys than queries; the
    queries are then the last ones of the sequence (causal mask aligned to the end of the keys).
    With ``block_table`` ([num_seqs, max_blocks] int32) k and v are a layer's paged caches
    ([num_blocks, block_size, Hkv, D]) and sequence b's keys are the first ``len_k`` positions of
    its pages (read in place, no gather)."""
    scale = reference.default_scale(head_dim) if scale is None else scale
    T = q.shape[0]
    if q.is_cuda:
        if head_dim != 128:
            raise ValueError("the native attention kernel supports head_dim 128")
        if block_table is not None and cu_seqlens_k is None:
            raise ValueError("paged keys need cu_seqlens_k")
        o = out if out is not None else torch.empty(T, n_heads * head_dim, dtype=q.dtype, device=q.device)
        lse = torch.empty(n_heads, T, dtype=torch.float32, device=q.device)
        native().attn_fwd(q, k, v, o, lse, cu_seqlens, cu_seqlens_k, max_seqlen, n_heads, n_kv_heads, scale, causal,
                          status_tensor(q.device), block_table)
        return o, lse
    if block_table is not None:
        # gather the pages into contiguous keys for the reference path
        bs = k.shape[1]
        lens = (cu_seqlens_k[1:] - cu_seqlens_k[:-1]).tolist()
        rows = []
        for b, n in enumerate(lens):
            pk = torch.arange(n, device=k.device)
            rows.append(block_table[b, pk // bs].long() * bs + pk % bs)
        idx = torch.cat(rows) if rows else torch.zeros(0, dtype=torch.long, device=k.device)
        k = k.reshape(-1, n_kv_heads * head_dim).index_select(0, idx)
        v = v.reshape(-1, n_kv_heads * head_dim).index_select(0, idx)
    if cu_seqlens_k is not None:
        o, lse = reference.attention_varlen_qk(
            q.reshape(T, n_heads, head_dim), k.reshape(-1, n_kv_heads, head_dim), v.reshape(-1, n_kv_heads, head_dim),
            cu_seqlens, cu_seqlens_k, scale, causal,
        )
    else:
        o, lse = reference.attention_varlen(
            q.reshape(T, n_heads, head_dim), k.reshape(T, n_kv_heads, head_dim), v.reshape(T, n_kv_heads, head_dim),
            cu_seqlens, scale, causal,
        )
    o = o.reshape(T, n_heads * head_dim)
    if out is not None:
        out.copy_(o)
        o = out
    return o, lse


def attention_varlen_backward(
    dout, q, k, v, o, lse, cu_seqlens, max_seqlen, n_heads, n_kv_heads, head_dim, scale=None, causal=True,
    dq=None, dk=None, dv=None, rope_pos=None, rope_theta: float = 0.0,
):
    """Gradients w.r.t. q, k, v. ``dq/dk/dv`` may be strided views into a fused d(qkv) buffer.
    With ``rope_pos`` (int64 [T]) the inverse rotary rotation (``rope_theta``) is applied to dq and dk,
    i.e. the gradients are returned w.r.t. q and k before RoPE (fused into the finishing kernel)."""
    scale = reference.default_scale(head_dim) if scale is None else scale
    T = q.shape[0]
    if q.is_cuda:
        dq = dq if dq is not None else torch.empty(T, n_heads * head_dim, dtype=q.dtype, device=q.device)
        dk = dk if dk is not None else torch.empty(T, n_kv_heads * head_dim, dtype=q.dtype, device=q.device)
        dv = dv if dv is not None else torch.empty(T, n_kv_heads * head_dim, dtype=q.dtype, device=q.device)
        acc = workspace(q.device, "attn_acc", 3 * T * n_heads * head_dim)
        delta = workspace(q.device, "attn_delta", n_heads * T)
        if rope_pos is not None and head_dim != 128:
            raise ValueError("fused inverse RoPE needs head_dim 128")
        native().attn_bwd(q, k, v, o, dout, lse, delta, acc, dq, dk, dv, cu_seqlens, max_seqlen, n_heads,
                          n_kv_heads, scale, causal, status_tensor(q.device), rope_pos, float(rope_theta))
        return dq, dk, dv
    with torch.enable_grad():
        qf = q.detach().float().reshape(T, n_heads, head_dim).requires_grad_(True)
        kf = k.detach().float().reshape(T, n_kv_heads, head_dim).requires_grad_(True)
        vf = v.detach().float().reshape(T, n_kv_heads, head_dim).requires_grad_(True)
        of, _ = reference.attention_varlen(qf, kf, vf, cu_seqlens, scale, causal)
        gq, gk, gv = torch.autograd.grad(of, (qf, kf, vf), dout.float().reshape(T, n_heads, head_dim))
    res = []
    for g, dst in ((gq, dq), (gk, dk), (gv, dv)):
        g = g.reshape(T, -1).to(q.dtype)
        if dst is not None:
            dst.copy_(g)
            res.append(dst)
        else:
            res.append(g)
    if rope_pos is not None:
        for g, heads in ((res[0], n_heads), (res[1], n_kv_heads)):
            view = g.reshape(T, heads, head_dim)
            view.copy_(reference.apply_rope(view, rope_pos.view(-1), rope_theta, True))
    return tuple(res)


# ------------------------------------------------------------------------------------------------
# loss side
# ------------------------------------------------------------------------------------------------
def logsoftmax_label(logits: torch.Tensor, labels: torch.Tensor, with_entropy: bool = False):
    """Per row: (label logprob, logsumexp, entropy or None). logits [n, V] bf16."""
    if logits.is_cuda:
        n = logits.shape[0]
        lp = torch.empty(n, dtype=torch.float32, device=logits.device)
        lse = torch.empty(n, dtype=torch.float32, device=logits.device)
        ent = torch.empty(n, dtype=torch.float32, device=logits.device) if with_entropy else None
        native().logsoftmax_label_fwd(logits, labels, lp, lse, ent)
        return lp, lse, ent
    lp, lse, ent = reference.logsoftmax_label(logits, labels)
    return lp, lse, (ent if with_entropy else None)


def logsoftmax_label_backward(logits: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor, grad: torch.Tensor):
    """Overwrites ``logits`` with d(logits) = grad * (onehot - softmax)."""
    if logits.is_cuda:
        native().logsoftmax_label_bwd(logits, labels, lse, grad, 0)
        return logits
    probs = torch.exp(logits.float() - lse.unsqueeze(1))
    d = -probs * grad.unsqueeze(1)
    d[torch.arange(logits.shape[0]), labels] += grad
    logits.copy_(d.to(logits.dtype))
    return logits


# Vocabulary columns per chunk of the response-only LM head: the [rows, chunk] bf16 buffer is all that
# is ever materialised of the logits (36 MB for 1100 rows), instead of [rows, 151936].
LM_HEAD_CHUNK = 16384


def lm_head_logprobs(rows: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, with_entropy: bool = False,
                     chunk: int = LM_HEAD_CHUNK):
    """Response-only LM head (accerl_agent/agent_textworld.py:855-871, ``logits_to_keep`` +
    cross-entropy): per row the label log-probability of ``rows @ w^T``, its log-sum-exp and,
    optionally, the entropy. On the GPU the vocabulary is processed in chunks: a tcgen05 GEMM writes one
    [rows, chunk] tile of logits, which a kernel folds into a running (max, sum exp, sum exp * x,
    label logit) per row. Returns (logprob, lse, entropy or None), all fp32."""
    if not rows.is_cuda:
        lp, lse, ent = logsoftmax_label(linear(rows, w), labels, with_entropy)
        return lp, lse, ent
    n, V = rows.shape[0], w.shape[0]
    state = workspace(rows.device, "lm_head_state", 4 * n).view(n, 4)
    buf = workspace(rows.device, "lm_head_chunk", n * min(chunk, V), dtype=rows.dtype)
    for c0 in range(0, V, chunk):
        cw = min(chunk, V - c0)
        logits = buf[: n * cw].view(n, cw)
        linear(rows, w[c0 : c0 + cw], out=logits)
        native().lse_chunk(logits, labels, c0, c0 == 0, state)
    lp = torch.empty(n, dtype=torch.float32, device=rows.device)
    lse = torch.empty_like(lp)
    ent = torch.empty_like(lp) if with_entropy else None
    native().lse_finish(state, lp, lse, ent)
    return lp, lse, ent


def lm_head_backward(rows: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor,
                     grad: torch.Tensor, grad_w: Optional[torch.Tensor] = None, need_drows: bool = True,
                     chunk: int = LM_HEAD_CHUNK) -> Optional[torch.Tensor]:
    """Backward of ``lm_head_logprobs`` for d(logprob) = ``grad``: recomputes every logits chunk,
    turns it in place into d(logits) = grad * (onehot - softmax), accumulates ``grad_w`` (fp32 [V, H],
    optional) and, with ``need_drows``, returns d(rows) (accumulated in fp32 over the chunks)."""
    if not rows.is_cuda:
        logits = linear(rows, w)
        dlogits = logsoftmax_label_backward(logits, labels, lse, grad)
        if grad_w is not None:
            linear_wgrad(dlogits, rows, grad_w, accumulate=True)
        return linear_dgrad(dlogits, w) if need_drows else None
    n, V = rows.shape[0], w.shape[0]
    buf = workspace(rows.device, "lm_head_chunk", n * min(chunk, V), dtype=rows.dtype)
    dacc = None
    if need_drows:
        dacc = workspace(rows.device, "lm_head_drows", n * rows.shape[1]).view(n, rows.shape[1])
        dacc.zero_()
    for c0 in range(0, V, chunk):
        cw = min(chunk, V - c0)
        logits = buf[: n * cw].view(n, cw)
        linear(rows, w[c0 : c0 + cw], out=logits)
        native().logsoftmax_label_bwd(logits, labels, lse, grad, c0)
        if grad_w is not None:
            linear_wgrad(logits, rows, grad_w[c0 : c0 + cw], accumulate=True)
        if need_drows:
            gemm(logits, w[c0 : c0 + cw], dacc, b_mn=True, beta=1.0, out_dtype=torch.float32, splits=1)
    if not need_drows:
        return None
    drows = torch.empty(n, rows.shape[1], dtype=rows.dtype, device=rows.device)
    native().splitk_finish(dacc, None, None, drows)
    return drows


def policy_loss(lp, old_lp, adv, cfg, loss_scale: float):
    """Fused objective. Returns (dlp [n] fp32 = d(loss*loss_scale)/d lp, stats float64[3])."""
    if lp.is_cuda:
        dlp = torch.empty_like(lp)
        stats = torch.zeros(3, dtype=torch.float64, device=lp.device)
        native().policy_loss(lp, old_lp.float(), adv.float(), dlp, stats, cfg.mode_id, cfg.clip_eps, cfg.gipo_sigma,
                             cfg.sapo_tau_pos, cfg.sapo_tau_neg, cfg.kl_coef, loss_scale)
        return dlp, stats
    from ..algo.objectives import varlen_token_sum_loss

    x = lp.detach().float().requires_grad_(True)
    with torch.enable_grad():
        loss, stats = varlen_token_sum_loss(x, old_lp, adv, cfg)
        (g,) = torch.autograd.grad(loss * loss_scale, x)
    return g, stats


def moe_combine(ys, pos, w, k: int, residual=None, shared=None, sg=None, out=None) -> torch.Tensor:
    """MoE combine per token t: ``residual[t] + sum_j w[t,j] * ys[pos[t,j]] + sg[t] * shared[t]``
    (fp32 accumulation). ``pos``/``w``: int64 / fp32 per (token, slot) pair in token-major order."""
    T, H = pos.numel() // k, ys.shape[1]
    if ys.is_cuda:
        out = out if out is not None else torch.empty(T, H, dtype=ys.dtype, device=ys.device)
        native().moe_combine_fwd(ys, pos, w, k, residual, shared, None if sg is None else sg.reshape(-1), out)
        return out
    y = residual.float() if residual is not None else torch.zeros(T, H, dtype=torch.float32, device=ys.device)
    y = y + (ys.float().index_select(0, pos) * w.float().unsqueeze(1)).view(T, k, H).sum(1)
    if shared is not None:
        y = y + sg.reshape(-1, 1).float() * shared.float()
    if out is not None:
        out.copy_(y)
        return out
    return y.to(ys.dtype)


def moe_combine_backward(dout, ys, pos, w, k: int, dys_out) -> torch.Tensor:
    """Backward of ``moe_combine`` w.r.t. the expert rows and the weights: writes
    ``dys_out[pos[t,j]] = w[t,j] * dout[t]`` and returns ``dw[t,j] = <dout[t], ys[pos[t,j]]>`` (fp32)."""
    if dout.is_cuda:
        dw = torch.empty(pos.numel(), dtype=torch.float32, device=dout.device)
        native().moe_combine_bwd(dout.contiguous(), ys, pos, w, k, dys_out, dw)
        return dw
    g = dout.float().repeat_interleave(k, 0)
    dw = (g * ys.float().index_select(0, pos)).sum(-1)
    dys_out.index_copy_(0, pos, (g * w.float().unsqueeze(1)).to(dys_out.dtype))
    return dw


def weight_pull(plan, src_addr: int, dst: torch.Tensor) -> None:
    """Run a copy plan (``weight_map.descs_tensor``) from the device address ``src_addr`` (a peer
    GPU's buffer mapped by CUDA IPC, or a local one) into ``dst``."""
    desc, unit_start, n_units = plan
    native().weight_pull(desc, unit_start, n_units, int(src_addr), dst)


def grad_sumsq(flat_grad: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.zeros(1, dtype=torch.float64, device=flat_grad.device)
    if flat_grad.is_cuda:
        native().sumsq(flat_grad, out)
        return out
    out += flat_grad.double().pow(2).sum()
    return out


def adamw_step(master, m, v, grad, param_bf16, sumsq, lr, beta1, beta2, eps, weight_decay, max_norm, step):
    """Fused clip (by the global norm in ``sumsq``) + AdamW; also zeroes ``grad``."""
    bc1 = 1.0 - beta1 ** step
    bc2_sqrt = math.sqrt(1.0 - beta2 ** step)
    if master.is_cuda:
        native().adamw(master, m, v, grad, param_bf16, sumsq, lr, beta1, beta2, eps, weight_decay, max_norm, bc1,
                       bc2_sqrt)
        return
    coef = 1.0
    if max_norm > 0:
        norm = float(sumsq.sqrt())
        coef = min(1.0, max_norm / (norm + 1e-6))
    g = grad * coef
    master.mul_(1 - lr * weight_decay)
    m.mul_(beta1).add_(g, alpha=1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    denom = v.sqrt() / bc2_sqrt + eps
    master.addcdiv_(m, denom, value=-lr / bc1)
    param_bf16.copy_(master.to(param_bf16.dtype))
    grad.zero_()


# ------------------------------------------------------------------------------------------------
# rollout
# ------------------------------------------------------------------------------------------------
def paged_decode(q, k_cache, v_cache, block_table, seq_lens, n_heads, n_kv_heads, scale, num_splits=1, out=None,
                 impl: int = 0):
    """q: [S, Hq*D] -> [S, Hq*D]. ``impl``: 0 = a tensor-core kernel where the shape allows it (head dim
    128, at most 32 query heads per KV head, pages dividing 128 tokens), 1 = the CUDA-core kernel,
    2 = the tensor-core kernel with the query heads as MMA rows, 3 = the tensor-core kernel with the
    128 keys of a tile as MMA rows (the default of 0)."""
    S = q.shape[0]
    D = k_cache.shape[-1]
    if q.is_cuda:
        o = out if out is not None else torch.empty(S, n_heads * D, dtype=q.dtype, device=q.device)
        part_o = workspace(q.device, "decode_o", S * n_heads * num_splits * D)
        part_ml = workspace(q.device, "decode_ml", S * n_heads * num_splits * 2)
        native().paged_decode(q, k_cache, v_cache, block_table, seq_lens, o, part_o, part_ml, n_heads, n_kv_heads,
                              num_splits, scale, impl, status_tensor(q.device))
        return o
    res = reference.paged_decode(q.reshape(S, n_heads, D), k_cache, v_cache, block_table, seq_lens, scale)
    res = res.reshape(S, n_heads * D)
    if out is not None:
        out.copy_(res)
        return out
    return res


def qkv_rope_cache(qkv, pos, slot_mapping, k_cache, v_cache, n_q_heads: int, n_kv_heads: int, theta: float,
                   q_norm=None, k_norm=None, eps: float = 1e-6):
    """The engine's step after the qkv projection, in place on ``qkv`` [T, (Hq + 2 Hkv) * D]: per-head
    RMSNorm of q and k (with ``q_norm``/``k_norm``, Qwen3), rotary embedding of q and k at ``pos``,
    and the k and v heads into the paged caches at ``slot_mapping`` (rows with slot < 0 skip). One
    kernel on the GPU (head dim 128); elsewhere the separate ops in the same order."""
    D = k_cache.shape[-1]
    if qkv.is_cuda and qkv.dtype == torch.bfloat16 and D == 128:
        native().qkv_rope_cache(qkv, pos.reshape(-1), slot_mapping, k_cache, v_cache, n_q_heads, n_kv_heads,
                                float(theta), q_norm, k_norm, float(eps))
        return qkv
    T = qkv.shape[0]
    qd, kd = n_q_heads * D, n_kv_heads * D
    if q_norm is not None:
        qn, _ = rmsnorm(qkv[:, :qd].reshape(T * n_q_heads, D).clone(), q_norm, eps)
        kn, _ = rmsnorm(qkv[:, qd : qd + kd].reshape(T * n_kv_heads, D).clone(), k_norm, eps)
        qkv[:, :qd].copy_(qn.view(T, qd))
        qkv[:, qd : qd + kd].copy_(kn.view(T, kd))
    rope_(qkv, pos, n_q_heads + n_kv_heads, D, theta)
    kv_cache_write(qkv[:, qd : qd + kd], qkv[:, qd + kd :], k_cache, v_cache, slot_mapping, n_kv_heads)
    return qkv


def kv_cache_write(k, v, k_cache, v_cache, slot_mapping, n_kv_heads):
    if k.is_cuda:
        native().kv_cache_write(k, v, k_cache, v_cache, slot_mapping, n_kv_heads)
        return
    valid = slot_mapping >= 0
    slots = slot_mapping[valid].long()
    D = k_cache.shape[-1]
    kc = k_cache.view(-1, n_kv_heads, D)
    vc = v_cache.view(-1, n_kv_heads, D)
    kc[slots] = k[valid].reshape(-1, n_kv_heads, D).to(kc.dtype)
    vc[slots] = v[valid].reshape(-1, n_kv_heads, D).to(vc.dtype)


def sample(logits, temperature, seeds, offsets, num_chunks: int = 16, generator=None, top_k=None, top_p=None):
    """Sample one token per row of ``logits`` ([rows, V] bf16 on the GPU).

    ``temperature`` [rows] (<= 0: argmax), optional ``top_k`` [rows] int32 (0: off) and ``top_p``
    [rows] float32 (1: off). The random stream of row i is keyed by (``seeds[i]``, ``offsets[i]``).
    Returns (tokens int64, log-probability of each token under the untempered softmax)."""
    if logits.is_cuda:
        rows = logits.shape[0]
        tokens = torch.empty(rows, dtype=torch.long, device=logits.device)
        lps = torch.empty(rows, dtype=torch.float32, device=logits.device)
        part = workspace(logits.device, "sample_part", rows * num_chunks * 4)
        if top_k is not None:
            top_k = top_k.to(device=logits.device, dtype=torch.int32).contiguous()
        if top_p is not None:
            top_p = top_p.to(device=logits.device, dtype=torch.float32).contiguous()
        native().sample_logits(logits, temperature, seeds, offsets, tokens, lps, part, num_chunks, top_k, top_p)
        if top_k is not None or top_p is not None:
            LAUNCHES[0] += 1
        return tokens, lps
    return reference.sample_reference(logits, temperature, generator, top_k, top_p)
