"""fp32 PyTorch implementations of every native op.

They serve two purposes: the oracle that each CUDA kernel test compares against, and the compute
path for CPU tensors (the gloo / CPU smoke configuration). They favour clarity over speed.
"""

from __future__ import annotations

import math
from typing import Optional, Tuple

import torch


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    y = (xf * rstd).to(x.dtype) * w
    return y.to(x.dtype), rstd.squeeze(-1)


def rmsnorm_backward(dy: torch.Tensor, x: torch.Tensor, w: torch.Tensor, rstd: torch.Tensor):
    dyf, xf, wf = dy.float(), x.float(), w.float()
    r = rstd.float().unsqueeze(-1)
    xhat = xf * r
    g = dyf * wf
    dx = r * (g - xhat * (g * xhat).mean(-1, keepdim=True))
    dw = (dyf * xhat).sum(0)
    return dx, dw


def rope_cos_sin(pos: torch.Tensor, head_dim: int, theta: float, dtype=torch.float32):
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32, device=pos.device) / head_dim))
    freqs = pos.float().unsqueeze(-1) * inv_freq
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def apply_rope(x: torch.Tensor, pos: torch.Tensor, theta: float, inverse: bool = False) -> torch.Tensor:
    """x: [T, H, D]; returns the rotated tensor in x's dtype (fp32 math)."""
    cos, sin = rope_cos_sin(pos, x.shape[-1], theta)
    if x.dtype == torch.bfloat16:
        cos = cos.to(torch.bfloat16).float()
        sin = sin.to(torch.bfloat16).float()
    if inverse:
        sin = -sin
    xf = x.float()
    out = xf * cos.unsqueeze(1) + rotate_half(xf) * sin.unsqueeze(1)
    return out.to(x.dtype)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    inter = gu.shape[-1] // 2
    g, u = gu[..., :inter], gu[..., inter:]
    return (torch.nn.functional.silu(g.float()).to(gu.dtype) * u).to(gu.dtype)


def swiglu_backward(dh: torch.Tensor, gu: torch.Tensor) -> torch.Tensor:
    inter = gu.shape[-1] // 2
    g, u = gu[..., :inter].float(), gu[..., inter:].float()
    sig = torch.sigmoid(g)
    act = g * sig
    dact = sig * (1 + g * (1 - sig))
    dhf = dh.float()
    return torch.cat([dhf * u * dact, dhf * act], dim=-1).to(gu.dtype)


def attention_varlen(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor, scale: float, causal: bool = True
) -> Tuple[torch.Tensor, torch.Tensor]:
    """q: [T, Hq, D], k/v: [T, Hkv, D]. Returns (o [T, Hq, D] in q.dtype, lse [Hq, T] fp32)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    group = Hq // Hkv
    out = torch.zeros(T, Hq, D, dtype=torch.float32, device=q.device)
    lse = torch.zeros(Hq, T, dtype=torch.float32, device=q.device)
    cu = cu_seqlens.tolist()
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        if e <= s:
            continue
        qb = q[s:e].float().transpose(0, 1)  # [Hq, L, D]
        kb = k[s:e].float().transpose(0, 1).repeat_interleave(group, 0)
        vb = v[s:e].float().transpose(0, 1).repeat_interleave(group, 0)
        scores = torch.matmul(qb, kb.transpose(1, 2)) * scale
        if causal:
            L = e - s
            mask = torch.ones(L, L, dtype=torch.bool, device=q.device).triu(1)
            scores = scores.masked_fill(mask, float("-inf"))
        lse_b = torch.logsumexp(scores, dim=-1)
        probs = torch.exp(scores - lse_b.unsqueeze(-1))
        out[s:e] = torch.matmul(probs, vb).transpose(0, 1)
        lse[:, s:e] = lse_b
    return out.to(q.dtype), lse


def attention_varlen_qk(q, k, v, cu_q, cu_k, scale: float, causal: bool = True):
    """Queries ``q[cu_q[b]:cu_q[b+1]]`` are the last ones of sequence b whose keys are
    ``k[cu_k[b]:cu_k[b+1]]`` (causal mask aligned to the end)."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    group = Hq // Hkv
    out = torch.zeros(T, Hq, D, dtype=torch.float32, device=q.device)
    lse = torch.zeros(Hq, T, dtype=torch.float32, device=q.device)
    cq, ck = cu_q.tolist(), cu_k.tolist()
    for b in range(len(cq) - 1):
        qs, qe, ks, ke = cq[b], cq[b + 1], ck[b], ck[b + 1]
        Lq, Lk = qe - qs, ke - ks
        if Lq <= 0:
            continue
        qb = q[qs:qe].float().transpose(0, 1)
        kb = k[ks:ke].float().transpose(0, 1).repeat_interleave(group, 0)
        vb = v[ks:ke].float().transpose(0, 1).repeat_interleave(group, 0)
        scores = torch.matmul(qb, kb.transpose(1, 2)) * scale
        if causal:
            qpos = torch.arange(Lq, device=q.device).unsqueeze(1) + (Lk - Lq)
            kpos = torch.arange(Lk, device=q.device).unsqueeze(0)
            scores = scores.masked_fill(kpos > qpos, float("-inf"))
        lse_b = torch.logsumexp(scores, dim=-1)
        out[qs:qe] = torch.matmul(torch.exp(scores - lse_b.unsqueeze(-1)), vb).transpose(0, 1)
        lse[:, qs:qe] = lse_b
    return out.to(q.dtype), lse


def logsoftmax_label(logits: torch.Tensor, labels: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    lp = lf.gather(1, labels.view(-1, 1)).squeeze(1) - lse
    probs = torch.softmax(lf, dim=-1)
    entropy = lse - (probs * lf).sum(-1)
    return lp, lse, entropy


def paged_decode(q, k_cache, v_cache, block_table, seq_lens, scale):
    """q: [S, Hq, D]; caches [NB, BS, Hkv, D]. Returns [S, Hq, D] (q dtype)."""
    S, Hq, D = q.shape
    bs = k_cache.shape[1]
    Hkv = k_cache.shape[2]
    group = Hq // Hkv
    out = torch.zeros(S, Hq, D, dtype=torch.float32, device=q.device)
    for s in range(S):
        n = int(seq_lens[s])
        nblk = (n + bs - 1) // bs
        blocks = block_table[s, :nblk].long()
        kk = k_cache[blocks].reshape(-1, Hkv, D)[:n].float().repeat_interleave(group, 1)
        vv = v_cache[blocks].reshape(-1, Hkv, D)[:n].float().repeat_interleave(group, 1)
        sc = torch.einsum("hd,thd->ht", q[s].float(), kk) * scale
        p = torch.softmax(sc, dim=-1)
        out[s] = torch.einsum("ht,thd->hd", p, vv)
    return out.to(q.dtype)


def sample_reference(logits: torch.Tensor, temperature: torch.Tensor, generator: Optional[torch.Generator] = None,
                     top_k: Optional[torch.Tensor] = None, top_p: Optional[torch.Tensor] = None):
    """Sampling with torch RNG (CPU path of the engine, and the oracle of the device sampler).

    Row i: argmax if temperature <= 0; otherwise softmax(x / T) restricted to the values >= the
    top_k-th largest (top_k <= 0: no restriction) and then to the nucleus of the renormalised
    distribution: the tokens, in descending probability, whose preceding cumulative mass is below
    top_p. Returns (tokens, log-probability of each token under the untempered softmax)."""
    lf = logits.float()
    logp = torch.log_softmax(lf, dim=-1)
    tokens = torch.empty(lf.shape[0], dtype=torch.long, device=lf.device)
    for i in range(lf.shape[0]):
        t = float(temperature[i])
        if t <= 0:
            tokens[i] = int(torch.argmax(lf[i]))
            continue
        z = lf[i] / t
        k = int(top_k[i]) if top_k is not None else 0
        if 0 < k < z.numel():
            z = z.masked_fill(z < torch.topk(z, k).values[-1], float("-inf"))
        probs = torch.softmax(z, dim=-1)
        p = float(top_p[i]) if top_p is not None else 1.0
        if p < 1.0:
            sorted_p, order = torch.sort(probs, descending=True)
            before = torch.cumsum(sorted_p, 0) - sorted_p
            kept = torch.zeros_like(probs).scatter_(0, order, sorted_p * (before < p))
            probs = kept / kept.sum()
        tokens[i] = int(torch.multinomial(probs, 1, generator=generator))
    return tokens, logp.gather(1, tokens.view(-1, 1)).squeeze(1)


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
