"""Mixture-of-experts MLP (Qwen2-MoE / Qwen3-MoE semantics) forward and backward.

Router: ``softmax(h W_g^T)`` in fp32, top-k, optional renormalisation of the kept weights
(``norm_topk_prob``), weights cast to the activation dtype; Qwen2-MoE adds a shared expert scaled by
``sigmoid(h W_sg^T)`` (installed transformers ``models/qwen2_moe/modeling_qwen2_moe.py:295-370``).
Dispatch sorts the (token, slot) pairs by expert so each expert's rows are one contiguous segment;
the expert MLPs run as tcgen05 GEMMs on those segments and the combine is a weighted index-add in
fp32. With expert parallelism (``parallel/expert_parallel.py``) the segments of remote experts are
exchanged between ranks before and after the expert GEMMs.
"""

from __future__ import annotations

from typing import Dict, Tuple

import torch

from .. import ops


def route(model, layer: int, h: torch.Tensor):
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp."
    logits = (h @ model.w(p + "gate.weight").t()).float()
    probs = torch.softmax(logits, dim=-1)
    topw, topi = probs.topk(cfg.num_experts_per_tok, dim=-1)
    if cfg.norm_topk_prob:
        topw = topw / topw.sum(-1, keepdim=True)
    return probs, topw, topi


def _expert_segments(topi: torch.Tensor, num_experts: int):
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=num_experts)
    bounds = [0]
    for c in counts.tolist():
        bounds.append(bounds[-1] + c)
    return order, counts, bounds


def experts_forward(model, layer: int, xs: torch.Tensor, bounds, expert_ids=None):
    """Run each expert's SwiGLU MLP on its contiguous row segment of ``xs``."""
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp.experts."
    Wgu = model.w(p + "gate_up_proj")
    Wd = model.w(p + "down_proj")
    Im = cfg.moe_intermediate_size
    n = xs.shape[0]
    gu = torch.empty(n, 2 * Im, dtype=xs.dtype, device=xs.device)
    ids = range(len(bounds) - 1) if expert_ids is None else expert_ids
    segs = list(zip(ids, bounds[:-1], bounds[1:]))
    for e, s, t in segs:
        if t > s:
            ops.linear(xs[s:t], Wgu[e], out=gu[s:t])
    act = ops.swiglu(gu)
    ys = torch.empty(n, cfg.hidden_size, dtype=xs.dtype, device=xs.device)
    for e, s, t in segs:
        if t > s:
            ops.linear(act[s:t], Wd[e], out=ys[s:t])
    return ys, gu, act


def experts_backward(model, layer: int, dys: torch.Tensor, xs, gu, act, bounds, expert_ids=None):
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp.experts."
    Wgu, Wd = model.w(p + "gate_up_proj"), model.w(p + "down_proj")
    gWgu, gWd = model.g(p + "gate_up_proj"), model.g(p + "down_proj")
    ids = range(len(bounds) - 1) if expert_ids is None else expert_ids
    segs = list(zip(ids, bounds[:-1], bounds[1:]))
    dact = torch.empty_like(act)
    for e, s, t in segs:
        if t > s:
            ops.linear_dgrad(dys[s:t], Wd[e], out=dact[s:t])
            if gWd is not None:
                ops.linear_wgrad(dys[s:t], act[s:t], gWd[e])
    dgu = ops.swiglu_backward(dact, gu)
    dxs = torch.empty_like(xs)
    for e, s, t in segs:
        if t > s:
            ops.linear_dgrad(dgu[s:t], Wgu[e], out=dxs[s:t])
            if gWgu is not None:
                ops.linear_wgrad(dgu[s:t], xs[s:t], gWgu[e])
    return dxs


def moe_forward(model, layer: int, h: torch.Tensor, residual: torch.Tensor, save: bool):
    cfg = model.cfg
    k = cfg.num_experts_per_tok
    probs, topw, topi = route(model, layer, h)
    w_act = topw.to(h.dtype)
    order, counts, bounds = _expert_segments(topi, cfg.num_experts)
    tok = torch.div(order, k, rounding_mode="floor")
    xs = h.index_select(0, tok)
    ep = getattr(model, "expert_parallel", None)
    if ep is not None:
        ys, gu, act, ep_state = ep.forward(model, layer, xs, counts)
    else:
        ys, gu, act = experts_forward(model, layer, xs, bounds)
        ep_state = None
    w_sorted = w_act.reshape(-1).index_select(0, order)
    y = torch.zeros(h.shape[0], cfg.hidden_size, dtype=torch.float32, device=h.device)
    y.index_add_(0, tok, ys.float() * w_sorted.float().unsqueeze(1))
    cache: Dict[str, torch.Tensor] = {}
    if cfg.shared_expert_intermediate_size > 0:
        p = f"model.layers.{layer}.mlp."
        sgu = ops.linear(h, model.w(p + "shared_expert.gate_up_proj.weight"))
        sact = ops.swiglu(sgu)
        sy = ops.linear(sact, model.w(p + "shared_expert.down_proj.weight"))
        sg = torch.sigmoid((h @ model.w(p + "shared_expert_gate.weight").t()).float())
        y += sg * sy.float()
        if save:
            cache.update(sgu=sgu, sact=sact, sy=sy, sg=sg)
    out = (residual.float() + y).to(h.dtype)
    if save:
        cache.update(probs=probs, topw=topw, topi=topi, order=order, tok=tok, xs=xs, gu=gu, act=act, ys=ys,
                     w_sorted=w_sorted)
        cache["bounds"] = torch.tensor(bounds)
        if ep_state is not None:
            cache["ep_state"] = ep_state  # type: ignore[assignment]
    return out, cache


def moe_backward(model, layer: int, dx3: torch.Tensor, c) -> torch.Tensor:
    cfg = model.cfg
    m = c.mlp
    h = c.h2
    k = cfg.num_experts_per_tok
    p = f"model.layers.{layer}.mlp."
    tok, order = m["tok"], m["order"]
    dxg = dx3.index_select(0, tok)
    dys = (dxg.float() * m["w_sorted"].float().unsqueeze(1)).to(dx3.dtype)
    dw_sorted = (dxg.float() * m["ys"].float()).sum(-1)
    bounds = m["bounds"].tolist()
    ep = getattr(model, "expert_parallel", None)
    if ep is not None:
        dxs = ep.backward(model, layer, dys, m)
    else:
        dxs = experts_backward(model, layer, dys, m["xs"], m["gu"], m["act"], bounds)
    dh = torch.zeros(h.shape[0], cfg.hidden_size, dtype=torch.float32, device=h.device)
    dh.index_add_(0, tok, dxs.float())
    # router
    dtopw = torch.zeros(order.numel(), dtype=torch.float32, device=h.device)
    dtopw[order] = dw_sorted
    dtopw = dtopw.view(-1, k)
    topw = m["topw"]
    if cfg.norm_topk_prob:
        probs_k = m["probs"].gather(1, m["topi"])
        S = probs_k.sum(-1, keepdim=True)
        dtopw = (dtopw - (dtopw * topw).sum(-1, keepdim=True)) / S
    probs = m["probs"]
    dprobs = torch.zeros_like(probs).scatter_(1, m["topi"], dtopw)
    dlogits = probs * (dprobs - (dprobs * probs).sum(-1, keepdim=True))
    Wg = model.w(p + "gate.weight")
    dh += dlogits @ Wg.float()
    gWg = model.g(p + "gate.weight")
    if gWg is not None:
        gWg += dlogits.t() @ h.float()
    if cfg.shared_expert_intermediate_size > 0:
        sg, sy = m["sg"], m["sy"]
        dsy = (dx3.float() * sg).to(dx3.dtype)
        dsg = (dx3.float() * sy.float()).sum(-1, keepdim=True) * sg * (1 - sg)
        dsact = ops.linear_dgrad(dsy, model.w(p + "shared_expert.down_proj.weight"))
        g = model.g(p + "shared_expert.down_proj.weight")
        if g is not None:
            ops.linear_wgrad(dsy, m["sact"], g)
        dsgu = ops.swiglu_backward(dsact, m["sgu"])
        dh += ops.linear_dgrad(dsgu, model.w(p + "shared_expert.gate_up_proj.weight")).float()
        g = model.g(p + "shared_expert.gate_up_proj.weight")
        if g is not None:
            ops.linear_wgrad(dsgu, h, g)
        Wsg = model.w(p + "shared_expert_gate.weight")
        dh += dsg * Wsg.float()
        g = model.g(p + "shared_expert_gate.weight")
        if g is not None:
            g += dsg.t() @ h.float()
    return dh.to(dx3.dtype)
