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

from typing import Dict, Optional

import torch

from .. import ops


def gate_pair(model, layer: int, grads: bool = False) -> Optional[torch.Tensor]:
    """[router weight; shared-expert gate weight] as one [E + 1, H] view of the parameter (or fp32
    gradient) storage, or None when the layer has no shared expert or the two are not adjacent."""
    p = f"model.layers.{layer}.mlp."
    get = model.g if grads else model.w
    if p + "shared_expert_gate.weight" not in model.layout.slots:
        return None
    a, b = get(p + "gate.weight"), get(p + "shared_expert_gate.weight")
    if a is None or b is None or a.data_ptr() + a.numel() * a.element_size() != b.data_ptr():
        return None
    E, H = a.shape
    return a.as_strided((E + 1, H), (H, 1))


def route(model, layer: int, h: torch.Tensor, counts: bool = False, shared_gate: Optional[list] = None):
    """Router probabilities, top-k weights and expert ids (and, with ``counts``, rows per expert).

    On the GPU the logits come from the tcgen05 GEMM (fp32 out, rounded to bf16 as the reference's
    bf16 linear gives them) and one fused kernel does softmax, top-k, renormalisation and the
    per-expert counts (``moe_router_kernel``, HF ``Qwen2MoeTopKRouter``). When ``shared_gate`` is a
    list and the layer has a shared expert, the same GEMM also computes the shared-expert gate logit
    (column E over ``gate_pair``) and the kernel appends sigmoid of it ([T] fp32) to the list."""
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp."
    Wg = model.w(p + "gate.weight")
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    if h.is_cuda and h.dtype == torch.bfloat16 and E <= 128 and k <= 8 and h.shape[0] > 0:
        T = h.shape[0]
        pair = gate_pair(model, layer) if shared_gate is not None else None
        ncol = E + (1 if pair is not None else 0)
        ld = (ncol + 3) // 4 * 4
        logits = ops.workspace(h.device, "router_logits", T * ld).view(T, ld)[:, :ncol]
        ops.gemm(h, pair if pair is not None else Wg, logits, out_dtype=torch.float32)
        probs = torch.empty(T, E, dtype=torch.float32, device=h.device)
        topw = torch.empty(T, k, dtype=torch.float32, device=h.device)
        topi = torch.empty(T, k, dtype=torch.long, device=h.device)
        cnt = torch.zeros(E, dtype=torch.int32, device=h.device)
        sg = torch.empty(T, dtype=torch.float32, device=h.device) if pair is not None else None
        ops.native().moe_router(logits, E, k, bool(cfg.norm_topk_prob), probs, topw, topi, cnt, sg)
        if sg is not None:
            shared_gate.append(sg)
        return (probs, topw, topi, cnt) if counts else (probs, topw, topi)
    logits = (h @ Wg.t()).float()
    probs = torch.softmax(logits, dim=-1)
    topw, topi = probs.topk(k, dim=-1)
    if cfg.norm_topk_prob:
        topw = topw / topw.sum(-1, keepdim=True)
    if counts:
        return probs, topw, topi, torch.bincount(topi.reshape(-1), minlength=E).to(torch.int32)
    return probs, topw, topi


def _expert_segments(topi: torch.Tensor, num_experts: int):
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=num_experts)
    bounds = [0]
    for c in counts.tolist():
        bounds.append(bounds[-1] + c)
    return order, counts, bounds


def experts_forward_local(Wgu: torch.Tensor, Wd: torch.Tensor, xs: torch.Tensor, bounds, expert_ids=None):
    """Each expert's SwiGLU MLP on its contiguous row segment ``xs[bounds[i]:bounds[i+1]]``;
    ``Wgu [E, 2I, H]`` and ``Wd [E, H, I]`` are indexed by ``expert_ids`` (default ``0..``)."""
    Im = Wd.shape[-1]
    n = xs.shape[0]
    gu = torch.empty(n, 2 * Im, dtype=xs.dtype, device=xs.device)
    ids = range(len(bounds) - 1) if expert_ids is None else expert_ids
    segs = list(zip(ids, bounds[:-1], bounds[1:]))
    for e, s, t in segs:
        if t > s:
            ops.linear(xs[s:t], Wgu[e], out=gu[s:t])
    act = ops.swiglu(gu)
    ys = torch.empty(n, Wd.shape[1], dtype=xs.dtype, device=xs.device)
    for e, s, t in segs:
        if t > s:
            ops.linear(act[s:t], Wd[e], out=ys[s:t])
    return ys, gu, act


def experts_forward(model, layer: int, xs: torch.Tensor, bounds, expert_ids=None):
    """Run each expert's SwiGLU MLP on its contiguous row segment of ``xs``."""
    p = f"model.layers.{layer}.mlp.experts."
    return experts_forward_local(model.w(p + "gate_up_proj"), model.w(p + "down_proj"), xs, bounds, expert_ids)


def experts_backward_local(Wgu, Wd, gWgu, gWd, dys: torch.Tensor, xs, gu, act, bounds, expert_ids=None):
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


def experts_backward(model, layer: int, dys: torch.Tensor, xs, gu, act, bounds, expert_ids=None):
    p = f"model.layers.{layer}.mlp.experts."
    return experts_backward_local(model.w(p + "gate_up_proj"), model.w(p + "down_proj"), model.g(p + "gate_up_proj"),
                                  model.g(p + "down_proj"), dys, xs, gu, act, bounds, expert_ids)


# ------------------------------------------------------------------------------------------------
# CUDA path: padded expert segments + one grouped tcgen05 GEMM launch per projection
# ------------------------------------------------------------------------------------------------
SEG = 128  # expert segments are padded to whole 128-row GEMM tiles


def padded_layout(counts, device):
    """Row layout of the dispatched tokens with every expert segment padded to SEG rows."""
    return padded_layout_from_pads([((c + SEG - 1) // SEG) * SEG for c in counts], device)


def padded_layout_from_pads(pads, device):
    """Grouped-GEMM metadata for expert segments of ``pads`` rows each (multiples of SEG)."""
    starts = [0]
    for pdd in pads[:-1]:
        starts.append(starts[-1] + pdd)
    tile_expert = [e for e, pdd in enumerate(pads) for _ in range(pdd // SEG)]
    meta = torch.tensor(tile_expert + starts + pads, dtype=torch.int32).to(device, non_blocking=True)
    nt = len(tile_expert)
    E = len(pads)
    return {
        "total": sum(pads),
        "num_groups": E,
        "starts": starts,
        "tile_expert": meta[:nt],
        "row_start": meta[nt : nt + E],
        "rows": meta[nt + E :],
    }


def device_padded_layout(topi: torch.Tensor, num_experts: int, lo: int = 0, El: Optional[int] = None,
                         counts: Optional[torch.Tensor] = None):
    """Grouped-GEMM layout from torch device ops, with no host synchronisation (the formulation that
    ``device_dispatch`` computes in two kernel launches; kept as its oracle and for CPU tensors).

    The pairs ``(token, slot)`` of ``topi`` are sorted by expert; experts ``[lo, lo + El)`` get row
    segments padded to SEG rows, laid out back to back. Sizes are bounded on the host without reading
    the counts: ``total = round_up(n + El * (SEG - 1), SEG)`` rows always hold every segment, and the
    128-row tiles past the real end carry ``tile_expert = -1`` (the GEMM skips them). Pairs routed to
    experts outside the range (tensor-parallel engine shards) are sent to the extra row ``total``.
    Returns ``(order, rows_sorted, valid_sorted, layout)``: the sorting permutation, every sorted
    pair's row and whether it runs here."""
    flat = topi.reshape(-1)
    n = flat.numel()
    El = num_experts if El is None else El
    dev = flat.device
    order = torch.argsort(flat, stable=True)
    e_sorted = flat.index_select(0, order)
    if counts is None:
        # scatter-add, not bincount: bincount sizes its output from the data (a device->host sync)
        counts = torch.zeros(num_experts, dtype=torch.long, device=dev).scatter_add_(0, flat, torch.ones_like(flat))
    else:
        counts = counts.to(torch.long)
    cstart = torch.cumsum(counts, 0) - counts
    cl = counts[lo : lo + El]
    pads = torch.div(cl + (SEG - 1), SEG, rounding_mode="floor") * SEG
    ends = torch.cumsum(pads, 0)
    starts = ends - pads
    total = ((n + El * (SEG - 1) + SEG - 1) // SEG) * SEG
    tiles = total // SEG
    te = torch.searchsorted(ends, torch.arange(tiles, device=dev, dtype=ends.dtype) * SEG, right=True)
    tile_expert = torch.where(te < El, te, torch.full_like(te, -1)).to(torch.int32)
    e_loc = e_sorted - lo
    valid = (e_loc >= 0) & (e_loc < El)
    e_idx = e_loc.clamp(0, El - 1)
    rows = starts.index_select(0, e_idx) + torch.arange(n, device=dev) - cstart.index_select(0, e_sorted)
    rows = torch.where(valid, rows, torch.full_like(rows, total))
    lay = {"total": total, "num_groups": El, "tile_expert": tile_expert, "row_start": starts.to(torch.int32),
           "rows": pads.to(torch.int32), "counts": counts}
    return order, rows, valid, lay


def _grouped(a, a_mn, b, b_mn, out, M, N, K, mode, lay, b_stride, c_stride=0, beta=0.0, row_dst=None):
    ops.native().grouped_gemm(a, a_mn, b, b_mn, out, M, N, K, beta, mode, lay["tile_expert"], lay["row_start"],
                              lay["rows"], lay["num_groups"], b_stride, c_stride, ops.status_tensor(a.device),
                              row_dst)


def experts_forward_grouped(model, layer: int, xs_pad: torch.Tensor, lay, out=None):
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp.experts."
    E, Im, H = model.w(p + "gate_up_proj").shape[0], cfg.moe_intermediate_size, cfg.hidden_size
    Wgu = model.w(p + "gate_up_proj").reshape(E * 2 * Im, H)
    Wd = model.w(p + "down_proj").reshape(E * H, Im)
    R = lay["total"]
    gu = torch.empty(R, 2 * Im, dtype=xs_pad.dtype, device=xs_pad.device)
    _grouped(xs_pad, False, Wgu, False, gu, R, 2 * Im, H, 1, lay, 2 * Im)
    act = ops.swiglu(gu)
    ys = out if out is not None else torch.empty(R, H, dtype=xs_pad.dtype, device=xs_pad.device)
    _grouped(act, False, Wd, False, ys, R, H, Im, 1, lay, H)
    return ys, gu, act


def experts_backward_grouped(model, layer: int, dys_pad, xs_pad, gu, act, lay):
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp.experts."
    E, Im, H = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size
    Wgu = model.w(p + "gate_up_proj").reshape(E * 2 * Im, H)
    Wd = model.w(p + "down_proj").reshape(E * H, Im)
    gWgu, gWd = model.g(p + "gate_up_proj"), model.g(p + "down_proj")
    R = lay["total"]
    dact = torch.empty(R, Im, dtype=dys_pad.dtype, device=dys_pad.device)
    _grouped(dys_pad, False, Wd, True, dact, R, Im, H, 1, lay, H)
    if gWd is not None:
        _grouped(dys_pad, True, act, True, gWd.view(E * H, Im), H, Im, R, 2, lay, 0, H, beta=1.0)
    dgu = ops.swiglu_backward(dact, gu)
    del dact
    dxs = torch.empty(R, H, dtype=dys_pad.dtype, device=dys_pad.device)
    _grouped(dgu, False, Wgu, True, dxs, R, H, 2 * Im, 1, lay, 2 * Im)
    if gWgu is not None:
        _grouped(dgu, True, xs_pad, True, gWgu.view(E * 2 * Im, H), 2 * Im, H, R, 2, lay, 0, 2 * Im, beta=1.0)
    return dxs


def moe_forward(model, layer: int, h: torch.Tensor, residual: torch.Tensor, save: bool):
    """MoE MLP of one layer: ``residual + sum_j w_j expert_j(h) (+ shared expert)``. Three paths:
    expert parallelism (``_moe_forward_ep``), the CUDA bf16 path (``_moe_forward_device``), and the
    host path below (CPU tensors, other dtypes) with per-expert loops."""
    cfg = model.cfg
    k = cfg.num_experts_per_tok
    ep = getattr(model, "expert_parallel", None)
    if ep is not None:
        return _moe_forward_ep(model, layer, h, residual, save, ep)
    if h.is_cuda and h.dtype == torch.bfloat16:
        shared_gate: list = []
        probs, topw, topi = route(model, layer, h, shared_gate=shared_gate)
        return _moe_forward_device(model, layer, h, residual, save, probs, topw, topi,
                                   sg=shared_gate[0].view(-1, 1) if shared_gate else None)
    probs, topw, topi = route(model, layer, h)
    w_act = topw.to(h.dtype)
    order, counts, bounds = _expert_segments(topi, cfg.num_experts)
    El = cfg.local_experts
    if El is not None and El != cfg.num_experts:
        # tensor-parallel engine shard: only the (token, slot) pairs routed to this rank's experts;
        # the caller all-reduces the partial outputs of the ranks
        lo = cfg.expert_offset
        a, b = bounds[lo], bounds[lo + El]
        order, counts = order[a:b], counts[lo : lo + El]
        bounds = [x - a for x in bounds[lo : lo + El + 1]]
    tok = torch.div(order, k, rounding_mode="floor")
    xs = h.index_select(0, tok)
    ys, gu, act = experts_forward(model, layer, xs, bounds)
    rows = torch.arange(order.numel(), device=h.device)
    # per (token, slot) pair in token-major order: its row in ``ys`` and its weight (pairs this rank
    # does not run keep weight 0)
    n_pairs = topi.numel()
    pos_pairs = torch.zeros(n_pairs, dtype=torch.long, device=h.device)
    pos_pairs[order] = rows
    w_pairs = torch.zeros(n_pairs, dtype=torch.float32, device=h.device)
    w_pairs[order] = w_act.reshape(-1).float().index_select(0, order)
    if ys.shape[0] == 0:
        # no pair runs here (a tensor-parallel shard whose experts got no tokens): row 0 must exist
        ys = torch.zeros(1, cfg.hidden_size, dtype=h.dtype, device=h.device)
    cache: Dict[str, torch.Tensor] = {}
    sy, sg = _shared_expert(model, layer, h, cache if save else None)
    out = ops.moe_combine(ys, pos_pairs, w_pairs, k, residual=residual, shared=sy, sg=sg)
    if save:
        cache.update(probs=probs, topw=topw, topi=topi, order=order, tok=tok, xs=xs, gu=gu, act=act, ys=ys,
                     pos_pairs=pos_pairs, w_pairs=w_pairs)
        cache["bounds"] = torch.tensor(bounds)
    return out, cache


def _moe_forward_ep(model, layer: int, h: torch.Tensor, residual: torch.Tensor, save: bool, ep):
    """Expert-parallel forward with one host synchronisation per layer, hidden behind GPU work.

    The router kernel gives the per-expert counts on the device; their all-gather and the copy of the
    ``W x E`` count matrix to pinned host memory are queued first, then the sort of the pairs and the
    shared expert. The host waits only for the copy, so it computes the dispatch plan while the GPU
    runs the shared expert; the exchange, the expert GEMMs and the combine follow."""
    import numpy as np

    cfg = model.cfg
    k = cfg.num_experts_per_tok
    shared_gate: list = []
    probs, topw, topi, counts = route(model, layer, h, counts=True, shared_gate=shared_gate)
    pending = ep.exchange_counts(counts)
    flat = topi.reshape(-1)
    order = torch.argsort(flat, stable=True)
    e_sorted = flat.index_select(0, order)
    tok = torch.div(order, k, rounding_mode="floor")
    cache: Dict[str, torch.Tensor] = {}
    sy, sg = _shared_expert(model, layer, h, cache if save else None,
                            shared_gate[0].view(-1, 1) if shared_gate else None)
    C = ep.wait_counts(pending)
    bounds = [0] + np.cumsum(C[ep.rank]).tolist()
    ys, ep_state = ep.forward(model, layer, h, tok, e_sorted, counts, bounds, C=C)
    n_pairs = topi.numel()
    pos_pairs = torch.empty(n_pairs, dtype=torch.long, device=h.device)
    pos_pairs[order] = torch.arange(n_pairs, device=h.device)
    w_pairs = torch.empty(n_pairs, dtype=torch.float32, device=h.device)
    w_pairs[order] = topw.to(h.dtype).reshape(-1).float().index_select(0, order)
    out = ops.moe_combine(ys, pos_pairs, w_pairs, k, residual=residual, shared=sy, sg=sg)
    if save:
        cache.update(probs=probs, topw=topw, topi=topi, order=order, tok=tok, xs=None, gu=None, act=None, ys=ys,
                     pos_pairs=pos_pairs, w_pairs=w_pairs)
        cache["bounds"] = torch.tensor(bounds)
        cache["ep_state"] = ep_state  # type: ignore[assignment]
    return out, cache


def _shared_expert(model, layer: int, h: torch.Tensor, cache, sg: Optional[torch.Tensor] = None):
    """Shared expert output and its sigmoid gate ([T, 1] fp32; computed here unless the router
    kernel already produced it)."""
    cfg = model.cfg
    if cfg.shared_expert_intermediate_size <= 0:
        return None, None
    p = f"model.layers.{layer}.mlp."
    if cache is not None:
        sgu = ops.linear(h, model.w(p + "shared_expert.gate_up_proj.weight"))
        sact = ops.swiglu(sgu)
    else:
        sact, sgu = ops.linear_swiglu(h, model.w(p + "shared_expert.gate_up_proj.weight"))
    sy = ops.linear(sact, model.w(p + "shared_expert.down_proj.weight"))
    if sg is None:
        sg = torch.sigmoid((h @ model.w(p + "shared_expert_gate.weight").t()).float())
    if cache is not None:
        cache.update(sgu=sgu, sact=sact, sy=sy, sg=sg)
    return sy, sg


def device_dispatch(topi: torch.Tensor, topw: torch.Tensor, h: torch.Tensor, num_experts: int, lo: int, El: int,
                    zero_pad: bool):
    """Dispatch in two kernel launches (``moe_layout``), with no host synchronisation and no sort.

    Gives the padded layout of experts ``[lo, lo + El)`` (the same rows as ``device_padded_layout``:
    an expert's pairs in token-major order), every (token, slot) pair's row and its weight (rounded
    to the activation dtype; 0 for pairs routed outside the range, whose row is ``total``), and the
    expert inputs ``xs[row] = h[token]``. With ``zero_pad`` the padding rows of ``xs`` are zero.
    Returns ``(xs, pos_pairs, w_pairs, lay)``."""
    n = topi.numel()
    dev = h.device
    total = ((n + El * (SEG - 1) + SEG - 1) // SEG) * SEG
    tiles = total // SEG
    xs = torch.empty(total, h.shape[1], dtype=h.dtype, device=dev)
    meta = torch.empty(tiles + 2 * El + num_experts, dtype=torch.int32, device=dev)
    te, rs, rows, cnt = (meta[:tiles], meta[tiles : tiles + El], meta[tiles + El : tiles + 2 * El],
                         meta[tiles + 2 * El :])
    pos = torch.empty(n, dtype=torch.long, device=dev)
    w = torch.empty(n, dtype=torch.float32, device=dev)
    hist = ops.workspace(dev, "moe_layout_hist", ((n + 1023) // 1024) * num_experts, dtype=torch.int32)
    ops.native().moe_layout(topi.contiguous(), topw.float().contiguous(), h.contiguous(), num_experts, lo, El, total,
                            xs, bool(zero_pad), hist, pos, w, te, rs, rows, cnt)
    lay = {"total": total, "num_groups": El, "tile_expert": te, "row_start": rs, "rows": rows, "counts": cnt}
    return xs, pos, w, lay


def _moe_forward_device(model, layer: int, h, residual, save: bool, probs, topw, topi, sg=None):
    """CUDA path without host synchronisation: one-pass device dispatch, grouped GEMMs over the
    bounded tile count, fused combine. Training (``save``) zeroes the padded input rows because the
    weight-gradient contraction runs over them; inference leaves them uninitialised (their output
    rows are never read)."""
    cfg = model.cfg
    k = cfg.num_experts_per_tok
    El = cfg.local_experts if cfg.local_experts is not None else cfg.num_experts
    lo = cfg.expert_offset if El != cfg.num_experts else 0
    xs, pos_pairs, w_pairs, lay = device_dispatch(topi, topw, h, cfg.num_experts, lo, El, zero_pad=save)
    R = lay["total"]
    ys_full = torch.empty(R + 1, cfg.hidden_size, dtype=h.dtype, device=h.device)
    ys_full[R].zero_()  # the row of pairs that do not run here (weight 0)
    ys, gu, act = experts_forward_grouped(model, layer, xs, lay, out=ys_full[:R])
    cache: Dict[str, torch.Tensor] = {}
    sy, sg = _shared_expert(model, layer, h, cache if save else None, sg)
    out = ops.moe_combine(ys_full, pos_pairs, w_pairs, k, residual=residual, shared=sy, sg=sg)
    if save:
        cache.update(probs=probs, topw=topw, topi=topi, xs=xs, gu=gu, act=act, ys=ys_full, pos_pairs=pos_pairs,
                     w_pairs=w_pairs)
        cache["layout"] = lay  # type: ignore[assignment]
    return out, cache


def _router_shared_backward_device(model, layer: int, m, h: torch.Tensor, dx3: torch.Tensor, dw: torch.Tensor,
                                   dh: torch.Tensor) -> torch.Tensor:
    """GPU backward of the router and the shared expert, added into ``dh`` ([T, H] fp32).

    ``moe_router_bwd`` (one warp per token) turns the routing-weight gradients into router-logit
    gradients and, with a shared expert, appends the gate-logit gradient as column E and writes the
    gate-scaled output gradient dsy. Two tcgen05 GEMMs against [router; shared gate] (one
    [E + 1, H] view of the flat buffers) then give the input gradient and the weight gradients of
    both; the shared expert's MLP backward follows from dsy."""
    cfg = model.cfg
    p = f"model.layers.{layer}.mlp."
    T, H = dx3.shape
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    shared = cfg.shared_expert_intermediate_size > 0
    pair = gate_pair(model, layer) if shared else None
    E_pad = (E + 1 + 63) // 64 * 64
    dlog = ops.workspace(dx3.device, "router_dlogits", T * E_pad, dtype=torch.bfloat16).view(T, E_pad)
    dsy = torch.empty_like(dx3) if shared else None
    sg = m["sg"].reshape(-1).float().contiguous() if shared else None
    ops.native().moe_router_bwd(m["probs"], m["topi"], m["topw"].float().contiguous(),
                                dw.reshape(-1, k).float().contiguous(), bool(cfg.norm_topk_prob),
                                dx3 if shared else None, m["sy"] if shared else None, sg, dlog, dsy)
    if shared:
        if pair is None:
            raise RuntimeError("the shared-expert gate must follow the router in the parameter layout")
        ncol, W, G = E + 1, pair, gate_pair(model, layer, grads=True)
    else:
        ncol, W, G = E, model.w(p + "gate.weight"), model.g(p + "gate.weight")
    ops.gemm(dlog[:, :ncol], W, dh, b_mn=True, beta=1.0, out_dtype=torch.float32)  # dh += dlogits [W]
    if G is not None:
        ops.linear_wgrad(dlog[:, :ncol], h, G, accumulate=True)
    if shared:
        dsact = ops.linear_dgrad(dsy, model.w(p + "shared_expert.down_proj.weight"))
        g = model.g(p + "shared_expert.down_proj.weight")
        if g is not None:
            ops.linear_wgrad(dsy, m["sact"], g)
        dsgu = ops.swiglu_backward(dsact, m["sgu"])
        ops.gemm(dsgu, model.w(p + "shared_expert.gate_up_proj.weight"), dh, b_mn=True, beta=1.0,
                 out_dtype=torch.float32)
        g = model.g(p + "shared_expert.gate_up_proj.weight")
        if g is not None:
            ops.linear_wgrad(dsgu, h, g)
    out = torch.empty(T, H, dtype=dx3.dtype, device=dx3.device)
    ops.native().splitk_finish(dh, None, None, out)
    return out


def moe_backward(model, layer: int, dx3: torch.Tensor, c) -> torch.Tensor:
    cfg = model.cfg
    m = c.mlp
    h = c.h2
    k = cfg.num_experts_per_tok
    p = f"model.layers.{layer}.mlp."
    pos_pairs, w_pairs, ys = m["pos_pairs"], m["w_pairs"], m["ys"]
    bounds = m["bounds"].tolist() if "bounds" in m else None
    ep = getattr(model, "expert_parallel", None)
    dx3c = dx3.contiguous()
    if "layout" in m:
        lay = m["layout"]
        # pad rows stay 0; one spare row for the device layout's row of pairs that do not run here
        dys = torch.zeros(lay["total"] + 1, cfg.hidden_size, dtype=dx3.dtype, device=dx3.device)
    else:
        dys = torch.empty(ys.shape[0], cfg.hidden_size, dtype=dx3.dtype, device=dx3.device)
    dw = ops.moe_combine_backward(dx3c, ys, pos_pairs, w_pairs, k, dys)
    if ep is not None:
        dxs = ep.backward(model, layer, dys, m["ep_state"])
    elif "layout" in m:
        R = m["layout"]["total"]
        dxs = experts_backward_grouped(model, layer, dys[:R], m["xs"], m["gu"], m["act"], m["layout"])
    else:
        dxs = experts_backward(model, layer, dys, m["xs"], m["gu"], m["act"], bounds)
    # every pair's input-gradient row back to its token (unit weights)
    dh = ops.moe_combine(dxs, pos_pairs, torch.ones_like(w_pairs), k).float()
    if dx3.is_cuda and dx3.dtype == torch.bfloat16:
        return _router_shared_backward_device(model, layer, m, h, dx3c, dw, dh)
    # router
    dtopw = dw.view(-1, k)
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
