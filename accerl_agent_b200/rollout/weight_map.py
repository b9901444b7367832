"""Trainer -> engine weight copy plans: which rectangle of the trainer's flat buffer lands where in the
engine's flat buffer, for any pair of layouts and any tensor-parallel rank.

The trainer keeps every parameter in one flat bf16 buffer laid out by ``ParamLayout`` for its
``--train-mode`` (trainable slots first, padded to the FSDP world size); an engine rank keeps its own
flat buffer in its layout (a TP shard has fewer heads / intermediate columns / experts). A plan is a
list of 2-D copies ``(src_off, src_ld, dst_off, dst_ld, rows, cols)`` in elements, built from the
parameter names, so the engine pulls exactly its slice straight from trainer memory (CUDA IPC) with
one kernel launch (``weight_pull`` in ``csrc/collectives.cu``) and no gather on the trainer side.

Tensor-parallel slicing (rank ``r`` of ``tp``), the Megatron scheme:
  * ``qkv_proj`` (weight and bias): rows of q heads ``[r*q/tp, ...)``, of k and of v heads likewise;
  * ``o_proj``: columns ``[r*q/tp, ...)`` (row-parallel; partial sums all-reduced);
  * ``gate_up_proj``: gate rows ``[r*I/tp, ...)`` and up rows ``[I + r*I/tp, ...)``;
  * ``down_proj``: columns ``[r*I/tp, ...)``; the shared expert of MoE layers likewise;
  * routed experts: the contiguous range of experts this rank owns (expert parallelism inside the
    TP group: every rank sees every token, runs only its experts, and the row-parallel all-reduce of
    the layer sums the experts' contributions);
  * embeddings, norms, router and ``lm_head``: replicated.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Sequence

import torch

from ..models.config import ModelConfig


@dataclass(frozen=True)
class CopyDesc:
    src_off: int
    src_ld: int
    dst_off: int
    dst_ld: int
    rows: int
    cols: int


def tp_shard_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    """Model config of one tensor-parallel rank (local head / column / expert counts)."""
    if tp == 1:
        return cfg
    import copy

    for name, val in (("num_attention_heads", cfg.num_attention_heads), ("num_key_value_heads", cfg.num_key_value_heads),
                      ("intermediate_size", cfg.intermediate_size)):
        if val % tp:
            raise ValueError(f"{name}={val} is not divisible by the tensor-parallel size {tp}")
    c = copy.deepcopy(cfg)
    c.num_attention_heads //= tp
    c.num_key_value_heads //= tp
    c.intermediate_size //= tp
    if cfg.num_experts:
        if cfg.num_experts % tp:
            raise ValueError(f"num_experts={cfg.num_experts} is not divisible by the tensor-parallel size {tp}")
        c.local_experts = cfg.num_experts // tp
        if cfg.shared_expert_intermediate_size % tp:
            raise ValueError("shared_expert_intermediate_size is not divisible by the tensor-parallel size")
        c.shared_expert_intermediate_size //= tp
    return c


def _slot_copies(name: str, shape: Sequence[int], cfg: ModelConfig, r: int, tp: int):
    """Copies of one parameter as (src_off, src_ld, dst_off, dst_ld, rows, cols) relative to the
    slot starts, for TP rank ``r``."""
    full = [(0, 1, 0, 1, 1, _numel(shape))]
    if tp == 1:
        return full
    D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    qd, kvd = Hq * D, Hkv * D
    ql, kvl = qd // tp, kvd // tp
    H = cfg.hidden_size
    if name.endswith("self_attn.qkv_proj.weight") or name.endswith("self_attn.qkv_proj.bias"):
        w = H if name.endswith("weight") else 1
        return [(r * ql * w, w, 0, w, ql, w),
                (qd * w + r * kvl * w, w, ql * w, w, kvl, w),
                ((qd + kvd) * w + r * kvl * w, w, (ql + kvl) * w, w, kvl, w)]
    if name.endswith("self_attn.o_proj.weight"):
        return [(r * ql, qd, 0, ql, H, ql)]
    if name.endswith("experts.gate_up_proj"):
        E, two_i, h = shape
        el = E // tp
        n = el * two_i * h
        return [(r * n, 1, 0, 1, 1, n)]
    if name.endswith("experts.down_proj"):
        E, h, im = shape
        el = E // tp
        n = el * h * im
        return [(r * n, 1, 0, 1, 1, n)]
    if name.endswith("gate_up_proj.weight"):  # dense MLP or shared expert [2I, H]
        two_i, h = shape
        i, il = two_i // 2, two_i // 2 // tp
        return [(r * il * h, h, 0, h, il, h), ((i + r * il) * h, h, il * h, h, il, h)]
    if name.endswith("down_proj.weight"):  # dense MLP or shared expert [H, I]
        h, i = shape
        il = i // tp
        return [(r * il, i, 0, il, h, il)]
    return full


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


def build_weight_map(cfg: ModelConfig, src_layout, dst_layout, tp_rank: int = 0, tp_size: int = 1,
                     scope: str = "all") -> List[CopyDesc]:
    """Copies that fill ``dst_layout`` (a TP rank's layout) from ``src_layout`` (the trainer's full
    layout). ``scope="trainable"`` limits them to parameters trainable in the source layout."""
    out: List[CopyDesc] = []
    for name, s in src_layout.slots.items():
        if scope == "trainable" and not s.trainable:
            continue
        d = dst_layout.slots.get(name)
        if d is None:
            raise KeyError(f"engine layout has no parameter {name}")
        for so, sl, do, dl, rows, cols in _slot_copies(name, s.shape, cfg, tp_rank, tp_size):
            out.append(CopyDesc(s.offset + so, sl, d.offset + do, dl, rows, cols))
    return coalesce(out)


def build_weight_map_multi(cfg: ModelConfig, sources, dst_layout, tp_rank: int = 0, tp_size: int = 1,
                           scope: str = "all", primary: int = 0) -> List[List[CopyDesc]]:
    """Copy plans from several trainer buffers: ``sources`` lists ``(src_layout, expert_lo,
    expert_count)`` per trainer (expert-partitioned trainers hold experts [lo, lo + count) only;
    ``count = num_experts`` for a full copy). Routed experts come from whichever trainer owns them;
    everything else from ``sources[primary]``. Returns one plan per source (possibly empty)."""
    from ..models.transformer import is_expert_param

    plans: List[List[CopyDesc]] = [[] for _ in sources]
    p_layout = sources[primary][0]
    for name, s in p_layout.slots.items():
        if scope == "trainable" and not s.trainable:
            continue
        if is_expert_param(name):
            continue
        d = dst_layout.slots.get(name)
        if d is None:
            raise KeyError(f"engine layout has no parameter {name}")
        for so, sl, do, dl, rows, cols in _slot_copies(name, s.shape, cfg, tp_rank, tp_size):
            plans[primary].append(CopyDesc(s.offset + so, sl, d.offset + do, dl, rows, cols))
    E = cfg.num_experts
    if E:
        el = E // tp_size if tp_size > 1 else E
        want_lo, want_hi = tp_rank * el if tp_size > 1 else 0, (tp_rank + 1) * el if tp_size > 1 else E
        for t, (layout, lo, cnt) in enumerate(sources):
            a, b = max(want_lo, lo), min(want_hi, lo + cnt)
            if a >= b:
                continue
            for name, s in layout.slots.items():
                if not is_expert_param(name) or (scope == "trainable" and not s.trainable):
                    continue
                d = dst_layout.slots.get(name)
                if d is None:
                    raise KeyError(f"engine layout has no parameter {name}")
                per = s.numel // s.shape[0]
                n = (b - a) * per
                plans[t].append(CopyDesc(s.offset + (a - lo) * per, n, d.offset + (a - want_lo) * per, n, 1, n))
    return [coalesce(pl) for pl in plans]


def split_by_pieces(descs: List[CopyDesc], pieces, n_sources: int) -> List[List[CopyDesc]]:
    """Copy plans against a source spread over several buffers. ``descs`` address one virtual flat
    source; ``pieces`` (sorted ``(start, end, source, shift)``) say that virtual elements
    ``[start, end)`` live in buffer ``source`` at ``element - start + shift``. The rows of a 2-D copy
    that lie inside one piece move as one 2-D copy from that buffer; a row that crosses a piece
    boundary is cut into 1-row copies. Returns one plan per source."""
    import bisect

    starts = [pc[0] for pc in pieces]
    plans: List[List[CopyDesc]] = [[] for _ in range(n_sources)]
    for d in descs:
        ld, R, C = d.src_ld, d.rows, d.cols
        first, last = d.src_off, d.src_off + (R - 1) * ld + C
        k = max(bisect.bisect_right(starts, first) - 1, 0)
        while k < len(pieces) and pieces[k][0] < last:
            a, b, src, shift = pieces[k]
            k += 1
            if b <= first:
                continue
            i0 = max(0, -(-(a - d.src_off) // ld))  # first row starting at or after a
            i1 = min(R, (b - C - d.src_off) // ld + 1) if b - C - d.src_off >= 0 else 0  # rows ending by b
            if i0 < i1:
                plans[src].append(CopyDesc(d.src_off + i0 * ld - a + shift, ld, d.dst_off + i0 * d.dst_ld, d.dst_ld,
                                           i1 - i0, C))
            for i in sorted({(a - d.src_off) // ld, (b - 1 - d.src_off) // ld}):
                if not 0 <= i < R or i0 <= i < i1:
                    continue  # outside the copy, or already moved whole
                r0 = d.src_off + i * ld
                lo, hi = max(r0, a), min(r0 + C, b)
                if lo < hi:
                    n = hi - lo
                    plans[src].append(CopyDesc(lo - a + shift, n, d.dst_off + i * d.dst_ld + (lo - r0), n, 1, n))
    return [coalesce(pl) for pl in plans]


def build_weight_map_sharded(cfg: ModelConfig, full_layout, pieces, n_sources: int, dst_layout, tp_rank: int = 0,
                             tp_size: int = 1, scope: str = "all") -> List[List[CopyDesc]]:
    """Copy plans from layer-sharded trainers (``parallel/zero3.py``): the plan of the unsharded
    layout, split by where each element lives (``shard_pieces``). Returns one plan per trainer."""
    return split_by_pieces(build_weight_map(cfg, full_layout, dst_layout, tp_rank, tp_size, scope), pieces, n_sources)


def coalesce(descs: List[CopyDesc]) -> List[CopyDesc]:
    """Merge copies that are contiguous in both buffers into single 1-D copies (identical layouts
    collapse to one copy per contiguous run)."""
    flat: List[List[int]] = []
    for d in descs:
        if d.cols == d.src_ld == d.dst_ld or d.rows == 1:
            n = d.rows * d.cols
            if flat and flat[-1][4] == 1:
                p = flat[-1]
                if p[0] + p[5] == d.src_off and p[2] + p[5] == d.dst_off:
                    p[5] += n
                    p[1] = p[3] = p[5]
                    continue
            flat.append([d.src_off, n, d.dst_off, n, 1, n])
        else:
            flat.append([d.src_off, d.src_ld, d.dst_off, d.dst_ld, d.rows, d.cols])
    return [CopyDesc(*x) for x in flat]


def map_bytes(descs: List[CopyDesc], elem: int = 2) -> int:
    return sum(d.rows * d.cols for d in descs) * elem


PULL_CHUNK = 4096  # elements per work unit of the pull kernel


def descs_tensor(descs: List[CopyDesc], device):
    """Device form of a plan for the pull kernel: ``(desc [n, 6], unit_start [n + 1], n_units)``."""
    starts = [0]
    for d in descs:
        starts.append(starts[-1] + d.rows * ((d.cols + PULL_CHUNK - 1) // PULL_CHUNK))
    desc = torch.tensor([[d.src_off, d.src_ld, d.dst_off, d.dst_ld, d.rows, d.cols] for d in descs],
                        dtype=torch.int64).reshape(-1, 6).to(device)
    return desc, torch.tensor(starts, dtype=torch.int64).to(device), starts[-1]


def apply_map_torch(src: torch.Tensor, dst: torch.Tensor, descs: List[CopyDesc]) -> None:
    """Reference implementation (CPU and tests): strided 2-D copies with torch views."""
    for d in descs:
        s = src.as_strided((d.rows, d.cols), (d.src_ld, 1), src.storage_offset() + d.src_off)
        t = dst.as_strided((d.rows, d.cols), (d.dst_ld, 1), dst.storage_offset() + d.dst_off)
        t.copy_(s)
