"""Cross-rank balancing of the packs of one optimizer window.

Every trainer rank draws its packs from its own replay shard (accerl_agent/agent_textworld.py:736-798),
so the work of a window differs from rank to rank: its token count and, through causal attention,
the sum of squared sequence lengths. The ranks meet at the end of every optimizer step, so the step
lasts as long as the busiest rank (measured on 2 B200s: up to 153 ms per 1.2 s step spent waiting).
The gradient is a sum over all packs of all ranks and the loss is normalised by the global target-token
count, so which rank computes a pack does not change the step (up to floating-point summation order).
``plan`` reassigns packs to even out the estimated work; ``exchange`` moves the packs that change rank.

1. Every rank all-gathers (cost, tokens, targets, sequences, max length) of its packs.
2. Every rank computes the same assignment: packs by descending cost, each to the least-loaded rank,
   ties to the pack's own rank and then to the lowest rank (longest-processing-time-first scheduling).
3. A pack that changes rank is sent as its three device buffers (int64 ids/positions/labels/indices,
   float32 old log-probs/advantages, int32 cu_seqlens) with point-to-point copies (NCCL over NVLink on
   GPUs, gloo on CPU ranks). A pack is a few hundred KB, so this costs microseconds per step.

The cost model is in FLOP units of the GEMMs: a token costs 6 FLOPs per linear parameter it passes
through (forward + backward), and a causal sequence of length L adds 7 L^2 head_dim q_heads FLOPs
per layer (2 L^2 head_dim q_heads forward, 2.5 times that backward), weighted by 2 because the
attention kernels run at about half the GEMM rate.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist

ATTENTION_WEIGHT = 2.0
_META = 5  # cost, tokens, targets, sequences, max sequence length


def linear_flops_per_token(cfg) -> float:
    """Forward + backward FLOPs of the linear layers for one token (LM head excluded: it runs only on
    the target rows, which the target count accounts for)."""
    H = cfg.hidden_size
    attn = H * cfg.qkv_dim + cfg.q_dim * H
    per_layer = []
    for layer in range(cfg.num_hidden_layers):
        if cfg.layer_is_moe(layer):
            mlp = 3 * H * (cfg.num_experts_per_tok * cfg.moe_intermediate_size + cfg.shared_expert_intermediate_size)
        else:
            mlp = 3 * H * cfg.intermediate_size
        per_layer.append(attn + mlp)
    return 6.0 * float(sum(per_layer))


def pack_cost(cfg, seq_lengths: Sequence[int], n_targets: int) -> float:
    lens = np.asarray(seq_lengths, dtype=np.float64)
    tokens = float(lens.sum())
    attn = ATTENTION_WEIGHT * 7.0 * cfg.head_dim * cfg.num_attention_heads * cfg.num_hidden_layers
    head = 6.0 * cfg.hidden_size * cfg.vocab_size
    return tokens * linear_flops_per_token(cfg) + float((lens * lens).sum()) * attn + n_targets * head


@dataclass(frozen=True)
class Move:
    src: int
    dst: int
    index: int  # position of the pack in its owner's window
    tokens: int
    targets: int
    seqs: int
    max_seqlen: int


def gather_meta(local: np.ndarray, group=None) -> np.ndarray:
    """All-gather the [packs, 5] float64 metadata of every rank: returns [world, packs, 5]."""
    world = dist.get_world_size(group)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.from_numpy(np.ascontiguousarray(local, dtype=np.float64)).to(dev)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t, group=group)
    return torch.stack(parts).cpu().numpy()


def plan(meta: np.ndarray) -> Tuple[List[List[Tuple[int, int]]], List[Move]]:
    """Deterministic longest-processing-time-first assignment of every rank's packs. Every rank keeps
    as many packs as it drew (expert-parallel layers run a collective per pack, so every rank must run
    the same number of forward and backward passes). Returns, per rank, the (owner, index) pairs it
    computes, and the packs that change rank."""
    world, packs, _ = meta.shape
    cap = [int((meta[r, :, 1] > 0).sum()) for r in range(world)]
    items = [(-float(meta[r, i, 0]), r, i) for r in range(world) for i in range(packs) if meta[r, i, 1] > 0]
    items.sort()
    load = [0.0] * world
    assign: List[List[Tuple[int, int]]] = [[] for _ in range(world)]
    for neg_cost, owner, i in items:
        open_ranks = [r for r in range(world) if len(assign[r]) < cap[r]]
        low = min(load[r] for r in open_ranks)
        dst = owner if (owner in open_ranks and load[owner] == low) else next(r for r in open_ranks if load[r] == low)
        load[dst] -= neg_cost
        assign[dst].append((owner, i))
    moves = []
    for dst in range(world):
        for owner, i in assign[dst]:
            if owner != dst:
                m = meta[owner, i]
                moves.append(Move(owner, dst, i, int(m[1]), int(m[2]), int(m[3]), int(m[4])))
    moves.sort(key=lambda mv: (mv.src, mv.index))
    return assign, moves


def exchange(moves: List[Move], rank: int, outgoing: Dict[int, Tuple[torch.Tensor, torch.Tensor, torch.Tensor]],
             device: torch.device, group=None) -> Dict[Tuple[int, int], Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]:
    """Send this rank's moving packs (``outgoing[index] = (ints, floats, cu)``) and receive the packs
    moving here. Returns the received buffers keyed by (owner, index)."""
    ops: List[dist.P2POp] = []
    received: Dict[Tuple[int, int], Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = {}
    for mv in moves:
        if mv.src == rank:
            for t in outgoing[mv.index]:
                ops.append(dist.P2POp(dist.isend, t, mv.dst, group))
        elif mv.dst == rank:
            bufs = (torch.empty(2 * mv.tokens + 2 * mv.targets, dtype=torch.int64, device=device),
                    torch.empty(2 * mv.targets, dtype=torch.float32, device=device),
                    torch.empty(mv.seqs + 1, dtype=torch.int32, device=device))
            received[(mv.src, mv.index)] = bufs
            for t in bufs:
                ops.append(dist.P2POp(dist.irecv, t, mv.src, group))
    if ops:
        for w in dist.batch_isend_irecv(ops):
            w.wait()
    return received
