"""Expert parallelism for the MoE layers: token dispatch and combine over NVLink peer memory.

The reference trainer has no expert parallelism (HF ``Qwen2MoeExperts`` loops over every expert on
every FSDP rank, installed ``transformers/models/qwen2_moe/modeling_qwen2_moe.py:295-331``); its
rollout side gets EP from vLLM (``agent_textworld.py:1926``). Here rank ``d`` of the EP group owns
a contiguous range of experts (``E/W`` each, the first ``E % W`` ranks one more) and runs them on the rows that every rank routed to them:

forward, per MoE layer
  1. per-expert row counts are all-gathered (``W x E`` int32) -- this is also the barrier that
     guarantees every owner has finished with its receive buffer;
  2. dispatch: one ``row_scatter`` kernel per source rank stores each routed token row straight
     into the owner's receive buffer (16-byte P2P stores), at a row the source computes from the
     count matrix alone: the owner's layout is expert-major, sources in rank order inside an
     expert, every expert segment padded to whole 128-row GEMM tiles;
  3. after a 4-byte barrier the owner runs the grouped tcgen05 GEMMs of its local experts; the
     down-projection's epilogue stores every output row straight into the source rank's combine
     buffer (scatter epilogue: GEMM and the return all-to-all are one kernel);
  4. after a second barrier each source weights and sums its rows (fp32) as in the local path.

backward mirrors it: weighted output gradients are dispatched to the same owner rows, the owner
runs dgrad/wgrad of its experts (expert weight gradients therefore only land on the owner; the
optimizer's reduce-scatter sums ranks, so the total is exact), and the gate/up dgrad GEMM scatters
the input-gradient rows back to their sources.

By default every rank keeps the full bf16 parameter copy (the resident-parameter design of
``fsdp.py``) and only the compute is partitioned. With expert-partitioned storage
(``expert_partition(cfg, rank, world)`` + ``build_model(..., experts_last=True)``) a rank holds only
its own experts' weights, gradients and optimizer state, which is what lets models whose experts
dominate the parameter count (30 B-class MoE) fit. Receive buffers are capacity-free: sized for the worst case in which
every source routes all of its rows to one owner (``W * max_tokens * top_k`` rows plus padding).
Pad rows of the receive buffer must read as zero (they enter the weight-gradient contraction), so
the owner clears the rows it used after copying them out; the buffer is zero between uses.

Two other transports share the plan. ``all_to_all`` moves the rows with ``all_to_all_single`` (source-major
blocks, re-laid out expert-major on arrival) around plain grouped GEMMs: it is the library baseline
the fused path is measured against, and works without peer access. ``emulated`` (CPU ranks on gloo)
exchanges (destination, row, data) triples with an all-gather and runs per-expert GEMM loops; it
exists to test the plan and is not fast.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..models import moe as moe_mod

SEG = moe_mod.SEG


def expert_ranges(num_experts: int, world: int):
    """Contiguous expert ranges of the ranks: the first ``E % W`` ranks own one extra expert."""
    base_n, extra = divmod(num_experts, world)
    nloc = [base_n + (1 if r < extra else 0) for r in range(world)]
    return nloc, [sum(nloc[:r]) for r in range(world)]


def expert_partition(cfg, rank: int, world: int):
    """Model config of one rank's expert-partitioned storage (its routed experts only)."""
    import copy

    nloc, lo = expert_ranges(cfg.num_experts, world)
    c = copy.deepcopy(cfg)
    c.local_experts = nloc[rank]
    c.expert_offset = lo[rank]
    return c


class ExpertParallel:
    def __init__(self, cfg, group=None, max_tokens: int = 16384, device: Optional[torch.device] = None,
                 dtype: torch.dtype = torch.bfloat16, transport: Optional[str] = None):
        """``transport``: ``"p2p"`` (fused, NCCL ranks with peer access; the default there),
        ``"all_to_all"`` (two ``all_to_all_single`` per direction around plain grouped GEMMs: the
        library baseline, also usable across nodes) or ``"emulated"`` (gloo/CPU test path)."""
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E = cfg.num_experts
        self.k = cfg.num_experts_per_tok
        self.H = cfg.hidden_size
        self.Im = cfg.moe_intermediate_size
        # contiguous expert ranges; the first E % W ranks own one extra expert (60 experts on 8 ranks:
        # 8,8,8,8,7,7,7,7)
        self.nloc, self.lo_of = expert_ranges(self.E, self.world)
        self.owner = [r for r in range(self.world) for _ in range(self.nloc[r])]
        self.E_loc = self.nloc[self.rank]
        self.lo = self.lo_of[self.rank]
        self.max_tokens = max_tokens
        self.device = device or torch.device("cpu")
        self.dtype = dtype
        self.cap_recv = self.world * max_tokens * self.k + max(self.nloc) * SEG
        self.cap_comb = max_tokens * self.k
        if transport is None:
            from .symmetric import peer_access_available

            if self.device.type == "cuda" and dist.get_backend(group) == "nccl":
                transport = "p2p" if peer_access_available(group) else "all_to_all"
            else:
                transport = "emulated"
        if transport not in ("p2p", "all_to_all", "emulated"):
            raise ValueError(f"unknown expert-parallel transport {transport!r}")
        self.transport = transport
        self.p2p = transport == "p2p"
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        if self.p2p:
            from .symmetric import PeerBuffers

            self.recv = torch.zeros(self.cap_recv, self.H, dtype=dtype, device=self.device)
            self.comb = torch.zeros(self.cap_comb, self.H, dtype=dtype, device=self.device)
            self._recv_peers = PeerBuffers(self.recv, group)
            self._comb_peers = PeerBuffers(self.comb, group)
        self.row_bytes = self.H * torch.empty((), dtype=dtype).element_size()
        # C operand of the scatter-epilogue GEMMs: their rows go to ``row_dst``, this is never written
        self._no_out = torch.empty(1, 8, dtype=dtype, device=self.device)

    # ---------------------------------------------------------------- plan
    def _barrier(self) -> None:
        dist.all_reduce(self._flag, group=self.group)

    def exchange_counts(self, counts: torch.Tensor):
        """Queue the all-gather of every rank's per-expert counts and, on the GPU, their copy into
        pinned host memory; ``wait_counts`` returns the ``W x E`` matrix. Work queued in between runs
        while the host waits."""
        W, E = self.world, self.E
        c_local = counts.to(torch.int64).reshape(1, E)
        c_all = torch.empty(W, E, dtype=torch.int64, device=counts.device)
        if not counts.is_cuda:
            dist.all_gather(list(c_all.chunk(W)), c_local, group=self.group)
            return c_all, None
        dist.all_gather_into_tensor(c_all, c_local, group=self.group)
        if getattr(self, "_pinned", None) is None:
            self._pinned = torch.empty(W, E, dtype=torch.int64, pin_memory=True)
        self._pinned.copy_(c_all, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return self._pinned, ev

    @staticmethod
    def wait_counts(pending):
        host, ev = pending
        if ev is not None:
            ev.synchronize()
        return host.numpy().copy()

    def plan(self, counts: torch.Tensor, C=None) -> Dict:
        """Derive every row's destination (both directions) from the ``W x E`` count matrix ``C``
        (exchanged here when not given). The arithmetic runs vectorised on the host."""
        import numpy as np

        W, E = self.world, self.E
        if C is None:
            C = self.wait_counts(self.exchange_counts(counts))
        # owner-side padded layout of every expert: rows from all sources, padded to whole tiles,
        # segments back to back inside each owner's range
        col = C.sum(0)
        pad = (col + SEG - 1) // SEG * SEG
        start = np.zeros(E, dtype=np.int64)
        owner_rows = np.zeros(W, dtype=np.int64)
        for d in range(W):
            lo, n = self.lo_of[d], self.nloc[d]
            cs = np.cumsum(pad[lo : lo + n])
            start[lo : lo + n] = cs - pad[lo : lo + n]
            owner_rows[d] = cs[-1] if n else 0
        if self.p2p:
            # every rank sees the same C, so an overflow raises on all ranks before any row moves
            if int(C.sum(1).max()) > self.cap_comb:
                raise RuntimeError(f"expert-parallel batch of {int(C.sum(1).max()) // self.k} tokens exceeds "
                                   f"max_tokens={self.max_tokens}")
            if int(owner_rows.max()) > self.cap_recv:
                raise RuntimeError("expert-parallel receive buffer overflow")
        me = self.rank
        # source side: destination row of the first row of each expert segment of this rank
        base = start + C[:me].sum(0)
        # owner side: one block per (local expert, source) with rows, in expert-major then source order
        sl = slice(self.lo, self.lo + self.E_loc)
        sub = C[:, sl].T  # [E_loc, W]
        row0 = start[sl][:, None] + np.cumsum(sub, axis=1) - sub
        slot0 = (np.cumsum(C, axis=1) - C)[:, sl].T  # rows of source s before expert e in its sorted order
        src = np.broadcast_to(np.arange(W), sub.shape)
        keep = sub.reshape(-1) > 0
        blk_row = row0.reshape(-1)[keep].tolist()
        blk_len = sub.reshape(-1)[keep].tolist()
        blk_src = src.reshape(-1)[keep].tolist()
        blk_slot = slot0.reshape(-1)[keep].tolist()
        pads = pad[sl].tolist()
        lay = moe_mod.padded_layout_from_pads(pads, self.device)
        plan = {"C": C, "base": base.tolist(), "lay": lay, "blocks": (blk_row, blk_len, blk_src, blk_slot),
                "n_send": int(C[me].sum()), "R": lay["total"]}
        if self.transport == "all_to_all":
            plan["send_splits"] = [int(C[me, self.lo_of[d] : self.lo_of[d] + self.nloc[d]].sum()) for d in range(W)]
            plan["recv_splits"] = [int(C[s, sl].sum()) for s in range(W)]
            # all_to_all delivers source-major blocks; their rows in the expert-major padded layout
            order = sorted(range(len(blk_len)), key=lambda b: (blk_src[b], blk_row[b]))
            plan["recv_idx"] = self._expand([blk_row[b] for b in order], [blk_len[b] for b in order])
        return plan

    def _expand(self, starts: List[int], lens: List[int]) -> torch.Tensor:
        """Concatenation of ``arange(starts[i], starts[i] + lens[i])`` on the device."""
        dev = self.device
        total = sum(lens)
        if total == 0:
            return torch.zeros(0, dtype=torch.int64, device=dev)
        meta = torch.tensor([lens, starts], dtype=torch.int64).to(dev, non_blocking=True)
        idx = torch.repeat_interleave(torch.arange(len(lens), device=dev), meta[0], output_size=total)
        off = torch.arange(total, device=dev) - torch.repeat_interleave(torch.cumsum(meta[0], 0) - meta[0], meta[0],
                                                                       output_size=total)
        return meta[1][idx] + off

    def _owner_maps(self, plan) -> None:
        """Per local row: source rank and slot in that source's sorted order (pad rows: -1)."""
        blk_row, blk_len, blk_src, blk_slot = plan["blocks"]
        R, dev = plan["R"], self.device
        src = torch.full((R,), -1, dtype=torch.int64, device=dev)
        slot = torch.zeros(R, dtype=torch.int64, device=dev)
        if blk_len:
            total = sum(blk_len)
            meta = torch.tensor([blk_len, blk_row, blk_src, blk_slot], dtype=torch.int64).to(dev, non_blocking=True)
            L = meta[0]
            idx = torch.repeat_interleave(torch.arange(len(blk_len), device=dev), L, output_size=total)
            off = torch.arange(total, device=dev) - torch.repeat_interleave(torch.cumsum(L, 0) - L, L, output_size=total)
            rows = meta[1][idx] + off
            src[rows] = meta[2][idx]
            slot[rows] = meta[3][idx] + off
        plan["row_src"], plan["row_slot"] = src, slot
        if self.p2p:
            addr = self._comb_peers.ptrs[src.clamp(min=0)] + slot * self.row_bytes
            plan["row_dst"] = torch.where(src >= 0, addr, torch.zeros_like(addr))

    def _source_maps(self, plan, e_sorted: torch.Tensor, bounds: List[int]) -> None:
        n = e_sorted.numel()
        base = torch.tensor(plan["base"], dtype=torch.int64, device=e_sorted.device)
        first = torch.tensor(bounds[:-1], dtype=torch.int64, device=e_sorted.device)
        dst_row = torch.arange(n, device=e_sorted.device) - first[e_sorted] + base[e_sorted]
        owner = torch.tensor(self.owner, dtype=torch.int64, device=e_sorted.device)
        dst_rank = owner[e_sorted]
        plan["dst_row"], plan["dst_rank"] = dst_row, dst_rank
        if self.p2p:
            plan["dst_addr"] = self._recv_peers.ptrs[dst_rank] + dst_row * self.row_bytes

    # ---------------------------------------------------------------- transports
    def _send_to_owners(self, src: torch.Tensor, src_row: Optional[torch.Tensor], plan) -> torch.Tensor:
        """Rows of ``src`` (``src_row[i]`` or ``i``) to their owners; returns this rank's received
        rows ``[R, H]`` in the padded expert-major layout (pad rows zero)."""
        R = plan["R"]
        if self.transport == "p2p":
            if plan["n_send"]:
                ops.native().row_scatter(src, src_row, plan["dst_addr"])
            self._barrier()
            out = self.recv[:R].clone()
            self.recv[:R].zero_()
            return out
        rows = src if src_row is None else src.index_select(0, src_row)
        if self.transport == "all_to_all":
            flat = torch.empty(sum(plan["recv_splits"]), self.H, dtype=src.dtype, device=src.device)
            dist.all_to_all_single(flat, rows.contiguous(), plan["recv_splits"], plan["send_splits"], group=self.group)
            out = torch.zeros(R, self.H, dtype=src.dtype, device=src.device)
            out.index_copy_(0, plan["recv_idx"], flat)
            return out
        gathered: List = [None] * self.world
        dist.all_gather_object(gathered, (plan["dst_rank"].cpu(), plan["dst_row"].cpu(), rows.cpu()), group=self.group)
        out = torch.zeros(R, self.H, dtype=src.dtype)
        for dr, drow, data in gathered:
            sel = dr == self.rank
            if bool(sel.any()):
                out[drow[sel]] = data[sel].to(out.dtype)
        return out.to(src.device)

    def _return_rows(self, rows_loc: torch.Tensor, plan) -> torch.Tensor:
        """Owner rows back to their sources' sorted slots (the combine without a scatter epilogue)."""
        if self.transport == "all_to_all":
            send = rows_loc.index_select(0, plan["recv_idx"])
            out = torch.empty(plan["n_send"], self.H, dtype=rows_loc.dtype, device=rows_loc.device)
            dist.all_to_all_single(out, send, plan["send_splits"], plan["recv_splits"], group=self.group)
            return out
        gathered: List = [None] * self.world
        valid = plan["row_src"] >= 0
        dsts = plan["row_src"][valid].cpu()
        slots = plan["row_slot"][valid].cpu()
        dist.all_gather_object(gathered, (dsts, slots, rows_loc[valid].cpu()), group=self.group)
        out = torch.zeros(plan["n_send"], self.H, dtype=rows_loc.dtype)
        for dr, sl, data in gathered:
            sel = dr == self.rank
            if bool(sel.any()):
                out[sl[sel]] = data[sel]
        return out.to(rows_loc.device)

    def _take_combined(self, plan) -> torch.Tensor:
        self._barrier()
        return self.comb[: plan["n_send"]].clone()

    # ---------------------------------------------------------------- expert compute
    def _weights(self, model, layer):
        p = f"model.layers.{layer}.mlp.experts."
        W = model.w(p + "gate_up_proj")
        if W.shape[0] == self.E:
            sl = slice(self.lo, self.lo + self.E_loc)  # every rank keeps the whole expert stack
        else:
            # expert-partitioned storage: the model holds exactly this rank's experts
            cfg = model.cfg
            if W.shape[0] != self.E_loc or cfg.expert_offset != self.lo:
                raise ValueError(f"model holds experts [{cfg.expert_offset}, +{W.shape[0]}) but this rank owns "
                                 f"[{self.lo}, +{self.E_loc})")
            sl = slice(0, self.E_loc)
        Wgu = model.w(p + "gate_up_proj")[sl]
        Wd = model.w(p + "down_proj")[sl]
        gWgu, gWd = model.g(p + "gate_up_proj"), model.g(p + "down_proj")
        return Wgu, Wd, (None if gWgu is None else gWgu[sl]), (None if gWd is None else gWd[sl])

    def forward(self, model, layer: int, h: torch.Tensor, tok: torch.Tensor, e_sorted: torch.Tensor,
                counts: torch.Tensor, bounds: List[int], C=None):
        """Dispatch ``h[tok]`` (sorted by expert), run the local experts, combine. Returns the
        unweighted expert outputs in this rank's sorted order plus the state backward needs. ``C``:
        the exchanged count matrix, when the caller already has it."""
        plan = self.plan(counts, C)
        self._source_maps(plan, e_sorted, bounds)
        self._owner_maps(plan)
        xs_loc = self._send_to_owners(h, tok, plan)
        Wgu, Wd, _, _ = self._weights(model, layer)
        lay = plan["lay"]
        R, H, Im, El = plan["R"], self.H, self.Im, self.E_loc
        if self.p2p:
            gu = torch.empty(R, 2 * Im, dtype=xs_loc.dtype, device=xs_loc.device)
            if R:
                moe_mod._grouped(xs_loc, False, Wgu.reshape(El * 2 * Im, H), False, gu, R, 2 * Im, H, 1, lay, 2 * Im)
            act = ops.swiglu(gu)
            if R:
                moe_mod._grouped(act, False, Wd.reshape(El * H, Im), False, self._no_out, R, H, Im, 1, lay, H,
                                 row_dst=plan["row_dst"])
            ys = self._take_combined(plan)
        elif xs_loc.is_cuda and xs_loc.dtype == torch.bfloat16:
            gu = torch.empty(R, 2 * Im, dtype=xs_loc.dtype, device=xs_loc.device)
            ys_loc = torch.empty(R, H, dtype=xs_loc.dtype, device=xs_loc.device)
            if R:
                moe_mod._grouped(xs_loc, False, Wgu.reshape(El * 2 * Im, H), False, gu, R, 2 * Im, H, 1, lay, 2 * Im)
            act = ops.swiglu(gu)
            if R:
                moe_mod._grouped(act, False, Wd.reshape(El * H, Im), False, ys_loc, R, H, Im, 1, lay, H)
            ys = self._return_rows(ys_loc, plan)
        else:
            bl = [lay["starts"][i] for i in range(El)] + [R]
            ys_loc, gu, act = moe_mod.experts_forward_local(Wgu, Wd, xs_loc, bl)
            ys = self._return_rows(ys_loc, plan)
        state = {"plan": plan, "xs": xs_loc, "gu": gu, "act": act}
        return ys, state

    def backward(self, model, layer: int, dys: torch.Tensor, state) -> torch.Tensor:
        """``dys``: weighted output gradients in this rank's sorted order. Returns the input
        gradients of the dispatched rows in the same order."""
        plan = state["plan"]
        dys_loc = self._send_to_owners(dys, None, plan)
        Wgu, Wd, gWgu, gWd = self._weights(model, layer)
        lay = plan["lay"]
        R, H, Im, El = plan["R"], self.H, self.Im, self.E_loc
        xs, gu, act = state["xs"], state["gu"], state["act"]
        if dys_loc.is_cuda and dys_loc.dtype == torch.bfloat16:
            dact = torch.empty(R, Im, dtype=dys.dtype, device=dys.device)
            if R:
                moe_mod._grouped(dys_loc, False, Wd.reshape(El * H, Im), True, dact, R, Im, H, 1, lay, H)
                if gWd is not None:
                    moe_mod._grouped(dys_loc, True, act, True, gWd.reshape(El * H, Im), H, Im, R, 2, lay, 0, H,
                                     beta=1.0)
            dgu = ops.swiglu_backward(dact, gu)
            del dact
            p2p = self.transport == "p2p"
            dxs_loc = None if p2p else torch.empty(R, H, dtype=dys.dtype, device=dys.device)
            if R:
                moe_mod._grouped(dgu, False, Wgu.reshape(El * 2 * Im, H), True, self._no_out if p2p else dxs_loc, R, H,
                                 2 * Im, 1, lay, 2 * Im, row_dst=plan["row_dst"] if p2p else None)
                if gWgu is not None:
                    moe_mod._grouped(dgu, True, xs, True, gWgu.reshape(El * 2 * Im, H), 2 * Im, H, R, 2, lay, 0,
                                     2 * Im, beta=1.0)
            return self._take_combined(plan) if p2p else self._return_rows(dxs_loc, plan)
        bl = [lay["starts"][i] for i in range(El)] + [R]
        dxs_loc = moe_mod.experts_backward_local(Wgu, Wd, gWgu, gWd, dys_loc, xs, gu, act, bl)
        return self._return_rows(dxs_loc, plan)
