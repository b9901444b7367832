"""Layer-sharded parameters: parameters, gradients and optimizer state all sharded (FSDP full sharding).

The reference wraps every decoder layer in FSDP2 ``fully_shard`` (``agent_textworld.py:474-476``): a
layer's parameters are all-gathered before its forward and again before its backward, and its
gradients are reduce-scattered after every micro-batch. ``parallel/fsdp.py`` keeps the bf16 compute
copy and a full fp32 gradient buffer on every rank instead (6 N bytes per rank plus 12 N / W of
optimizer state), which caps dense models near 25 B parameters on 180 GB. With ``--shard-params``
this module shards everything:

* the full flat layout (``ParamLayout``) is cut into units -- the embedding, one unit per decoder
  layer, and [final norm | LM head] -- each a contiguous range of the layout, padded to a multiple
  of ``world * 64`` elements and split evenly over the ranks. A rank stores its shard of every unit:
  bf16 compute copy, fp32 gradient, fp32 master and both Adam moments (18 N / W bytes);
* the embedding and head units are all-gathered once after each optimizer step and stay resident
  (both are used at both ends of every micro-batch);
* decoder layer l is all-gathered into one of two ping-pong buffers on a communication stream while
  layer l - 1 runs its forward (or layer l + 1 its backward), so the gather overlaps the compute;
* after layer l's backward its fp32 gradient unit is reduce-scattered on the communication stream
  and added to the rank's gradient shard while layer l - 1's backward runs;
* the optimizer (global-norm clip + AdamW) updates the shards in place; nothing is gathered after
  the step (the next forward gathers what it needs).

The model object binds its parameter (and gradient) views to whichever buffer holds the unit at the
moment, so the layer code is the same as with resident parameters. On CPU ranks (gloo) the
collectives run synchronously (reduce-scatter as an all-reduce).

Supported: every ``--train-mode`` (frozen units are gathered for the forward and the backward that
passes through them but get no gradient or optimizer state), dense and MoE models without expert
parallelism.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional

import torch
import torch.distributed as dist

from .. import ops
from ..models.transformer import ALIGN, CausalLM, ParamLayout


@dataclass
class Unit:
    name: str
    names: List[str]
    lo: int  # first element in the full layout
    span: int  # elements of the full layout it covers
    numel: int  # padded to a multiple of world * ALIGN
    shard: int  # numel // world
    base: int  # start of this rank's shard in the local buffers
    layer: int  # decoder layer, -1 for the embedding and head units
    trainable: bool = True

    def pinned(self) -> bool:
        return self.layer < 0


def _unit_key(name: str) -> str:
    if name.startswith("model.layers."):
        return "layer." + name.split(".")[2]
    return "embed" if name == "model.embed_tokens.weight" else "head"


def build_units(layout: ParamLayout, world: int, trainable: Optional[Dict[str, bool]] = None) -> List[Unit]:
    """The units of ``layout`` (laid out in parameter order, as ``ParamLayout.build(cfg, "full")``
    does), each a contiguous range of it. ``trainable`` (name -> flag, default all) splits a unit
    where the flag changes (the final norm and the LM head of the head unit under ``--train-mode
    lm_head``); a decoder layer is trained whole or not at all. Local storage holds the trainable
    units' shards first, so the optimizer works on one prefix."""
    slots = sorted(layout.slots.values(), key=lambda s: s.offset)
    flag = (lambda n: True) if trainable is None else (lambda n: bool(trainable[n]))
    groups: List[List] = []
    seen: set = set()
    for s in slots:
        k = _unit_key(s.name)
        if groups and _unit_key(groups[-1][0].name) == k and flag(groups[-1][0].name) == flag(s.name):
            groups[-1].append(s)
            continue
        if k in seen and _unit_key(groups[-1][0].name) != k:
            raise ValueError(f"parameters of unit {k} are not contiguous in the layout")
        if k in seen and k.startswith("layer."):
            raise ValueError(f"decoder layer {k} is partly trainable")
        seen.add(k)
        groups.append([s])
    q = ALIGN * max(world, 1)
    units: List[Unit] = []
    for ss in groups:
        k = _unit_key(ss[0].name)
        lo = ss[0].offset
        hi = ss[-1].offset + (ss[-1].numel + ALIGN - 1) // ALIGN * ALIGN
        numel = (hi - lo + q - 1) // q * q
        name = k if sum(_unit_key(g[0].name) == k for g in groups) == 1 else f"{k}.{ss[0].name}"
        units.append(Unit(name, [s.name for s in ss], lo, hi - lo, numel, numel // max(world, 1), 0,
                          int(k.split(".")[1]) if k.startswith("layer.") else -1, flag(ss[0].name)))
    base = 0
    for u in sorted(units, key=lambda u: not u.trainable):  # stable: trainable units first
        u.base = base
        base += u.shard
    return units


def shard_pieces(units: List[Unit], world: int):
    """Where every element of the full layout lives: ``(start, end, rank, local_start)`` ranges of
    the full layout, sorted by start."""
    out = []
    for u in units:
        for r in range(world):
            a = u.lo + r * u.shard
            b = min(u.lo + (r + 1) * u.shard, u.lo + u.span)
            if a < b:
                out.append((a, b, r, u.base))
    return out


class LayerShardedParams:
    """Sharded storage of one rank plus the gather / reduce-scatter schedule around the layers."""

    def __init__(self, cfg, device: torch.device, dtype: torch.dtype, group=None, train_mode: str = "full"):
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.device = device
        self.dtype = dtype
        self.layout = sharded_layout(cfg, train_mode)
        self.units = build_units(self.layout, self.world, {n: s.trainable for n, s in self.layout.slots.items()})
        self.layer_unit = {u.layer: u for u in self.units if not u.pinned()}
        self.n_trainable = sum(u.shard for u in self.units if u.trainable)  # the optimizer's prefix
        if self.n_trainable == 0:
            raise RuntimeError(f"No trainable parameters found for mode: {train_mode}")
        n_local = sum(u.shard for u in self.units)
        self.local = torch.zeros(n_local, dtype=dtype, device=device)
        self.local_grads = torch.zeros(n_local, dtype=torch.float32, device=device)
        big = max((u.numel for u in self.units if not u.pinned()), default=ALIGN)
        self.pbuf = [torch.zeros(big, dtype=dtype, device=device) for _ in range(2)]
        self.gbuf = [torch.zeros(big, dtype=torch.float32, device=device) for _ in range(2)]
        self.gtmp = [torch.zeros(big // max(self.world, 1), dtype=torch.float32, device=device) for _ in range(2)]
        self.pin_p = {u.name: torch.zeros(u.numel, dtype=dtype, device=device) for u in self.units if u.pinned()}
        self.pin_g = {u.name: torch.zeros(u.numel, dtype=torch.float32, device=device)
                      for u in self.units if u.pinned()}
        self.pin_tmp = {u.name: torch.zeros(u.shard, dtype=torch.float32, device=device)
                        for u in self.units if u.pinned()}
        self.cuda = device.type == "cuda"
        self.nccl = dist.is_initialized() and dist.get_backend(group) == "nccl"
        self.comm = torch.cuda.Stream(device) if self.cuda else None
        self.resident: List[Optional[int]] = [None, None]  # layer held by each ping-pong buffer
        # per ping-pong buffer: how the compute stream waits for its pending gather (None: nothing
        # pending), and the event of the reduce-scatter that last read its gradient buffer
        self._gather_wait: List[Optional[Callable[[], None]]] = [None, None]
        self._gather_ev = [torch.cuda.Event() for _ in range(2)] if self.cuda else [None, None]
        self._rs_done = [torch.cuda.Event() for _ in range(2)] if self.cuda else [None, None]
        self._rs_pending = [False, False]
        self.params_dirty = True  # shards changed since the pinned units were gathered
        self.model = CausalLM.without_buffers(cfg, self.layout)
        self.model.units = self
        trained = [u.layer for u in self.units if u.trainable and not u.pinned()]
        self.model.first_trainable_layer = min(trained) if trained else cfg.num_hidden_layers

    # ---------------------------------------------------------------- views
    def _bind(self, u: Unit, pbuf: torch.Tensor, gbuf: Optional[torch.Tensor]) -> None:
        m = self.model
        for name in u.names:
            s = self.layout.slots[name]
            o = s.offset - u.lo
            m._views[name] = pbuf[o : o + s.numel].view(s.shape)
            if gbuf is not None and u.trainable:
                m._gviews[name] = gbuf[o : o + s.numel].view(s.shape)

    def shard_of(self, u: Unit) -> torch.Tensor:
        return self.local[u.base : u.base + u.shard]

    # ---------------------------------------------------------------- collectives
    def _gather(self, u: Unit, out: torch.Tensor, async_op: bool):
        src = self.shard_of(u)
        full = out[: u.numel]
        if self.world == 1:
            full.copy_(src)
            return None
        if self.nccl:
            return dist.all_gather_into_tensor(full, src, group=self.group, async_op=async_op)
        dist.all_gather(list(full.chunk(self.world)), src.clone(), group=self.group)
        return None

    def _reduce_scatter_add(self, u: Unit, grad_full: torch.Tensor, tmp: torch.Tensor) -> None:
        """This rank's shard of the sum over ranks of ``grad_full`` added into its gradient shard."""
        g = grad_full[: u.numel]
        dst = self.local_grads[u.base : u.base + u.shard]
        if self.world == 1:
            dst.add_(g)
            return
        if self.nccl:
            dist.reduce_scatter_tensor(tmp[: u.shard], g, op=dist.ReduceOp.SUM, group=self.group)
            dst.add_(tmp[: u.shard])
            return
        dist.all_reduce(g, op=dist.ReduceOp.SUM, group=self.group)
        dst.add_(g[self.rank * u.shard : (self.rank + 1) * u.shard])

    def gather_pinned(self) -> None:
        for u in self.units:
            if u.pinned():
                self._gather(u, self.pin_p[u.name], async_op=False)
                self._bind(u, self.pin_p[u.name], self.pin_g[u.name])
        self.resident = [None, None]
        self.params_dirty = False

    def _issue_layer_gather(self, layer: int) -> None:
        """Gather ``layer`` into its ping-pong buffer on the communication stream, after the compute
        stream's work so far (the previous user of that buffer) has run."""
        b = layer % 2
        if self.resident[b] == layer:
            return
        u = self.layer_unit[layer]
        if self.cuda:
            self.comm.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                work = self._gather(u, self.pbuf[b], async_op=True)
                if work is not None:
                    self._gather_wait[b] = work.wait  # waits on the current (compute) stream
                else:  # a single rank: the copy ran on the comm stream
                    ev = self._gather_ev[b]
                    ev.record(self.comm)
                    self._gather_wait[b] = lambda ev=ev: torch.cuda.current_stream(self.device).wait_event(ev)
        else:
            self._gather(u, self.pbuf[b], async_op=False)
        self.resident[b] = layer

    def _await_layer(self, layer: int) -> None:
        b = layer % 2
        if self.resident[b] != layer:
            self._issue_layer_gather(layer)
        wait = self._gather_wait[b]
        if wait is not None:
            wait()
            self._gather_wait[b] = None

    # ---------------------------------------------------------------- hooks called by the model
    def begin_forward(self) -> None:
        if self.params_dirty:
            self.gather_pinned()

    def before_forward(self, layer: int) -> None:
        self._await_layer(layer)
        self._bind(self.layer_unit[layer], self.pbuf[layer % 2], None)
        if layer + 1 in self.layer_unit:
            self._issue_layer_gather(layer + 1)

    def begin_backward(self) -> None:
        for u in self.units:
            if u.pinned() and u.trainable:
                self.pin_g[u.name].zero_()

    def before_backward(self, layer: int) -> None:
        b = layer % 2
        self._await_layer(layer)
        if self.cuda and self._rs_pending[b]:
            torch.cuda.current_stream(self.device).wait_event(self._rs_done[b])
        u = self.layer_unit[layer]
        if u.trainable:
            self.gbuf[b][: u.numel].zero_()
        self._bind(u, self.pbuf[b], self.gbuf[b])
        if layer - 1 in self.layer_unit and layer - 1 >= self.model.first_trainable_layer:
            self._issue_layer_gather(layer - 1)  # the backward stops below the first trained layer

    def after_backward(self, layer: int) -> None:
        b = layer % 2
        u = self.layer_unit[layer]
        if not u.trainable:
            return
        if self.cuda:
            self.comm.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                self._reduce_scatter_add(u, self.gbuf[b], self.gtmp[b])
                self._rs_done[b].record(self.comm)
                self._rs_pending[b] = True
        else:
            self._reduce_scatter_add(u, self.gbuf[b], self.gtmp[b])
        for name in u.names:
            self.model._gviews.pop(name, None)

    def end_backward(self) -> None:
        if self.cuda:
            self.comm.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                for u in self.units:
                    if u.pinned() and u.trainable:
                        self._reduce_scatter_add(u, self.pin_g[u.name], self.pin_tmp[u.name])
            torch.cuda.current_stream(self.device).wait_stream(self.comm)
        else:
            for u in self.units:
                if u.pinned() and u.trainable:
                    self._reduce_scatter_add(u, self.pin_g[u.name], self.pin_tmp[u.name])

    def invalidate(self) -> None:
        """The shards changed (optimizer step, checkpoint load): every gathered copy is stale."""
        self.params_dirty = True
        self.resident = [None, None]

    # ---------------------------------------------------------------- whole-model passes
    def for_each_unit_gathered(self, fn, write_back: bool = False) -> None:
        """``fn(unit, views)`` for every unit in order with the unit gathered into a scratch buffer
        (``views``: name -> tensor). A collective: every rank calls it. With ``write_back`` the
        rank's shard is taken from the buffer afterwards (initialisation, checkpoint load)."""
        for u in self.units:
            buf = torch.zeros(u.numel, dtype=self.dtype, device=self.device)
            if not write_back:
                self._gather(u, buf, async_op=False)
            views = {}
            for name in u.names:
                s = self.layout.slots[name]
                o = s.offset - u.lo
                views[name] = buf[o : o + s.numel].view(s.shape)
            fn(u, views)
            if write_back:
                self.shard_of(u).copy_(buf[self.rank * u.shard : (self.rank + 1) * u.shard])
        if write_back:
            self.invalidate()

    def init_weights(self, seed: int = 0, std: float = 0.02) -> None:
        """The values ``CausalLM.init_weights`` gives the unsharded model, this rank's shards of them."""
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        order = [n for u in self.units for n in u.names]
        if order != list(self.layout.order):
            raise RuntimeError("unit order differs from the parameter order")

        def fill(u, views):
            for name in u.names:
                self.model._init_param(name, views[name], gen, std)

        with torch.no_grad():
            self.for_each_unit_gathered(fill, write_back=True)

    def full_numel(self) -> int:
        return self.layout.total_numel


class ShardedParamAdamW:
    """Global-norm clip + AdamW on the rank's shards (fp32 master and moments); the bf16 shard is
    written by the same kernel. Same interface as ``ShardedAdamW``."""

    def __init__(self, sharding: LayerShardedParams, lr: float, weight_decay: float = 0.0, betas=(0.9, 0.999),
                 eps: float = 1e-8, max_grad_norm: float = 1.0):
        self.sharding = sharding
        self.group = sharding.group
        self.world = sharding.world
        self.lr = lr
        self.weight_decay = weight_decay
        self.betas = betas
        self.eps = eps
        self.max_grad_norm = max_grad_norm
        self.step_count = 0
        self.params = sharding.local[: sharding.n_trainable]
        self.grads = sharding.local_grads[: sharding.n_trainable]
        self.master = self.params.detach().float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self._sumsq = torch.zeros(1, dtype=torch.float64, device=sharding.device)

    def refresh_master_from_params(self) -> None:
        self.master.copy_(self.params.float())

    def step(self, lr: Optional[float] = None, timer=None) -> torch.Tensor:
        if lr is not None:
            self.lr = lr
        mark = timer.mark if timer is not None else (lambda name: None)
        sh = self.sharding
        self._sumsq.zero_()
        ops.grad_sumsq(self.grads, self._sumsq)
        if self.world > 1:
            dist.all_reduce(self._sumsq, op=dist.ReduceOp.SUM, group=self.group)
        mark("norm_allreduce")
        self.step_count += 1
        ops.adamw_step(self.master, self.exp_avg, self.exp_avg_sq, self.grads, self.params, self._sumsq, self.lr,
                       self.betas[0], self.betas[1], self.eps, self.weight_decay, self.max_grad_norm,
                       self.step_count)  # (the kernel zeroes the gradient shard)
        sh.invalidate()
        mark("adamw")
        return self._sumsq

    def state_dict(self):
        return {"step": self.step_count, "master": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq}

    def load_state_dict(self, state):
        self.step_count = int(state["step"])
        self.master.copy_(state["master"])
        self.exp_avg.copy_(state["exp_avg"])
        self.exp_avg_sq.copy_(state["exp_avg_sq"])
        self.params.copy_(self.master.to(self.params.dtype))
        self.sharding.invalidate()


def sharded_layout(cfg, train_mode: str = "full") -> ParamLayout:
    """The full layout in parameter order (every parameter at its ``"full"``-mode offset) with the
    trainable flags of ``train_mode``; trainers and engines build the same units from it."""
    layout = ParamLayout.build(cfg, "full", pad_to=1)
    flags = ParamLayout.build(cfg, train_mode, pad_to=1).slots
    for name, s in layout.slots.items():
        s.trainable = flags[name].trainable
    return layout


def bytes_per_rank(num_params: int, world: int, sharded: bool) -> float:
    """Bytes of parameter, gradient and optimizer state per rank (bf16 compute copy, fp32 gradient,
    fp32 master + two moments), without activations or gather buffers."""
    if sharded:
        return 18.0 * num_params / world
    return 6.0 * num_params + 12.0 * num_params / world


__all__ = ["Unit", "build_units", "shard_pieces", "sharded_layout", "LayerShardedParams", "ShardedParamAdamW",
           "bytes_per_rank"]
