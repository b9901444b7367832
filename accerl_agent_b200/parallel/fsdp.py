"""FSDP-style sharded optimizer state over flat parameter buffers.

The reference shards every decoder layer with FSDP2 ``fully_shard`` and re-gathers parameters before
each forward and backward, reduce-scattering bf16 gradients after every micro-batch
(agent_textworld.py:474-496). On B200 (180 GB per GPU) the compute copy of the parameters of every
benchmarked model fits on each rank, so this runtime keeps it resident and shards only what is big and
fp32: master weights, Adam moments and the reduced gradient. Per optimizer step:

1. gradients accumulate locally in one flat fp32 buffer over all micro-batches (wgrad GEMMs add in
   their epilogue);
2. one reduce-scatter (SUM) gives every rank the gradient of its shard;
3. the global gradient norm is one 8-byte all-reduce of per-shard sums of squares;
4. the fused clip + AdamW kernel updates the fp32 shard and writes the bf16 compute shard;
5. one in-place all-gather refreshes the full bf16 copy on every rank.

Micro-batches therefore run with no parameter traffic at all. The loss is scaled by
``1 / global_valid_tokens`` and gradients are summed over ranks, which equals the reference's
``world / global_tokens`` pre-scale followed by FSDP's ``1 / world`` gradient divide.

On a single rank the shard is the whole trainable segment and no collective is issued. CPU ranks use
gloo (reduce-scatter is emulated with an all-reduce there).

With expert-partitioned storage (``ParamLayout.build(..., experts_last=True)``) only the replicated
prefix of the trainable segment is sharded and reduced; each rank's own routed experts (the rest of the
segment) keep their full fp32 state on that rank and are updated locally (their gradients only ever
land on the owner). The global gradient norm sums both parts before its all-reduce.

With NCCL ranks on one node (``fused_collectives``, the default when every GPU pair has peer access)
steps 2-5 run as two kernels over NVLink peer memory instead (``csrc/collectives.cu``): a
reduce-scatter that reads the shard range of every peer's fp32 gradient buffer and accumulates the
squared norm in the same pass, then clip + AdamW whose epilogue stores the new bf16 shard into every
peer's parameter buffer (the all-gather). Only the 8-byte norm all-reduce and a 4-byte barrier stay
on NCCL.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


def dist_ready() -> bool:
    return dist.is_available() and dist.is_initialized()


class ShardedAdamW:
    def __init__(self, model, lr: float, weight_decay: float = 0.0, betas=(0.9, 0.999), eps: float = 1e-8,
                 max_grad_norm: float = 1.0, group=None):
        self.model = model
        self.group = group
        self.world = dist.get_world_size(group) if dist_ready() else 1
        self.rank = dist.get_rank(group) if dist_ready() else 0
        n = model.layout.replicated_numel
        if n % max(self.world, 1):
            raise ValueError("trainable segment must be padded to a multiple of the world size")
        self.shard_numel = n // self.world
        self.local_lo, self.local_hi = n, model.layout.trainable_numel  # rank-local experts (may be empty)
        self.lr = lr
        self.weight_decay = weight_decay
        self.betas = betas
        self.eps = eps
        self.max_grad_norm = max_grad_norm
        self.step_count = 0
        lo = self.rank * self.shard_numel
        self.param_shard = model.params[lo : lo + self.shard_numel]
        self.master = self.param_shard.detach().float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.has_local = self.local_hi > self.local_lo
        if self.has_local:
            self.local_params = model.params[self.local_lo : self.local_hi]
            self.local_master = self.local_params.detach().float().clone()
            self.local_m = torch.zeros_like(self.local_master)
            self.local_v = torch.zeros_like(self.local_master)
            self.local_grads = model.grads[self.local_lo : self.local_hi]
        if self.world == 1:
            self.grad_shard = model.grads[: self.shard_numel]
        else:
            self.grad_shard = torch.zeros(self.shard_numel, dtype=torch.float32, device=model.params.device)
        self._sumsq = torch.zeros(1, dtype=torch.float64, device=model.params.device)
        self.backend = dist.get_backend(group) if dist_ready() else "none"
        self.fused = False
        if self.world > 1 and self.backend == "nccl" and os.environ.get("ACCERL_FUSED_COLLECTIVES", "1") != "0":
            from .symmetric import PeerBuffers, peer_access_available

            if peer_access_available(group):
                self._grad_peers = PeerBuffers(model.grads, group)
                self._param_peers = PeerBuffers(model.params, group)
                self._barrier_flag = torch.zeros(1, dtype=torch.int32, device=model.params.device)
                self.fused = True

    def refresh_master_from_params(self) -> None:
        """Re-seed fp32 master weights after parameters were overwritten (e.g. checkpoint load)."""
        self.master.copy_(self.param_shard.float())
        if self.has_local:
            self.local_master.copy_(self.local_params.float())

    def reduce_gradients(self) -> None:
        if self.world == 1:
            return
        full = self.model.grads[: self.local_lo]
        if self.backend == "nccl":
            dist.reduce_scatter_tensor(self.grad_shard, full, op=dist.ReduceOp.SUM, group=self.group)
        else:
            dist.all_reduce(full, op=dist.ReduceOp.SUM, group=self.group)
            lo = self.rank * self.shard_numel
            self.grad_shard.copy_(full[lo : lo + self.shard_numel])
        full.zero_()

    def global_grad_sumsq(self) -> torch.Tensor:
        self._sumsq.zero_()
        ops.grad_sumsq(self.grad_shard, self._sumsq)
        if self.has_local:
            ops.grad_sumsq(self.local_grads, self._sumsq)
        if self.world > 1:
            dist.all_reduce(self._sumsq, op=dist.ReduceOp.SUM, group=self.group)
        return self._sumsq

    def step(self, lr: Optional[float] = None, timer=None) -> torch.Tensor:
        """Reduce, clip (global norm ``max_grad_norm``), update and re-gather. Returns the float64
        sum of squared gradients (a device tensor; no host sync). ``timer`` (a
        ``utils.timing.PhaseTimer``) marks the end of each phase."""
        if lr is not None:
            self.lr = lr
        if self.fused:
            return self._fused_step(timer)
        mark = timer.mark if timer is not None else (lambda name: None)
        self.reduce_gradients()
        mark("reduce_scatter")
        sumsq = self.global_grad_sumsq()
        mark("norm_allreduce")
        self.step_count += 1
        ops.adamw_step(self.master, self.exp_avg, self.exp_avg_sq, self.grad_shard, self.param_shard, sumsq,
                       self.lr, self.betas[0], self.betas[1], self.eps, self.weight_decay, self.max_grad_norm,
                       self.step_count)
        self._local_step(sumsq)
        mark("adamw")
        self.all_gather_params()
        mark("all_gather")
        return sumsq

    def _local_step(self, sumsq: torch.Tensor) -> None:
        """Clip + AdamW of this rank's own experts (full state here, no collective)."""
        if not self.has_local:
            return
        ops.adamw_step(self.local_master, self.local_m, self.local_v, self.local_grads, self.local_params, sumsq,
                       self.lr, self.betas[0], self.betas[1], self.eps, self.weight_decay, self.max_grad_norm,
                       self.step_count)  # (the kernel zeroes the gradients it consumed)

    def _fused_step(self, timer=None) -> torch.Tensor:
        import math

        mark = timer.mark if timer is not None else (lambda name: None)
        native = ops.native()
        self._sumsq.zero_()
        # every peer has finished accumulating its gradients before anyone reads them
        dist.all_reduce(self._barrier_flag, group=self.group)
        mark("barrier_grads_ready")
        native.rs_sumsq(self._grad_peers.ptrs, self.rank, self.shard_numel, self.grad_shard, self._sumsq)
        if self.has_local:
            ops.grad_sumsq(self.local_grads, self._sumsq)
        mark("rs_sumsq")
        # the norm all-reduce also guarantees every peer has finished reading this rank's gradients
        dist.all_reduce(self._sumsq, op=dist.ReduceOp.SUM, group=self.group)
        mark("norm_allreduce")
        self.step_count += 1
        self._local_step(self._sumsq)
        self.model.grads.zero_()
        mark("grad_zero")
        b1, b2 = self.betas
        native.adamw_push(self.master, self.exp_avg, self.exp_avg_sq, self.grad_shard, self._param_peers.ptrs,
                          self.rank, self._sumsq, self.lr, b1, b2, self.eps, self.weight_decay, self.max_grad_norm,
                          1.0 - b1 ** self.step_count, math.sqrt(1.0 - b2 ** self.step_count))
        mark("adamw_push")
        # every peer's parameter pushes into this rank's buffer land before the next forward
        dist.all_reduce(self._barrier_flag, group=self.group)
        mark("barrier_params_ready")
        return self._sumsq

    def all_gather_params(self) -> None:
        if self.world == 1:
            return
        full = self.model.params[: self.local_lo]
        if self.backend == "nccl":
            dist.all_gather_into_tensor(full, self.param_shard, group=self.group)
        else:
            parts = list(full.chunk(self.world))
            local = self.param_shard.clone()
            dist.all_gather(parts, local, group=self.group)

    def state_dict(self):
        st = {"step": self.step_count, "master": self.master, "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq}
        if self.has_local:
            st.update(local_master=self.local_master, local_exp_avg=self.local_m, local_exp_avg_sq=self.local_v)
        return st

    def load_state_dict(self, state):
        self.step_count = int(state["step"])
        self.master.copy_(state["master"])
        self.exp_avg.copy_(state["exp_avg"])
        self.exp_avg_sq.copy_(state["exp_avg_sq"])
        self.param_shard.copy_(self.master.to(self.param_shard.dtype))
        if self.has_local:
            self.local_master.copy_(state["local_master"])
            self.local_m.copy_(state["local_exp_avg"])
            self.local_v.copy_(state["local_exp_avg_sq"])
            self.local_params.copy_(self.local_master.to(self.local_params.dtype))
        self.all_gather_params()
