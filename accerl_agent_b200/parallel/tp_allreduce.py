"""All-reduce of tensor-parallel partial sums over NVLink peer memory (one kernel per call).

Each rank owns a symmetric bf16 buffer with two slots and a small int32 flag array, both mapped into
every other rank of the group (``PeerBuffers``). A row-parallel GEMM writes its partial straight into
the slot of the current call (``slot(k)``, alternating with the call index ``k`` inside a forward);
``reduce`` then launches ``tp_allreduce`` (``csrc/collectives.cu``): it publishes a per-call epoch to
every peer, waits (bounded) for theirs, and sums all ranks' partials plus the residual in rank order,
so every rank gets bit-identical results. The epoch counter lives on the device, so the calls can be
captured in CUDA graphs and replayed. Ranks must issue the same calls in the same order.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .symmetric import PeerBuffers


class TPAllReduce:
    def __init__(self, group, device: torch.device, max_elems: int, dtype=torch.bfloat16):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.max_elems = int(max_elems)
        self.buf = torch.zeros(2 * self.max_elems, dtype=dtype, device=device)
        self.flags = torch.zeros(2 * self.world, dtype=torch.int32, device=device)
        self.ctr = torch.zeros(2, dtype=torch.int32, device=device)
        self.status = ops.status_tensor(device)
        self._data = PeerBuffers(self.buf, group)
        self._flags = PeerBuffers(self.flags, group)
        # every rank's buffers exist before any rank signals into them
        dist.barrier(group=group)

    def slot(self, k: int, rows: int, cols: int) -> torch.Tensor:
        """The partial-sum buffer of call ``k`` as a ``[rows, cols]`` view."""
        n = rows * cols
        if n > self.max_elems:
            raise ValueError(f"tensor-parallel all-reduce of {n} elements exceeds the buffer ({self.max_elems})")
        s = (k & 1) * self.max_elems
        return self.buf[s : s + n].view(rows, cols)

    def reduce(self, k: int, partial: torch.Tensor, residual=None, out=None) -> torch.Tensor:
        """``out = residual + sum over ranks of partial``; ``partial`` must be ``slot(k, ...)``."""
        out = out if out is not None else torch.empty_like(partial)
        ops.native().tp_allreduce(self._data.ptrs, self._flags.ptrs, self.rank, k & 1, self.max_elems,
                                  partial.numel(), residual, out, self.ctr, self.status)
        return out

    def check(self) -> None:
        st = int(self.status[0].item())
        if st != 0:
            raise RuntimeError(f"tensor-parallel all-reduce timed out waiting for a peer (status {st})")
