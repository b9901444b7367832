"""Peer-mapped buffers: every rank's tensor made addressable from every other rank's kernels.

Each rank exports a CUDA IPC handle of its local tensor (``torch.multiprocessing`` reductions), the
handles are exchanged once with ``all_gather_object``, and each rank opens its peers' handles and
enables peer access from its device. ``ptrs`` is an int64 device tensor of the ``world`` base
addresses (own rank included) that fused kernels index directly. This is plumbing only; the data
moves inside the kernels with plain P2P loads and stores.
"""

from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist


class PeerBuffers:
    def __init__(self, local: torch.Tensor, group=None):
        from torch.multiprocessing.reductions import reduce_tensor

        from ..ops import native

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local = local
        handles: List = [None] * self.world
        dist.all_gather_object(handles, reduce_tensor(local), group=group)
        self.peers: List[torch.Tensor] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.peers.append(local)
                continue
            fn, args = h
            t = fn(*args)
            native().enable_peer_access(t.device.index)
            self.peers.append(t)
        self.ptrs = torch.tensor([t.data_ptr() for t in self.peers], dtype=torch.int64, device=local.device)


def peer_access_available(group=None) -> bool:
    """True when every pair of local ranks' GPUs can reach each other (same node, P2P capable)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_backend(group) != "nccl":
        return False
    dev = torch.cuda.current_device()
    devs: List = [None] * dist.get_world_size(group)
    dist.all_gather_object(devs, dev, group=group)
    ok = all(d == dev or torch.cuda.can_device_access_peer(dev, d) for d in devs)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    return bool(flag.item())
