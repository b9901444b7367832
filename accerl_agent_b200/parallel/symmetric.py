"""Peer-mapped buffers: every rank's tensor made addressable from every other rank's kernels.

Each rank exports a CUDA IPC handle of the allocation that holds its local tensor (plus the tensor's
byte offset in it); the handles are exchanged once with ``all_gather_object`` and every rank opens
its peers' handles on its OWN current device with lazy peer access, so the mappings live in the
context that the fused kernels run in. Before any kernel dereferences a mapping, each rank reads the
first 16 bytes of every peer buffer through it with a synchronous host copy and compares them with
what the owner reported: a bad mapping fails here as a host error instead of a device fault.

``ptrs`` is an int64 device tensor of the ``world`` base addresses (own rank included) that fused
kernels index directly. This is plumbing only; the data moves inside the kernels with plain P2P loads
and stores.
"""

from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist


def _ext():
    from ..ops._ext import native

    return native()


class PeerBuffers:
    def __init__(self, local: torch.Tensor, group=None):
        ext = _ext()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local = local
        if not local.is_contiguous():
            raise ValueError("PeerBuffers needs a contiguous tensor")
        dev = local.device.index
        if torch.cuda.current_device() != dev:
            raise RuntimeError(f"current device {torch.cuda.current_device()} is not the buffer's device {dev}")
        rc, handle, offset = ext.ipc_export(local)
        if rc != 0:
            raise RuntimeError(f"cudaIpcGetMemHandle failed with code {rc}")
        nprobe = min(16, local.numel() * local.element_size())
        torch.cuda.synchronize()
        probe = bytes(local.view(-1).view(torch.uint8)[:nprobe].cpu().numpy().tobytes()) if nprobe else b""
        infos: List = [None] * self.world
        dist.all_gather_object(infos, (dev, handle, int(offset), probe), group=group)
        self._opened: List[int] = []
        addrs: List[int] = []
        for r, (pdev, h, off, pr) in enumerate(infos):
            if r == self.rank:
                addrs.append(local.data_ptr())
                continue
            from ..ops import native as checked_native

            checked_native().enable_peer_access(pdev)
            rc, base = ext.ipc_open(h)
            if rc != 0:
                raise RuntimeError(f"cudaIpcOpenMemHandle of rank {r}'s buffer failed with code {rc}")
            self._opened.append(base)
            addr = base + off
            if pr:
                rc, got = ext.peer_read(addr, len(pr))
                if rc != 0 or bytes(got) != pr:
                    raise RuntimeError(f"peer mapping of rank {r}'s buffer is not readable or holds other data")
            addrs.append(addr)
        self.addrs = addrs
        self.ptrs = torch.tensor(addrs, dtype=torch.int64, device=local.device)

    def close(self) -> None:
        """Unmap the peers' buffers. Only call when no kernel that uses ``ptrs`` is in flight."""
        ext = _ext()
        for base in self._opened:
            ext.ipc_close(base)
        self._opened = []


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
