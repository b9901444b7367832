"""Device timing helpers: CUDA events on the launching stream, warm-up, L2 flush, max over ranks."""

from __future__ import annotations

import statistics
from typing import Callable, List, Optional

import torch

L2_FLUSH_BYTES = 256 * 1024 * 1024  # > 126 MB L2 of B200

_flush_buf: Optional[torch.Tensor] = None


def flush_l2(device=None) -> None:
    """Overwrite a buffer larger than L2 so the next kernel starts cold."""
    global _flush_buf
    if _flush_buf is None or (device is not None and _flush_buf.device != torch.device(device)):
        _flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=device or "cuda")
    _flush_buf.fill_(1.0)


def time_cuda(fn: Callable[[], None], iters: int = 20, warmup: int = 3, flush: bool = True) -> List[float]:
    """Per-iteration device time in milliseconds (CUDA events around each call)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    return times


def median_ms(fn: Callable[[], None], iters: int = 20, warmup: int = 3, flush: bool = True) -> float:
    return statistics.median(time_cuda(fn, iters, warmup, flush))


def max_over_ranks(value: float) -> float:
    """Max of a per-rank scalar over the default process group (identity without one)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class PhaseTimer:
    """CUDA events recorded on the current stream at named points of a step; ``durations()`` gives
    the device time between consecutive marks (ms), summed over repeats of the same phase name.

    Used to split a multi-GPU optimizer step into compute and each collective phase per rank."""

    def __init__(self):
        self._marks: List = []

    def mark(self, name: str) -> None:
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        self._marks.append((name, ev))

    def durations(self) -> dict:
        out: dict = {}
        for (_, a), (name, b) in zip(self._marks, self._marks[1:]):
            out[name] = out.get(name, 0.0) + a.elapsed_time(b)
        return out

    def reset(self) -> None:
        self._marks = []


def gather_phases(local: dict) -> dict:
    """Per-phase max / min / mean over ranks of a ``PhaseTimer.durations()`` dict (every rank must
    call it; identity on one rank)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return {k: {"max": v, "min": v, "mean": v} for k, v in local.items()}
    allv: List[dict] = [None] * dist.get_world_size()
    dist.all_gather_object(allv, local)
    out = {}
    for k in local:
        vals = [d.get(k, 0.0) for d in allv]
        out[k] = {"max": max(vals), "min": min(vals), "mean": sum(vals) / len(vals)}
    return out
