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
