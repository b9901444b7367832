"""CUDA memory report of the calling process (the reference's vLLM worker extension
``vllm_memory_reporter.py:6-37``: allocated / reserved / peak / driver-used GiB)."""

from __future__ import annotations

import os
from typing import Dict, Optional

import torch


def cuda_memory_report(label: str, empty_cache: bool = False, device: Optional[int] = None,
                       verbose: bool = True) -> Dict[str, float]:
    if empty_cache:
        torch.cuda.empty_cache()
    torch.cuda.synchronize()
    dev = torch.cuda.current_device() if device is None else device
    free_b, total_b = torch.cuda.mem_get_info(dev)
    g = 1024**3
    stats = {
        "label": label,
        "pid": os.getpid(),
        "device": dev,
        "allocated_gib": torch.cuda.memory_allocated(dev) / g,
        "reserved_gib": torch.cuda.memory_reserved(dev) / g,
        "max_allocated_gib": torch.cuda.max_memory_allocated(dev) / g,
        "max_reserved_gib": torch.cuda.max_memory_reserved(dev) / g,
        "driver_used_gib": (total_b - free_b) / g,
        "driver_total_gib": total_b / g,
    }
    if verbose:
        print(f"[engine CUDA memory] {label} pid={stats['pid']} cuda:{dev} allocated={stats['allocated_gib']:.2f}GiB "
              f"reserved={stats['reserved_gib']:.2f}GiB max_reserved={stats['max_reserved_gib']:.2f}GiB "
              f"driver_used={stats['driver_used_gib']:.2f}/{stats['driver_total_gib']:.2f}GiB", flush=True)
    return stats
