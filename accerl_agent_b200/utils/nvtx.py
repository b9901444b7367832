"""NVTX ranges around the framework's phases, for timeline profilers (Nsight Systems, ``ncu --nvtx``).

The reference has no tracing hooks; its only timing is ``time.perf_counter()`` around training
segments and weight syncs (``accerl_agent/agent_textworld.py:3114-3127``). Here every phase that a
timeline should show is wrapped in ``nvtx.range("phase")``:

  trainer:   ``train/prepare_window``, ``train/h2d``, ``train/forward``, ``train/loss``,
             ``train/backward``, ``train/stats_allreduce``, ``train/optimizer``
  engine:    ``engine/schedule``, ``engine/launch``, ``engine/complete``, ``engine/pull_weights``

Ranges are off unless ``ACCERL_NVTX=1`` is set in the environment (or ``enable()`` is called), so
the default path costs one attribute check per phase. Ranges nest; ``ncu --nvtx --nvtx-include
"train/backward/"`` then limits a capture to the kernels of one phase.
"""

from __future__ import annotations

import contextlib
import os

import torch

_enabled = os.environ.get("ACCERL_NVTX", "0") not in ("", "0", "false", "False")


def enable(on: bool = True) -> None:
    global _enabled
    _enabled = bool(on)


def enabled() -> bool:
    return _enabled


class _Range:
    __slots__ = ("name",)

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        torch.cuda.nvtx.range_pop()
        return False


_NULL = contextlib.nullcontext()


def range(name: str):  # noqa: A001 - mirrors torch.cuda.nvtx.range
    """Context manager that marks ``name`` on the NVTX timeline when ranges are enabled."""
    return _Range(name) if _enabled else _NULL


def mark(name: str) -> None:
    if _enabled:
        torch.cuda.nvtx.mark(name)
