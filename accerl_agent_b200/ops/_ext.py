"""Loader of the in-tree sm_100a extension (``accerl_agent_b200/_C*.so``).

CUDA tensors always go through the native kernels; if the extension is missing on a machine with a
GPU, ``native()`` raises instead of silently falling back. CPU tensors use the fp32 PyTorch
implementations in ``ops/reference.py`` (those are also the oracles of the kernel tests).
"""

from __future__ import annotations

import importlib
from typing import Dict, Optional

import torch

_EXT = None
_ERR: Optional[BaseException] = None
_STATUS: Dict[int, torch.Tensor] = {}


def native():
    global _EXT, _ERR
    if _EXT is not None:
        return _EXT
    try:
        _EXT = importlib.import_module("accerl_agent_b200._C")
    except ImportError as exc:  # pragma: no cover - depends on the build
        _ERR = exc
        raise RuntimeError(
            "accerl_agent_b200 native kernels are not built (run `python setup.py build_ext --inplace`): " f"{exc}"
        ) from exc
    return _EXT


def available() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


def status_tensor(device: torch.device) -> torch.Tensor:
    """Per-device int32[16] status words that bounded device-side waits write on timeout."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        t = torch.zeros(16, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def check_status(device: torch.device) -> None:
    """Raise if any kernel on ``device`` recorded a timeout (synchronises the device)."""
    t = status_tensor(device)
    value = int(t[0].item())
    if value != 0:
        t.zero_()
        raise RuntimeError(f"device-side wait timed out (status code {value}); the kernel returned early")


DEBUG_CHECK_NAMES = {1: "embedding token id", 2: "KV-cache slot", 3: "KV-cache page id", 4: "MoE row position"}


def debug_checks_enabled() -> bool:
    """True when the loaded extension was built with ``ACCERL_DEBUG_CHECKS=1`` (range checks on every
    data-dependent index; a failing check is recorded and the access skipped, never trapped)."""
    return len(native().debug_status(False)) > 0


def debug_status(reset: bool = False):
    """Failed range checks of a debug-checks build, as ``{kernel file: (check name, index)}`` (empty
    when nothing failed or in a release build). ``reset`` clears the records after reading."""
    out = {}
    for unit, code, index in native().debug_status(bool(reset)):
        if code:
            out[unit] = (DEBUG_CHECK_NAMES.get(int(code), str(code)), int(index))
    return out
