"""Roofline arithmetic against the measured B200 peaks.

The denominators are the driver-measured figures in ``MEASURED_PEAKS.json`` at the repository root
(a STREAM-style copy for HBM, a cuBLAS bf16 GEMM burst and its seconds-long sustained figure under
the power cap). Without that file the fallback figures below, an earlier measurement on the same
hardware, are used and ``source`` says so. NVLink figures are the measured peer copy (770 GB/s per
direction per GPU) and the 8-rank all-reduce bus bandwidth (725 GB/s at 1 GiB).

    python -m accerl_agent_b200.utils.roofline gemm M N K MS [--sustained]
    python -m accerl_agent_b200.utils.roofline bytes NBYTES MS
    python -m accerl_agent_b200.utils.roofline fused FLOPS LINK_BYTES MS

A fused compute+collective kernel's target time is the slower of FLOPs at the GEMM peak and the
bytes that must cross NVLink at the link bandwidth; ``frac`` is target / achieved (1.0 = on the
roofline). A fraction a little above 1.0 is possible because the denominators are a plain copy and
cuBLAS; far above it means the timed kernel did not do the work.
"""

from __future__ import annotations

import argparse
import json
import os
from dataclasses import dataclass
from typing import Dict, Optional

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0
NVLINK_PEER_GBS = 770.0
NVLINK_ALLREDUCE_BUS_GBS = 725.0

_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


@dataclass(frozen=True)
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    nvlink_gbs: float = NVLINK_PEER_GBS
    source: str = "measured"


def load_peaks(path: Optional[str] = None) -> Peaks:
    path = path or os.path.join(_ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return Peaks(float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                     float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), source="measured")
    except (OSError, KeyError, ValueError):
        return Peaks(FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS_SUSTAINED, source="fallback")


def gemm(M: int, N: int, K: int, ms: float, sustained: bool = False, peaks: Optional[Peaks] = None) -> Dict:
    """Achieved TFLOP/s of an ``M x N x K`` GEMM that took ``ms`` and its fraction of the peak."""
    p = peaks or load_peaks()
    flops = 2.0 * M * N * K
    tf = flops / (ms * 1e-3) / 1e12
    peak = p.bf16_tflops_sustained if sustained else p.bf16_tflops
    return {"flops": flops, "tflops": tf, "peak_tflops": peak, "frac": tf / peak, "of": p.source,
            "ideal_ms": flops / (peak * 1e12) * 1e3}


def memory(nbytes: float, ms: float, peaks: Optional[Peaks] = None) -> Dict:
    """Achieved GB/s of a kernel that must move ``nbytes`` (reads + writes) in ``ms``."""
    p = peaks or load_peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"bytes": nbytes, "gbs": gbs, "peak_gbs": p.hbm_gbs, "frac": gbs / p.hbm_gbs, "of": p.source,
            "ideal_ms": nbytes / (p.hbm_gbs * 1e9) * 1e3}


def fused(flops: float, link_bytes: float, ms: float, sustained: bool = False, peaks: Optional[Peaks] = None) -> Dict:
    """Roofline of a compute step fused with its collective: the target is the slower of the math
    at the GEMM peak and the bytes over NVLink at the measured link bandwidth."""
    p = peaks or load_peaks()
    peak = p.bf16_tflops_sustained if sustained else p.bf16_tflops
    t_math = flops / (peak * 1e12) * 1e3
    t_link = link_bytes / (p.nvlink_gbs * 1e9) * 1e3
    target = max(t_math, t_link)
    return {"math_ms": t_math, "link_ms": t_link, "target_ms": target, "bound": "math" if t_math >= t_link else "link",
            "achieved_ms": ms, "frac": target / ms, "of": p.source}


def arithmetic_intensity_gemm(M: int, N: int, K: int, elem_bytes: int = 2, out_bytes: int = 2) -> float:
    """FLOPs per DRAM byte of a GEMM that reads A and B once and writes C once."""
    return 2.0 * M * N * K / (elem_bytes * (M * K + N * K) + out_bytes * M * N)


def ridge_point(peaks: Optional[Peaks] = None) -> float:
    """FLOPs per byte above which a kernel is compute-bound on this GPU."""
    p = peaks or load_peaks()
    return p.bf16_tflops * 1e12 / (p.hbm_gbs * 1e9)


def main(argv=None) -> Dict:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="kind", required=True)
    g = sub.add_parser("gemm")
    for k in ("M", "N", "K"):
        g.add_argument(k, type=int)
    g.add_argument("ms", type=float)
    g.add_argument("--sustained", action="store_true")
    b = sub.add_parser("bytes")
    b.add_argument("nbytes", type=float)
    b.add_argument("ms", type=float)
    f = sub.add_parser("fused")
    f.add_argument("flops", type=float)
    f.add_argument("link_bytes", type=float)
    f.add_argument("ms", type=float)
    f.add_argument("--sustained", action="store_true")
    a = ap.parse_args(argv)
    if a.kind == "gemm":
        out = gemm(a.M, a.N, a.K, a.ms, a.sustained)
    elif a.kind == "bytes":
        out = memory(a.nbytes, a.ms)
    else:
        out = fused(a.flops, a.link_bytes, a.ms, a.sustained)
    print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in out.items()}))
    return out


if __name__ == "__main__":
    main()
