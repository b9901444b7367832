"""Kernel micro-benchmarks on one GPU: achieved TFLOP/s or GB/s of each native kernel on the
Qwen2.5-1.5B-shape training workload (16384 packed tokens), next to the library path PyTorch would
use (cuBLAS for GEMMs, flash-attn 2 for attention where importable).

    python -m accerl_agent_b200.bench_kernels [--only gemm,attn,...] [--json out.json]

Times are CUDA-event medians after warm-up with an L2 flush before every launch.
"""

from __future__ import annotations

import argparse
import json
import math

import torch

from . import ops
from .utils.timing import median_ms


def _peaks():
    try:
        with open("MEASURED_PEAKS.json") as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), float(p["hbm_gbs"])
    except Exception:
        return 1590.0, 6650.0


def bench_gemm(results):
    T, H, I, Hq, Hkv, D = 16384, 1536, 8960, 12, 2, 128
    shapes = {
        "qkv_fwd": (T, (Hq + 2 * Hkv) * D, H),
        "o_fwd": (T, H, Hq * D),
        "gate_up_fwd": (T, 2 * I, H),
        "down_fwd": (T, H, I),
    }
    for name, (M, N, K) in shapes.items():
        a = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * M * N * K
        t_ours = median_ms(lambda: ops.gemm(a, w, out))
        t_cublas = median_ms(lambda: torch.matmul(a, w.t(), out=out))
        results[f"gemm/{name}"] = {"M": M, "N": N, "K": K, "ms": t_ours, "tflops": flops / t_ours / 1e9,
                                   "cublas_ms": t_cublas, "cublas_tflops": flops / t_cublas / 1e9}
        # dgrad and wgrad of the same layer
        dy = torch.randn(M, N, device="cuda").bfloat16()
        dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
        gw = torch.zeros(N, K, device="cuda", dtype=torch.float32)
        t_d = median_ms(lambda: ops.linear_dgrad(dy, w, out=dx))
        t_w = median_ms(lambda: ops.linear_wgrad(dy, a, gw))
        t_dc = median_ms(lambda: torch.matmul(dy, w, out=dx))
        gwb = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        t_wc = median_ms(lambda: torch.matmul(dy.t(), a, out=gwb))
        results[f"gemm/{name.replace('_fwd', '')}_dgrad"] = {"ms": t_d, "tflops": flops / t_d / 1e9,
                                                              "cublas_ms": t_dc, "cublas_tflops": flops / t_dc / 1e9}
        results[f"gemm/{name.replace('_fwd', '')}_wgrad"] = {"ms": t_w, "tflops": flops / t_w / 1e9,
                                                              "cublas_ms": t_wc, "cublas_tflops": flops / t_wc / 1e9}
        del a, w, out, dy, dx, gw, gwb


def bench_attention(results):
    Hq, Hkv, D = 12, 2, 128
    for lengths in ([8192, 8192], [2048] * 8):
        T = sum(lengths)
        cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0)), dtype=torch.int32, device="cuda")
        qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
        q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D : (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D :]
        flops = sum(2.0 * 2 * L * L * D * Hq / 2 for L in lengths)  # causal fwd
        o, lse = ops.attention_varlen(q, k, v, cu, max(lengths), Hq, Hkv, D)
        t_f = median_ms(lambda: ops.attention_varlen(q, k, v, cu, max(lengths), Hq, Hkv, D, out=o))
        do = torch.randn_like(o)
        dq = torch.empty(T, Hq * D, device="cuda", dtype=torch.bfloat16)
        dk = torch.empty(T, Hkv * D, device="cuda", dtype=torch.bfloat16)
        dv = torch.empty_like(dk)
        t_b = median_ms(lambda: ops.attention_varlen_backward(do, q, k, v, o, lse, cu, max(lengths), Hq, Hkv, D,
                                                              dq=dq, dk=dk, dv=dv))
        key = f"attn/{len(lengths)}x{lengths[0]}"
        results[key] = {"fwd_ms": t_f, "fwd_tflops": flops / t_f / 1e9, "bwd_ms": t_b,
                        "bwd_tflops": 2.5 * flops / t_b / 1e9}
        try:
            from flash_attn import flash_attn_varlen_func

            q3, k3, v3 = q.reshape(T, Hq, D), k.reshape(T, Hkv, D), v.reshape(T, Hkv, D)
            t_fa = median_ms(lambda: flash_attn_varlen_func(q3, k3, v3, cu, cu, max(lengths), max(lengths),
                                                            causal=True))
            results[key]["fa2_fwd_ms"] = t_fa
            results[key]["fa2_fwd_tflops"] = flops / t_fa / 1e9
        except Exception as exc:  # library may not run on sm_100
            results[key]["fa2"] = f"unavailable: {type(exc).__name__}: {exc}"[:200]


def bench_memory_bound(results):
    _, hbm = _peaks()
    T, H, I = 16384, 1536, 8960
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda").bfloat16()
    t = median_ms(lambda: ops.rmsnorm(x, w, 1e-6))
    b = 2 * T * H * 2
    results["rmsnorm_fwd"] = {"ms": t, "gbs": b / t / 1e6, "frac_hbm": b / t / 1e6 / hbm}
    gu = torch.randn(T, 2 * I, device="cuda").bfloat16()
    t = median_ms(lambda: ops.swiglu(gu))
    b = 3 * T * I * 2
    results["swiglu_fwd"] = {"ms": t, "gbs": b / t / 1e6, "frac_hbm": b / t / 1e6 / hbm}
    n, V = 2048, 151936
    logits = torch.randn(n, V, device="cuda").bfloat16()
    labels = torch.randint(0, V, (n,), device="cuda")
    t = median_ms(lambda: ops.logsoftmax_label(logits, labels))
    b = n * V * 2
    results["logsoftmax_label_fwd"] = {"ms": t, "gbs": b / t / 1e6, "frac_hbm": b / t / 1e6 / hbm}
    flat = torch.randn(1_500_000_000 // 4, device="cuda")
    m = torch.zeros_like(flat)
    v = torch.zeros_like(flat)
    g = torch.randn_like(flat)
    pb = torch.empty(flat.numel(), dtype=torch.bfloat16, device="cuda")
    ss = torch.zeros(1, dtype=torch.float64, device="cuda")
    t = median_ms(lambda: ops.adamw_step(flat, m, v, g, pb, ss, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1.0, 1), iters=5)
    b = flat.numel() * (4 * 4 + 4 * 3 + 2)
    results["adamw_375M"] = {"ms": t, "gbs": b / t / 1e6, "frac_hbm": b / t / 1e6 / hbm}


def profile_case(kind: str):
    """One small launch of a kernel family (for ncu captures): attention fwd+bwd on 1 x 4096 tokens,
    12 q / 2 kv heads; or the layer GEMMs of 4096 tokens of the 1.5B shape."""
    if kind == "attnprof":
        Hq, Hkv, D, T = 12, 2, 128, 4096
        cu = torch.tensor([0, T], dtype=torch.int32, device="cuda")
        qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda").bfloat16()
        q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D : (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D :]
        for _ in range(2):
            o, lse = ops.attention_varlen(q, k, v, cu, T, Hq, Hkv, D)
            ops.attention_varlen_backward(torch.randn_like(o), q, k, v, o, lse, cu, T, Hq, Hkv, D)
    elif kind == "gemmprof":
        T, H, I = 4096, 1536, 8960
        x = torch.randn(T, H, device="cuda").bfloat16()
        w = torch.randn(2 * I, H, device="cuda").bfloat16()
        gw = torch.zeros(2 * I, H, device="cuda")
        for _ in range(2):
            y = ops.gemm(x, w)
            ops.linear_dgrad(y, w)
            ops.linear_wgrad(y, x, gw)
    torch.cuda.synchronize()
    ops.check_status(torch.device("cuda"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,attn,mem")
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    peak_tf, _ = _peaks()
    results = {"peak_bf16_tflops_measured": peak_tf}
    sel = set(args.only.split(","))
    if sel & {"attnprof", "gemmprof"}:
        for kind in sel & {"attnprof", "gemmprof"}:
            profile_case(kind)
        print("profile case done")
        return
    if "gemm" in sel:
        bench_gemm(results)
    if "attn" in sel:
        bench_attention(results)
    if "mem" in sel:
        bench_memory_bound(results)
    for k, v in results.items():
        if isinstance(v, dict) and "tflops" in v:
            v["frac_of_measured_peak"] = v["tflops"] / peak_tf
    text = json.dumps(results, indent=1)
    print(text)
    if args.json:
        with open(args.json, "w") as f:
            f.write(text)


if __name__ == "__main__":
    main()
