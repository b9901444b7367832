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
from .utils.roofline import load_peaks
from .utils.timing import median_ms


def _peaks():
    p = load_peaks()
    return p.bf16_tflops, p.hbm_gbs


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
        # tile variants: one CTA per 128 x 256 tile vs a CTA pair per 256 x 256 tile (cta_group::2)
        for tag, bn in (("single256", 256), ("pair256", -256)):
            t = median_ms(lambda: ops.gemm(a, w, out, block_n=bn))
            results[f"gemm/{name}"][f"{tag}_tflops"] = flops / t / 1e9
        # dgrad and wgrad of the same layer
        dy = torch.randn(M, N, device="cuda").bfloat16()
        dx = torch.empty(M, K, device="cuda", dtype=torch.bfloat16)
        gw = torch.zeros(N, K, device="cuda", dtype=torch.float32)
        t_d = median_ms(lambda: ops.linear_dgrad(dy, w, out=dx))
        t_w = median_ms(lambda: ops.linear_wgrad(dy, a, gw))
        variants = {}
        for tag, bn in (("single256", 256), ("single128", 128), ("pair256", -256)):
            td = median_ms(lambda: ops.gemm(dy, w, dx, b_mn=True, block_n=bn))
            tw = median_ms(lambda: ops.gemm(dy, a, gw, a_mn=True, b_mn=True, beta=1.0, out_dtype=torch.float32,
                                            block_n=bn, splits=1))
            variants[f"dgrad_{tag}_tflops"] = flops / td / 1e9
            variants[f"wgrad_{tag}_tflops"] = flops / tw / 1e9
        t_dc = median_ms(lambda: torch.matmul(dy, w, out=dx))
        gwb = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        t_wc = median_ms(lambda: torch.matmul(dy.t(), a, out=gwb))
        results[f"gemm/{name.replace('_fwd', '')}_dgrad"] = {"ms": t_d, "tflops": flops / t_d / 1e9,
                                                              "cublas_ms": t_dc, "cublas_tflops": flops / t_dc / 1e9}
        results[f"gemm/{name.replace('_fwd', '')}_wgrad"] = {"ms": t_w, "tflops": flops / t_w / 1e9,
                                                              "cublas_ms": t_wc, "cublas_tflops": flops / t_wc / 1e9}
        results[f"gemm/{name.replace('_fwd', '')}_variants"] = variants
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
    """Small launches of one kernel family for ncu captures (each a few hundred MB at most, inputs
    still larger than L2 where the kernel streams memory):

    * ``attnprof``: attention fwd+bwd on 1 x 4096 tokens, 12 q / 2 kv heads (the 1.5B shape);
    * ``gemmprof``: the gate_up GEMMs of 4096 tokens of the 1.5B shape (fwd, dgrad, wgrad);
    * ``moeprof``: grouped expert GEMMs of 4096 tokens x top-4 over 60 experts (Qwen1.5-MoE shape);
    * ``opsprof``: RMSNorm fwd/bwd, RoPE, SwiGLU fwd/bwd, embedding fwd/bwd, log-softmax/label
      fwd/bwd on 4096 response rows of a 151936 vocabulary, policy loss, AdamW on 64 M parameters;
    * ``decodeprof``: paged decode attention for 256 sequences of 1024 cached tokens, KV-cache write
      and sampling of 256 rows of a 151936 vocabulary.
    """
    dev = "cuda"
    if kind == "attnprof":
        Hq, Hkv, D, T = 12, 2, 128, 4096
        cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
        qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=dev).bfloat16()
        q, k, v = qkv[:, : Hq * D], qkv[:, Hq * D : (Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D :]
        for _ in range(2):
            o, lse = ops.attention_varlen(q, k, v, cu, T, Hq, Hkv, D)
            ops.attention_varlen_backward(torch.randn_like(o), q, k, v, o, lse, cu, T, Hq, Hkv, D)
    elif kind == "gemmprof":
        T, H, I = 4096, 1536, 8960
        x = torch.randn(T, H, device=dev).bfloat16()
        w = torch.randn(2 * I, H, device=dev).bfloat16()
        gw = torch.zeros(2 * I, H, device=dev)
        for _ in range(2):
            y = ops.gemm(x, w)
            ops.linear_dgrad(y, w)
            ops.linear_wgrad(y, x, gw)
    elif kind == "moeprof":
        from .models import moe

        E, k, H, Im, T = 60, 4, 2048, 1408, 4096
        g = torch.Generator().manual_seed(0)
        counts = torch.bincount(torch.randint(0, E, (T * k,), generator=g), minlength=E).tolist()
        lay = moe.padded_layout(counts, torch.device(dev))
        R = lay["total"]
        xs = torch.randn(R, H, device=dev).bfloat16()
        wgu = (torch.randn(E * 2 * Im, H, device=dev) * 0.02).bfloat16()
        wd = (torch.randn(E * H, Im, device=dev) * 0.02).bfloat16()
        gu = torch.empty(R, 2 * Im, device=dev, dtype=torch.bfloat16)
        ys = torch.empty(R, H, device=dev, dtype=torch.bfloat16)
        gwd = torch.zeros(E * H, Im, device=dev)
        for _ in range(2):
            moe._grouped(xs, False, wgu, False, gu, R, 2 * Im, H, 1, lay, 2 * Im)
            act = ops.swiglu(gu)
            moe._grouped(act, False, wd, False, ys, R, H, Im, 1, lay, H)
            moe._grouped(ys, True, act, True, gwd, H, Im, R, 2, lay, 0, H, beta=1.0)
    elif kind == "opsprof":
        from .algo.objectives import ObjectiveConfig

        T, H, I, V = 16384, 1536, 8960, 151936
        x = torch.randn(T, H, device=dev).bfloat16()
        w = torch.ones(H, device=dev).bfloat16()
        y, rstd = ops.rmsnorm(x, w, 1e-6)
        dw = torch.zeros(H, device=dev)
        ops.rmsnorm_backward(torch.randn_like(y), x, w, rstd, dw_grad=dw)
        qkv = torch.randn(T, 16 * 128, device=dev).bfloat16()
        pos = torch.arange(T, device=dev)
        ops.rope_(qkv, pos, 14, 128, 1e6)
        gu = torch.randn(T, 2 * I, device=dev).bfloat16()
        a = ops.swiglu(gu)
        ops.swiglu_backward(torch.randn_like(a), gu)
        emb = torch.randn(V, H, device=dev).bfloat16()
        ids = torch.randint(0, V, (T,), device=dev)
        ops.embedding(ids, emb)
        gemb = torch.zeros(V, H, device=dev)
        ops.embedding_backward(ids, x, gemb)
        n = 4096
        logits = torch.randn(n, V, device=dev).bfloat16()
        labels = torch.randint(0, V, (n,), device=dev)
        lp, lse, ent = ops.logsoftmax_label(logits, labels, with_entropy=True)
        ops.logsoftmax_label_backward(logits, labels, lse, torch.randn(n, device=dev))
        adv = torch.randn(n, device=dev)
        ops.policy_loss(lp, lp + 0.1 * torch.randn_like(lp), adv, ObjectiveConfig(), loss_scale=1e-4)
        N = 64 << 20
        master = torch.randn(N, device=dev)
        m, v, gr = torch.zeros_like(master), torch.zeros_like(master), torch.randn_like(master)
        pb = torch.empty(N, dtype=torch.bfloat16, device=dev)
        ss = torch.zeros(1, dtype=torch.float64, device=dev)
        ops.grad_sumsq(gr, ss)
        ops.adamw_step(master, m, v, gr, pb, ss, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1.0, 1)
    elif kind == "decodeprof":
        B, L, Hq, Hkv, D, bs, V = 256, 1024, 12, 2, 128, 16, 151936
        nb = B * L // bs
        kc = torch.randn(nb, bs, Hkv, D, device=dev).bfloat16()
        vc = torch.randn(nb, bs, Hkv, D, device=dev).bfloat16()
        tables = torch.arange(nb, device=dev, dtype=torch.int32).view(B, L // bs)
        lens = torch.full((B,), L, device=dev, dtype=torch.int32)
        q = torch.randn(B, Hq * D, device=dev).bfloat16()
        for impl in (1, 2, 3):  # the CUDA-core and both tensor-core kernels
            ops.paged_decode(q, kc, vc, tables, lens, Hq, Hkv, 1.0 / D ** 0.5, num_splits=4, impl=impl)
        knew = torch.randn(B, Hkv * D, device=dev).bfloat16()
        slots = (torch.arange(B, device=dev, dtype=torch.int32) * (L // bs)) * bs
        ops.kv_cache_write(knew, knew, kc, vc, slots, Hkv)
        logits = torch.randn(B, V, device=dev).bfloat16()
        temp = torch.ones(B, device=dev)
        seeds = torch.arange(B, device=dev, dtype=torch.int64)
        offs = torch.zeros(B, device=dev, dtype=torch.int64)
        ops.sample(logits, temp, seeds, offs)
    torch.cuda.synchronize()
    ops.check_status(torch.device("cuda"))


def bench_decode(results):
    """Paged decode attention: the 1.5B shape (12 q / 2 kv heads; 256 sequences of 1024 and 4096 cached
    tokens), one KV head of 8 query heads, and the Qwen1.5-MoE shape (16 q / 16 kv heads, 128 x 4096);
    achieved GB/s over the K/V bytes read, for the CUDA-core kernel and both tensor-core kernels."""
    D = 128
    _, peak_gbs = _peaks()
    # (12, 2): the 1.5B shape, KV heads interleaved in each cached token row; (8, 1): one KV head, so
    # every page of a head is one contiguous 4 KB run; (16, 16): the Qwen1.5-MoE shape (one query head
    # per KV head). 64-token pages show how much the page gathers (TMA boxes per tile) cost.
    for B, L, Hq, Hkv, bs in ((256, 1024, 12, 2, 16), (256, 4096, 12, 2, 16), (256, 4096, 12, 2, 64),
                              (256, 4096, 8, 1, 16), (128, 4096, 16, 16, 16), (128, 4096, 16, 16, 64)):
        nb = B * L // bs
        kc = torch.randn(nb, bs, Hkv, D, device="cuda").bfloat16()
        vc = torch.randn(nb, bs, Hkv, D, device="cuda").bfloat16()
        tables = torch.randperm(nb, device="cuda").to(torch.int32).view(B, L // bs)
        lens = torch.full((B,), L, device="cuda", dtype=torch.int32)
        q = torch.randn(B, Hq * D, device="cuda").bfloat16()
        nbytes = 2 * B * L * Hkv * D * 2
        entry = {"bytes": nbytes}
        for tag, impl in (("cuda_core", 1), ("tensor_core", 2), ("tensor_core_keys_as_rows", 3)):
            for splits in (1, 4):
                t = median_ms(lambda: ops.paged_decode(q, kc, vc, tables, lens, Hq, Hkv, 1.0 / D ** 0.5,
                                                       num_splits=splits, impl=impl))
                entry[f"{tag}_s{splits}_ms"] = t
                entry[f"{tag}_s{splits}_gbs"] = nbytes / t / 1e6
                entry[f"{tag}_s{splits}_frac"] = nbytes / t / 1e6 / peak_gbs
        results[f"decode/{B}x{L}/hq{Hq}_hkv{Hkv}/page{bs}"] = entry
        del kc, vc
        torch.cuda.empty_cache()


PROFILE_CASES = ("attnprof", "gemmprof", "moeprof", "opsprof", "decodeprof")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="gemm,attn,mem")
    ap.add_argument("--json", default=None)
    args = ap.parse_args()
    peak_tf, _ = _peaks()
    results = {"peak_bf16_tflops_measured": peak_tf}
    sel = set(args.only.split(","))
    if "profall" in sel:
        sel |= set(PROFILE_CASES)
    if sel & set(PROFILE_CASES):
        for kind in [c for c in PROFILE_CASES if c in sel]:
            profile_case(kind)
            torch.cuda.empty_cache()  # keep the footprint (and ncu's save/restore) small
        print("profile case done")
        return
    if "gemm" in sel:
        bench_gemm(results)
    if "attn" in sel:
        bench_attention(results)
    if "mem" in sel:
        bench_memory_bound(results)
    if "decode" in sel:
        bench_decode(results)
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
