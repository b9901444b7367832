"""MoE block benchmark: router, expert dispatch, grouped expert GEMMs, combine, shared expert, forward
and backward, at the Qwen1.5-MoE-A2.7B layer shape (hidden 2048, 60 experts top-4, expert
intermediate 1408, shared expert 5632) with 16384 tokens per GPU.

    python -m accerl_agent_b200.bench_moe [--tokens 16384] [--steps 10] [--warmup 3]
    torchrun --nproc-per-node N -m accerl_agent_b200.bench_moe --transport p2p|all_to_all

One GPU runs the local grouped-GEMM path. With N ranks the experts are partitioned over the ranks
(expert parallelism) and rows move either through the fused peer-memory path (``p2p``: P2P dispatch
stores, down-projection GEMM whose epilogue stores rows into the source rank) or through NCCL
``all_to_all_single`` around plain grouped GEMMs (``all_to_all``, the library baseline). Timing is
CUDA events on each rank, max over ranks; the MoE input (64 MB per rank) is regenerated between
steps and the expert weights (1 GB per layer) exceed L2, so steps do not run from cache.
"""

from __future__ import annotations

import argparse
import json
import os
import types

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen1.5-moe-a2.7b")
    ap.add_argument("--tokens", type=int, default=16384, help="tokens per GPU")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--transport", default="p2p", choices=("p2p", "all_to_all"))
    ap.add_argument("--json", default=None)
    a = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from .models import moe
    from .models.config import get_preset
    from .models.transformer import build_model

    cfg = get_preset(a.model)
    cfg.num_hidden_layers = 1
    cfg.vocab_size = 1024  # only the MoE block of layer 0 runs
    model = build_model(cfg, "full", dev, torch.bfloat16, pad_to=world)
    model.init_weights(seed=0)
    if world > 1:
        from .parallel.expert_parallel import ExpertParallel

        model.expert_parallel = ExpertParallel(cfg, max_tokens=a.tokens, device=dev, transport=a.transport)
    T, H = a.tokens, cfg.hidden_size
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    hs = [torch.randn(T, H, device=dev, dtype=torch.bfloat16, generator=gen) for _ in range(2)]
    resid = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
    dy = torch.randn(T, H, device=dev, dtype=torch.bfloat16, generator=gen) * 1e-3

    def step(i):
        h = hs[i % 2]
        out, cache = moe.moe_forward(model, 0, h, resid, True)
        ctx = types.SimpleNamespace(mlp=cache, h2=h)
        moe.moe_backward(model, 0, dy, ctx)
        return out

    for i in range(a.warmup):
        step(i)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(a.steps):
        step(i)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / a.steps
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms = float(t.item())
    k, Im, Is = cfg.num_experts_per_tok, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    # fwd + dgrad + wgrad of the routed and shared expert MLPs (router and combine excluded)
    flops = 3 * 2 * T * (k * 3 * H * Im + 3 * H * Is)
    if rank == 0:
        res = {
            "metric": "moe block tok/s",
            "value": round(world * T / (ms / 1e3), 1),
            "unit": "tokens/s through one MoE block, forward+backward, all GPUs",
            "n_gpus": world,
            "ms_per_step": round(ms, 3),
            "expert_tflops_per_gpu": round(flops / (ms / 1e3) / 1e12, 1),
            "transport": a.transport if world > 1 else "local",
            "config": {"model": a.model, "tokens_per_gpu": T, "hidden": H, "experts": cfg.num_experts, "top_k": k,
                       "expert_intermediate": Im, "shared_intermediate": Is},
            "steps": a.steps, "warmup": a.warmup, "dtype": "bf16", "data": "synthetic",
        }
        print(json.dumps(res))
        if a.json:
            with open(a.json, "w") as f:
                json.dump(res, f, indent=1)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
