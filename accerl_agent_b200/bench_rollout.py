"""Rollout throughput of the native engine: synthetic text-game GRPO groups played against one engine
(one GPU), the way rollout workers drive it (every request carries the whole growing transcript,
16-token actions at temperature 1.0, prefix caching on).

    python -m accerl_agent_b200.bench_rollout [--model qwen2.5-1.5b] [--groups 32] [--seconds 30] [--tp 2]
    python -m accerl_agent_b200.bench_rollout --impl reference   # the reference's vLLM inference actor

Reports generated tokens/s (``Infer/TokensPerSec``), prefix-cache hit rate and engine step counts.
``--tp N`` runs one tensor-parallel engine over GPUs 0..N-1 (rank 0 in this process, the others in
spawned follower processes); every rank pulls its weight shard from a seeded full copy on its GPU.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import time

import torch

from .core.config import make_args
from .models.config import get_preset
from .rollout.inference import InferenceService
from .rollout.worker import RolloutWorker


async def _drive(service, args, groups: int, seconds: float, profile: float = 0.0, warmup: float = 3.0):
    sink_samples = []
    worker_list = [RolloutWorker(args, service, i, sink_samples.extend, lambda *a: None) for i in range(groups)]
    tasks = [asyncio.create_task(w.run()) for w in worker_list]
    await asyncio.sleep(warmup)  # warm-up: prefill of the first observations, kernel caches
    if profile > 0:
        # kernel-time breakdown of a window of engine steps (not a throughput measurement)
        from torch.profiler import ProfilerActivity, profile as tprof

        with tprof(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as prof:
            await asyncio.sleep(profile)
        steps = service.engine.stats["steps"]
        print(prof.key_averages().table(sort_by="cuda_time_total", row_limit=25, max_name_column_width=60))
        print(prof.key_averages().table(sort_by="self_cpu_time_total", row_limit=25, max_name_column_width=60))
        print(f"[profile] engine steps so far: {steps}")
    tok0 = service.total_tokens
    t0 = time.perf_counter()
    await asyncio.sleep(seconds)
    tok1 = service.total_tokens
    el = time.perf_counter() - t0
    for w in worker_list:
        await w.stop()
    await asyncio.wait(tasks, timeout=60)
    return (tok1 - tok0) / el, el, len(sink_samples)


def _seed_weights(engine, dev):
    """Every rank builds the same seeded full model on its GPU and pulls its shard from it."""
    from .models.transformer import build_model

    full = build_model(engine.full_cfg, "full", dev, torch.bfloat16)
    full.init_weights(seed=0)
    engine.set_weight_source(full.layout, addr=full.params.data_ptr())
    return full


def _follower(rank: int, tp: int, port: int, args):
    from .rollout.inference import build_engine, init_tp_groups

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    engine = build_engine(args, dev, tp_groups=init_tp_groups(rank, tp, port, dev))
    full = _seed_weights(engine, dev)
    engine.serve_follower()
    del full


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-1.5b")
    ap.add_argument("--groups", type=int, default=32, help="concurrent GRPO groups (x8 trajectories)")
    ap.add_argument("--seconds", type=float, default=30.0)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--max-num-batched-tokens", type=int, default=8192)
    ap.add_argument("--window", type=int, default=8192)
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks of the engine (GPUs 0..tp-1)")
    ap.add_argument("--profile-seconds", type=float, default=0.0,
                    help="print a torch.profiler kernel table of this many seconds before timing")
    ap.add_argument("--warmup-seconds", type=float, default=3.0)
    ap.add_argument("--gpu-memory-utilization", type=float, default=0.8,
                    help="share of the device the engine may hold (weights + KV cache), as the reference passes to vLLM")
    ap.add_argument("--impl", default="native", choices=("native", "reference"),
                    help="reference: the reference's own vLLM inference actor, driven by the same rollout loop")
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    if a.impl == "reference":
        import os
        import sys

        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        from baseline.reference_rollout import run_reference_rollout

        run_reference_rollout(a)
        return
    args = make_args(model_path=a.model, env="synthetic", rl_algorithm="grpo", rollout_batch_size=8,
                     tw_max_episode_steps=50, tw_history_token_window=a.window, max_length=a.window,
                     infer_max_tokens=16, infer_temperature=1.0, vllm_max_num_seqs=a.max_num_seqs,
                     vllm_max_num_batched_tokens=a.max_num_batched_tokens)
    args.gpu_memory_utilization = a.gpu_memory_utilization
    dev = torch.device("cuda", 0)
    procs, full = [], None
    if a.tp > 1:
        import socket

        import torch.multiprocessing as mp

        from .rollout.inference import init_tp_groups

        args.infer_tp_size = a.tp
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            port = sk.getsockname()[1]
        ctx = mp.get_context("spawn")
        procs = [ctx.Process(target=_follower, args=(r, a.tp, port, args)) for r in range(1, a.tp)]
        for p in procs:
            p.start()
        service = InferenceService(args, dev, tp_groups=init_tp_groups(0, a.tp, port, dev))
        full = _seed_weights(service.engine, dev)
        service.engine.pull_weights("all")
        del full
        torch.cuda.empty_cache()
    else:
        service = InferenceService(args, dev)
        service.engine.model.init_weights(seed=0)
    rate, el, samples = asyncio.run(_drive(service, args, a.groups, a.seconds, a.profile_seconds,
                                                a.warmup_seconds))
    st = service.get_stats()
    out = {
        "metric": "rollout tok/s",
        "value": round(rate, 1),
        "kv_cache_tokens": service.engine.num_blocks * service.engine.block_size,
        "unit": f"generated tokens/s (Infer/TokensPerSec), one engine on {a.tp} GPU(s)",
        "tp": a.tp,
        "model": a.model,
        "concurrent_trajectories": a.groups * 8,
        "max_num_seqs": a.max_num_seqs,
        "seconds": round(el, 2),
        "samples_produced": samples,
        "prefix_cache_hit_rate": round(st["prefix_cache_hit_rate"], 4),
        "engine_steps": st["steps"],
        "preemptions": st["preemptions"],
        "step_phase_ms": {k[2:-2]: round(1e3 * st[k] / max(st["steps"], 1), 3)
                          for k in ("t_schedule_s", "t_launch_s", "t_complete_s")},
        "rows_per_step": {"prefill": round(st["prefill_rows"] / max(st["steps"], 1), 1),
                          "decode": round(st["decode_rows"] / max(st["steps"], 1), 1)},
    }
    print(json.dumps(out))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(out, f, indent=1)
    asyncio.run(service.shutdown())
    for p in procs:
        p.join(120)


if __name__ == "__main__":
    main()
