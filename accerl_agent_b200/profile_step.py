"""Per-kernel device-time breakdown of one trainer optimizer step (CUPTI via torch.profiler).

    python -m accerl_agent_b200.profile_step [--packs 2] [--json out.json]

Prints each kernel family's share of device time. Numbers taken under the profiler are shares for
finding hot spots, not benchmark results (``bench.py`` reports those).
"""

from __future__ import annotations

import argparse
import json
from collections import defaultdict

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--packs", type=int, default=2)
    ap.add_argument("--model", default="qwen2.5-1.5b")
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    from .core.config import make_args
    from .env.synthetic_samples import benchmark_pool
    from .replay import ReplayBuffer
    from .trainer.worker import TrainWorker

    args = make_args(model_path=a.model, train_packing="varlen", train_token_budget=16384, max_length=8192,
                     tw_history_token_window=8192, batch_size=2, grad_accum_steps=a.packs,
                     train_logprob_mode="response_only_lm_head", learning_rate=1e-6, lr_warmup_steps=0,
                     max_steps=10**6, dtype="bfloat16", fsdp_world_size=1, device="cuda")
    rb = ReplayBuffer(args.replay_capacity, seed=0)
    rb.add_samples(benchmark_pool(0, args.replay_capacity, 8192))
    w = TrainWorker(args, replay_buffer=rb, device=torch.device("cuda", 0))
    w.train_until_next_sync(1)
    packs, gtok = w.stage_window()
    torch.cuda.synchronize()
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
        w.train_step_on_device(packs, gtok)
        torch.cuda.synchronize()
    fam = defaultdict(float)
    count = defaultdict(int)
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA:
            name = ev.name
            key = name.split("<")[0].split("(")[0]
            if "gemm_bf16_tcgen05" in name:
                key = "gemm_bf16_tcgen05<" + name.split("<", 1)[1].split(">")[0] + ">"
            fam[key] += ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
            count[key] += 1
    total = sum(fam.values())
    rows = sorted(fam.items(), key=lambda kv: -kv[1])
    tokens = sum(int(p.batch["input_ids"].numel()) for p in packs)
    out = {"total_device_ms": total / 1e3, "packs": a.packs, "tokens": tokens,
           "kernels": [{"name": k, "ms": v / 1e3, "share": v / total, "launches": count[k]} for k, v in rows]}
    print(f"total device time {total / 1e3:.2f} ms for {a.packs} packs ({tokens} tokens)")
    for r in out["kernels"][:30]:
        print(f"{r['share'] * 100:6.2f}%  {r['ms']:9.3f} ms  x{r['launches']:5d}  {r['name']}")
    if a.json:
        with open(a.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
