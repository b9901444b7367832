"""Headline benchmark: trainer tokens/s of the async-GRPO varlen optimizer step on the
Qwen2.5-1.5B-shape dense model (28 layers, hidden 1536, 12 q / 2 KV heads, intermediate 8960,
vocab 151936, tied embeddings), bf16, random init, fed with synthetic text-game episodes
(observations of U[64,256] random tokens, 16-token actions, end at 50 steps or p=0.02, history window
8192, groups of 8, GRPO advantages), packed varlen to a 16384-token budget with PPO clip 0.2.

``value`` follows the reference's ``Train/TokensPerSec``: global valid response (target) tokens per
second of optimizer steps, device-timed with CUDA events (barrier + synchronize on both sides, max over
ranks). ``e2e`` times the public ``TrainWorker.train_until_next_sync(1)`` call, which samples the
replay buffer, packs on the CPU, copies the pack from pinned memory and reads the step statistics back.

    python bench.py --gpus N --steps K --warmup W            # this framework
    python bench.py --impl reference --gpus N ...            # the reference's own trainer code
For N > 1 run under ``torch.distributed.run`` (one rank per GPU).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

REFERENCE_PUBLISHED_VALUE = None  # the reference publishes no numbers

MODEL_DESC = "Qwen2.5-1.5B-shape dense (28L, H1536, 12q/2kv heads, I8960, V151936, tied)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=("native", "reference"))
    ap.add_argument("--grad-accum-steps", type=int, default=8)
    ap.add_argument("--batch-size", type=int, default=2)
    ap.add_argument("--token-budget", type=int, default=16384)
    ap.add_argument("--max-length", type=int, default=8192)
    ap.add_argument("--model", default="qwen2.5-1.5b")
    ap.add_argument("--expert-parallel", action="store_true",
                    help="MoE models: experts partitioned over the ranks, token dispatch/combine over NVLink")
    ap.add_argument("--shard-params", action="store_true",
                    help="parameters, gradients and optimizer state sharded per layer (FSDP full sharding)")
    return ap.parse_args()


def model_desc(name: str) -> str:
    if name == "qwen2.5-1.5b":
        return MODEL_DESC
    from accerl_agent_b200.models.config import get_preset

    c = get_preset(name)
    moe = (f", {c.num_experts} experts top-{c.num_experts_per_tok} (I{c.moe_intermediate_size}"
           f"{f', shared {c.shared_expert_intermediate_size}' if c.shared_expert_intermediate_size else ''})"
           if c.num_experts else f", I{c.intermediate_size}")
    return (f"{name}-shape {'MoE' if c.num_experts else 'dense'} ({c.num_hidden_layers}L, H{c.hidden_size}, "
            f"{c.num_attention_heads}q/{c.num_key_value_heads}kv heads{moe}, V{c.vocab_size})")


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def synthetic_pool(rank: int, samples: int, window: int):
    from accerl_agent_b200.env.synthetic_samples import benchmark_pool

    return benchmark_pool(rank, samples, window)


def emit(line: dict):
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------
# native arm
# ----------------------------------------------------------------------------------------------
def run_native(a):
    import torch
    import torch.distributed as dist

    from accerl_agent_b200 import ops
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker
    from accerl_agent_b200.utils.clocks import ClockSampler
    from accerl_agent_b200.utils.timing import PhaseTimer, gather_phases, max_over_ranks

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    args = make_args(
        model_path=a.model, train_packing="varlen", train_token_budget=a.token_budget, max_length=a.max_length,
        tw_history_token_window=a.max_length, batch_size=a.batch_size, grad_accum_steps=a.grad_accum_steps,
        train_logprob_mode="response_only_lm_head", rl_algorithm="grpo", clip_mode="ppo", clip_eps=0.2,
        learning_rate=1e-6, lr_warmup_steps=0, max_steps=10**6, dtype="bfloat16", fsdp_world_size=world,
        device="cuda", seed=42, expert_parallel=a.expert_parallel, shard_params=a.shard_params,
    )
    pool = synthetic_pool(rank, 256, a.max_length)
    replay = ReplayBuffer(args.replay_capacity, seed=rank)
    replay.add_samples(pool[: args.replay_capacity])
    trainer = TrainWorker(args, rank=rank, fsdp_world_size=world, replay_buffer=replay,
                          device=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- warm-up through the public API
    for _ in range(a.warmup):
        trainer.train_until_next_sync(1)
    torch.cuda.synchronize()

    # ---- device-timed optimizer steps on device-resident packs
    staged = [trainer.stage_window() for _ in range(a.steps)]
    torch.cuda.synchronize()
    barrier()
    launches0 = ops.LAUNCHES[0]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # per-rank phase split of the multi-GPU step (event records only; no synchronisation is added)
    timer = PhaseTimer() if world > 1 else None
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        start.record()
        for packs, gtok in staged:
            if timer is not None:
                timer.mark("step_start")
            trainer.train_step_on_device(packs, gtok, timer=timer)
        end.record()
        torch.cuda.synchronize()
        barrier()
    launches = (ops.LAUNCHES[0] - launches0) / a.steps
    dev_ms = max_over_ranks(start.elapsed_time(end))
    phases = None
    if timer is not None:
        per_phase = {k: v / a.steps for k, v in timer.durations().items() if k != "step_start"}
        lens = [(dp.batch["cu_seqlens"][1:] - dp.batch["cu_seqlens"][:-1]).double() for packs, _ in staged
                for dp in packs]
        per_phase["tokens"] = sum(float(x.sum()) for x in lens) / a.steps
        per_phase["attn_sum_len_sq_1e6"] = sum(float((x * x).sum()) for x in lens) / a.steps / 1e6
        phases = {k: {kk: round(vv, 3) for kk, vv in v.items()} for k, v in gather_phases(per_phase).items()}
    tokens = sum(g for _, g in staged)
    total_tokens_local = sum(int(dp.batch["input_ids"].numel()) for packs, _ in staged for dp in packs)
    total_tokens = total_tokens_local
    if world > 1:
        t = torch.tensor([total_tokens_local], dtype=torch.float64, device="cuda")
        dist.all_reduce(t)
        total_tokens = float(t.item())
    del staged

    # ---- end-to-end through the public API
    torch.cuda.synchronize()
    barrier()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_tokens = 0.0
    h2d = 0
    with ClockSampler(local) as clocks2:
        barrier()
        torch.cuda.synchronize()
        s2.record()
        for _ in range(a.steps):
            summary = trainer.train_until_next_sync(1)  # includes the D2H read of the step statistics
            e2e_tokens += summary["segment_valid_tokens"]
            h2d += trainer.last_h2d_bytes
        e2.record()
        torch.cuda.synchronize()
        barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))

    value = tokens / (dev_ms / 1e3)
    cs = clocks.summary()
    if rank == 0:
        emit({
            "metric": "trainer tok/s",
            "value": round(value, 1),
            "unit": "target tokens/s (global valid response tokens per second, Train/TokensPerSec)",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": round(dev_ms / a.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None if REFERENCE_PUBLISHED_VALUE is None else value / REFERENCE_PUBLISHED_VALUE,
            "dtype": "bf16",
            "data": "synthetic (seeded synthetic text-game episodes, random-init weights)",
            "impl": "native",
            "config": {
                "model": model_desc(a.model),
                "global_batch": a.batch_size * a.grad_accum_steps * world,
                "seq_len": a.max_length,
                "token_budget_per_pack": a.token_budget,
                "grad_accum_steps": a.grad_accum_steps,
                "parallelism": f"fsdp{world}" + (f"+ep{world}" if a.expert_parallel and world > 1 else "")
                               + ("-full-shard" if a.shard_params else ""),
                "algorithm": "grpo advantages + ppo clip 0.2, varlen packing, response-only LM head",
                "l2": "inputs larger than L2 (GBs of weights/activations per step); no flush needed",
            },
            "total_tokens_per_s": round(total_tokens / (dev_ms / 1e3), 1),
            "target_tokens_per_step": round(tokens / a.steps, 1),
            "e2e": {
                "value": round(e2e_tokens / (e2e_ms / 1e3), 1),
                "unit": "target tokens/s through TrainWorker.train_until_next_sync",
                "ms_per_step": round(e2e_ms / a.steps, 3),
                "h2d_bytes_per_step": int(h2d / a.steps),
                "d2h_bytes_per_step": 3 * 8 + 2 * 8 + 8,
            },
            "gpu_launches": int(launches),
            **({"phases_ms_per_step": phases} if phases is not None else {}),
            "clocks": {"sm_mhz": cs.get("sm_mhz"), "sm_max_mhz": cs.get("sm_max_mhz"),
                       "reasons": cs.get("reasons", []), "samples": cs.get("samples", 0),
                       "e2e_region": clocks2.summary()},
        })
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    a = parse()
    if a.impl == "reference":
        from baseline.reference_arm import run_reference

        run_reference(a)
    else:
        run_native(a)


if __name__ == "__main__":
    main()
