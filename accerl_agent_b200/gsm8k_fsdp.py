"""Math (GSM8K) variant of the asynchronous RL loop: sharded trainer + native rollout engines.

Command-line surface of the reference's GSM8K loop (``vllm_fsdp.py:2251-2529``: same flag names,
defaults and validation rules), running on this framework's runtime: trainer ranks (one process per
GPU, sharded AdamW), rollout engines with in-process math rollout workers
(``rollout/math_worker.py``), the CUDA-IPC weight pull every ``--sync-every-optimizer-steps``.

Differences from the TextWorld loop, all from the reference variant: R1-zero prompts, one prompt per
group of ``--rollout-batch-size`` sampled answers that stop at ``</answer>``, rewards from the math
grader, a group advantage that is zero unless two or more answers are right, the padded per-sample
mean loss, ``--clip-mode none`` (advantage x log-prob) by default, a constant learning rate and
sampling at temperature 0.7 / top-p 0.9.

``--gsm8k-train-path synthetic`` (the default here: there is no dataset download) trains on seeded
arithmetic word problems; a real GSM8K ``train.jsonl`` path is read as the reference reads it.
``--model-path`` accepts a preset name (random init) or a local HF model directory; without tokenizer
files a byte-level tokenizer is used.
"""

from __future__ import annotations

import argparse
import os
import time
from typing import List, Optional

from .core.config import build_parser as build_agent_parser
from .core.config import finalize_args

FSDP_WORLD_SIZE = 6
INFERENCE_DP_SIZE = 2


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description="GSM8K GRPO on B200: sharded trainer + native interruptible rollout engine.")
    a = p.add_argument
    a("--model-path", default="qwen1.5-moe-a2.7b")
    a("--dtype", default="auto", choices=("auto", "bfloat16", "float16", "float32"))
    a("--train-mode", default="lm_head", choices=("lm_head", "last_layer", "full"))
    a("--gsm8k-train-path", default="synthetic", help="Path to GSM8K train jsonl, or 'synthetic'.")
    a("--gsm8k-limit", type=int, default=None)
    a("--max-length", type=int, default=2048)
    a("--batch-size", type=int, default=16)
    a("--max-steps", type=int, default=5000)
    a("--learning-rate", type=float, default=1e-5)
    a("--weight-decay", type=float, default=0.0)
    a("--grad-accum-steps", type=int, default=8)
    a("--train-logprob-mode", type=str, default="full_logits_ce", choices=["full_logits_ce", "response_only_lm_head"])
    a("--clip-mode", type=str, default="none", choices=["none", "ppo", "gipo", "sapo"])
    a("--clip-eps", type=float, default=0.2)
    a("--gipo-sigma", type=float, default=1.0)
    a("--sapo-tau-pos", type=float, default=1.0)
    a("--sapo-tau-neg", type=float, default=2.0)
    a("--replay-capacity", type=int, default=None)
    a("--replay-wait-sleep-seconds", type=float, default=0.2)
    a("--replay-sample-timeout-seconds", type=float, default=None)
    a("--log-every", type=int, default=1)
    a("--metrics-window-size", type=int, default=1000)
    a("--metrics-active-timeout-seconds", type=float, default=600.0)
    a("--log-dir", default=None)
    a("--seed", type=int, default=42)
    a("--trust-remote-code", action="store_true")
    a("--gradient-checkpointing", action="store_true")
    a("--fsdp-world-size", type=int, default=FSDP_WORLD_SIZE)
    a("--fsdp-master-addr", default=None)
    a("--fsdp-master-port", type=int, default=None)
    a("--ray-address", default=None, help="Accepted for command-line compatibility; this runtime does not use Ray.")
    a("--sync-every-optimizer-steps", type=int, default=8)
    a("--infer-max-tokens", type=int, default=512)
    a("--infer-temperature", type=float, default=0.7)
    a("--infer-top-p", type=float, default=0.9)
    a("--infer-actor-max-concurrency", type=int, default=1024,
      help="Upper bound on in-flight generation requests per engine (the engine admits at most "
           "--vllm-max-num-seqs of them per step).")
    a("--num-rollout-workers", type=int, default=8)
    a("--rollout-batch-size", type=int, default=8)
    a("--rollout-stop-timeout", type=float, default=10.0)
    a("--vllm-max-num-seqs", type=int, default=128)
    a("--vllm-max-num-batched-tokens", type=int, default=8192)
    a("--max-sync-rounds", type=int, default=None)
    # additions of this framework
    a("--infer-size", type=int, default=INFERENCE_DP_SIZE, help="Number of rollout engines (one GPU each).")
    a("--device", default="auto", help="auto | cpu | cuda")
    a("--kv-cache-gb", type=float, default=None)
    a("--expert-parallel", action="store_true")
    a("--save-checkpoint", action="store_true")
    a("--checkpoint-dir", default=None)
    return p


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    args = build_parser().parse_args(argv)
    if args.clip_eps <= 0:
        raise ValueError(f"--clip-eps must be > 0, got {args.clip_eps}")
    if args.gipo_sigma <= 0:
        raise ValueError(f"--gipo-sigma must be > 0, got {args.gipo_sigma}")
    if args.sapo_tau_pos <= 0 or args.sapo_tau_neg <= 0:
        raise ValueError(f"--sapo-tau-pos and --sapo-tau-neg must be > 0, got {args.sapo_tau_pos}, {args.sapo_tau_neg}")
    if args.replay_capacity is None:
        args.replay_capacity = args.batch_size * args.grad_accum_steps * 4
    if args.replay_sample_timeout_seconds is None:
        args.replay_sample_timeout_seconds = 0.0
    if args.log_dir is None:
        args.log_dir = os.path.join("runs", "VLLM_FSDP", time.strftime("%Y-%m-%d_%H-%M-%S"))
    return args


def validate_args(args: argparse.Namespace) -> None:
    """The reference's rules (``vllm_fsdp.py:2478-2529``); ``synthetic`` replaces a dataset path."""
    if args.gsm8k_train_path != "synthetic" and not os.path.isfile(args.gsm8k_train_path):
        raise ValueError(f"--gsm8k-train-path must point to an existing jsonl file: {args.gsm8k_train_path!r}")
    checks = [
        (args.gsm8k_limit is not None and args.gsm8k_limit < 1, "--gsm8k-limit must be >= 1 when set"),
        (args.grad_accum_steps < 1, "--grad-accum-steps must be >= 1"),
        (args.max_steps < 1, "--max-steps must be >= 1"),
        (args.batch_size < 1, "--batch-size must be >= 1"),
        (args.replay_capacity < 1, "--replay-capacity must be >= 1"),
        (args.replay_wait_sleep_seconds <= 0, "--replay-wait-sleep-seconds must be > 0"),
        (args.replay_sample_timeout_seconds < 0, "--replay-sample-timeout-seconds must be >= 0"),
        (args.max_length < 1, "--max-length must be >= 1"),
        (args.log_every < 1, "--log-every must be >= 1"),
        (args.metrics_window_size < 1, "--metrics-window-size must be >= 1"),
        (args.metrics_active_timeout_seconds <= 0, "--metrics-active-timeout-seconds must be > 0"),
        (args.fsdp_world_size < 1, "--fsdp-world-size must be >= 1"),
        (args.sync_every_optimizer_steps < 1, "--sync-every-optimizer-steps must be >= 1"),
        (args.infer_max_tokens < 1, "--infer-max-tokens must be >= 1"),
        (args.infer_temperature < 0.0, "--infer-temperature must be >= 0"),
        (not 0.0 < args.infer_top_p <= 1.0, "--infer-top-p must be in (0, 1]"),
        (args.infer_actor_max_concurrency < 1, "--infer-actor-max-concurrency must be >= 1"),
        (args.num_rollout_workers < 1, "--num-rollout-workers must be >= 1"),
        (args.rollout_batch_size < 1, "--rollout-batch-size must be >= 1"),
        (args.rollout_stop_timeout <= 0, "--rollout-stop-timeout must be > 0"),
        (args.vllm_max_num_seqs < 1, "--vllm-max-num-seqs must be >= 1"),
        (args.vllm_max_num_batched_tokens < 1, "--vllm-max-num-batched-tokens must be >= 1"),
        (args.max_sync_rounds is not None and args.max_sync_rounds < 0, "--max-sync-rounds must be >= 0 when set"),
    ]
    for bad, msg in checks:
        if bad:
            raise ValueError(msg)


def to_runtime_args(g: argparse.Namespace) -> argparse.Namespace:
    """The shared runtime's namespace (TextWorld loop defaults) carrying this variant's settings."""
    args = build_agent_parser().parse_args(["--model-path", g.model_path])
    for k, v in vars(g).items():
        setattr(args, k, v)
    args.env = "gsm8k"
    args.rl_algorithm = "grpo"
    args.train_packing = "padded"
    args.grpo_group_size = g.rollout_batch_size
    args.lr_schedule = "constant"
    args.lr_warmup_steps = 0
    args.old_new_kl_coef = 0.0
    args.infer_tp_size = 1
    args.vllm_max_model_len = None
    args.min_replay_size_per_rank = None
    args.train_pack_candidate_pool_size = None
    args.num_rollout_workers = g.num_rollout_workers
    args.checkpoint_every_sync_rounds = 0
    args = finalize_args(args)
    # finalize_args derives the TextWorld log dir; keep this variant's
    args.log_dir = g.log_dir
    return args


def main(argv: Optional[List[str]] = None) -> None:
    g = parse_args(argv)
    validate_args(g)
    from .agent_textworld import run_train

    run_train(to_runtime_args(g))


if __name__ == "__main__":
    main()
