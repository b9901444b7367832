"""Command-line surface of the ``agent_textworld`` entry point.

Every flag of the reference (agent_textworld.py:3361-3815) is accepted with the same name, default and
derived default, and ``validate_args`` applies the same rules (agent_textworld.py:3818-3950). Additions
of this framework are grouped at the end: ``--env synthetic`` (a seeded token-level text game that
needs no game files), ``--synthetic-*`` shape knobs, ``--device``, and the engine's KV-cache sizing.
``--model-path`` also accepts a preset name (``qwen2.5-1.5b``, ``qwen1.5-moe-a2.7b``, ``qwen3-8b``,
``qwen3-30b-a3b``, ``tiny-qwen2``) for random-init runs of those shapes.
"""

from __future__ import annotations

import argparse
import os
import time
from typing import List, Optional


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(
        description="Asynchronous online RL for LLM agents on B200: sharded trainer + native paged-KV rollout engine."
    )
    a = p.add_argument
    a("--model-path", required=True, help="Local HF model directory, or a preset name for a random-init model.")
    a("--dtype", default="auto", choices=("auto", "bfloat16", "float16", "float32"))
    a("--train-mode", default="full", choices=("lm_head", "last_layer", "full"))
    a("--tw-game-dir", default=None, help="Directory containing TextWorld .z8 games (required with --env textworld).")
    a("--tw-game-pattern", default="*.z8")
    a("--tw-game-limit", type=int, default=None)
    a("--tw-max-episode-steps", type=int, default=20)
    a("--tw-history-token-window", type=int, default=2048)
    a("--rl-algorithm", type=str, default="grpo", choices=("ppo", "grpo"))
    a("--tw-gamma", type=float, default=1.0)
    a("--tw-step-penalty", type=float, default=0.0)
    a("--tw-win-bonus", type=float, default=1.0)
    a("--tw-lost-penalty", type=float, default=0.0)
    a("--tw-invalid-action-penalty", type=float, default=0.0)
    a("--grpo-group-size", type=int, default=None)
    a("--grpo-adv-eps", type=float, default=1e-8)
    a("--max-length", type=int, default=2048)
    a("--batch-size", type=int, default=16)
    a("--train-packing", choices=["padded", "varlen"], default="padded")
    a("--train-token-budget", type=int, default=None)
    a("--train-pack-candidate-pool-size", type=int, default=None)
    a("--max-steps", type=int, default=5000)
    a("--learning-rate", type=float, default=1e-6)
    a("--lr-warmup-steps", type=int, default=500)
    a("--weight-decay", type=float, default=0.0)
    a("--grad-accum-steps", type=int, default=8)
    a("--train-logprob-mode", type=str, default="full_logits_ce", choices=["full_logits_ce", "response_only_lm_head"])
    a("--clip-mode", type=str, default="ppo", choices=["ppo", "gipo", "sapo", "none"])
    a("--ppo-normalize-advantages", action="store_true")
    a("--ppo-adv-norm-eps", type=float, default=1e-8)
    a("--clip-eps", type=float, default=0.2)
    a("--old-new-kl-coef", type=float, default=0.0)
    a("--gipo-sigma", type=float, default=1.0)
    a("--sapo-tau-pos", type=float, default=1.0)
    a("--sapo-tau-neg", type=float, default=2.0)
    a("--replay-capacity", type=int, default=None)
    a("--replay-wait-sleep-seconds", type=float, default=0.2)
    a("--replay-sample-timeout-seconds", type=float, default=None)
    a("--min-replay-size-per-rank", type=int, default=None)
    a("--log-every", type=int, default=1)
    a("--metrics-window-size", type=int, default=1000)
    a("--metrics-active-timeout-seconds", type=float, default=600.0)
    a("--log-dir", default=None)
    a("--save-checkpoint", action="store_true")
    a("--checkpoint-dir", default=None)
    a("--checkpoint-name", default="latest")
    a("--checkpoint-every-sync-rounds", type=int, default=0)
    a("--save-optimizer-state", action="store_true",
      help="Also save each rank's optimizer shard (fp32 master, Adam moments) and step counters.")
    a("--resume-from", default=None, help="Checkpoint directory to resume the trainer from.")
    a("--seed", type=int, default=42)
    a("--trust-remote-code", action="store_true")
    a("--gradient-checkpointing", action="store_true")
    a("--fsdp-world-size", type=int, default=6)
    a("--fsdp-master-addr", default=None)
    a("--fsdp-master-port", type=int, default=None)
    a("--ray-address", default=None, help="Accepted for command-line compatibility; this runtime does not use Ray.")
    a("--sync-every-optimizer-steps", type=int, default=8)
    a("--infer-size", type=int, default=2, help="Rollout engine data-parallel size (independent engines).")
    a("--infer-tp-size", type=int, default=1, help="Rollout engine tensor-parallel size.")
    a("--infer-max-tokens", type=int, default=16)
    a("--infer-temperature", type=float, default=1.0)
    a("--infer-top-p", type=float, default=1.0)
    a("--num-rollout-workers", type=int, default=None)
    a("--rollout-batch-size", type=int, default=8)
    a("--rollout-stop-timeout", type=float, default=10.0)
    a("--vllm-max-num-seqs", type=int, default=128, help="Maximum concurrently scheduled sequences per engine.")
    a("--vllm-max-num-batched-tokens", type=int, default=8192, help="Maximum tokens per engine step.")
    a("--vllm-max-model-len", type=int, default=None)
    a("--disable-vllm-prefix-caching", action="store_true")
    a("--max-sync-rounds", type=int, default=None)
    # ---- additions of this framework
    a("--env", default="textworld", choices=("textworld", "synthetic", "gsm8k"))
    a("--lr-schedule", default="warmup_cosine", choices=("warmup_cosine", "constant"))
    a("--gsm8k-train-path", default="synthetic",
      help="GSM8K train jsonl for --env gsm8k; 'synthetic' uses seeded arithmetic word problems.")
    a("--gsm8k-limit", type=int, default=None)
    a("--synthetic-obs-min", type=int, default=64)
    a("--synthetic-obs-max", type=int, default=256)
    a("--synthetic-reward-prob", type=float, default=0.1)
    a("--synthetic-end-prob", type=float, default=0.02)
    a("--device", default="auto", help="auto | cpu | cuda")
    a("--kv-cache-gb", type=float, default=None, help="KV cache size per rollout GPU (default: 60%% of free memory).")
    a("--kv-block-size", type=int, default=16)
    a("--shard-params", action="store_true",
      help="Shard parameters, gradients and optimizer state over the FSDP ranks per decoder layer "
           "(all-gathered before each layer's forward and backward, gradients reduce-scattered after "
           "it, as FSDP full sharding does); for models whose compute copy does not fit on every rank.")
    a("--expert-parallel", action="store_true",
      help="MoE models: partition the experts over the trainer ranks (token dispatch/combine over NVLink).")
    a("--expert-storage", default="partitioned", choices=("partitioned", "replicated"),
      help="With --expert-parallel: each rank stores only its routed experts (weights, gradients, optimizer "
           "state), or every rank keeps the whole expert stack.")
    a("--weight-sync", default="ipc", choices=("ipc", "nccl"), help="Trainer->rollout weight transfer path.")
    a("--rollout-worker-procs", type=int, default=None,
      help="Processes that run each engine's rollout workers (default: one per worker; 0: the workers run as "
           "asyncio tasks inside the engine process).")
    a("--no-balance-packs", dest="balance_packs", action="store_false",
      help="Varlen training: compute every pack on the rank that drew it instead of spreading each "
           "optimizer window's packs over the trainer ranks by estimated work.")
    return p


def finalize_args(args: argparse.Namespace) -> argparse.Namespace:
    """Derived defaults, exactly as the reference computes them (agent_textworld.py:3797-3814)."""
    if args.clip_eps <= 0:
        raise ValueError(f"--clip-eps must be > 0, got {args.clip_eps}")
    if args.old_new_kl_coef < 0:
        raise ValueError(f"--old-new-kl-coef must be >= 0, got {args.old_new_kl_coef}")
    if args.gipo_sigma <= 0:
        raise ValueError(f"--gipo-sigma must be > 0, got {args.gipo_sigma}")
    if args.sapo_tau_pos <= 0 or args.sapo_tau_neg <= 0:
        raise ValueError(
            f"--sapo-tau-pos and --sapo-tau-neg must be > 0, got {args.sapo_tau_pos}, {args.sapo_tau_neg}"
        )
    if args.replay_capacity is None:
        args.replay_capacity = args.batch_size * args.grad_accum_steps * 4
    if args.train_pack_candidate_pool_size is None:
        args.train_pack_candidate_pool_size = args.batch_size * 4
    if args.replay_sample_timeout_seconds is None:
        args.replay_sample_timeout_seconds = 0.0
    if args.min_replay_size_per_rank is None:
        args.min_replay_size_per_rank = args.batch_size
    if args.num_rollout_workers is None:
        args.num_rollout_workers = args.fsdp_world_size
    if args.grpo_group_size is None:
        args.grpo_group_size = args.rollout_batch_size
    if args.log_dir is None:
        args.log_dir = os.path.join("runs", "TextWorld_FSDP", time.strftime("%Y-%m-%d_%H-%M-%S"))
    if args.checkpoint_dir is None:
        args.checkpoint_dir = os.path.join(args.log_dir, "checkpoints")
    return args


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    return finalize_args(build_parser().parse_args(argv))


def validate_args(args: argparse.Namespace, check_games: bool = True) -> None:
    if args.train_packing == "varlen" and args.ppo_normalize_advantages:
        raise ValueError(
            "--ppo-normalize-advantages is not supported with --train-packing varlen because the Varlen "
            "baseline uses a global valid-response-token weighted objective."
        )
    if args.tw_game_limit is not None and args.tw_game_limit < 1:
        raise ValueError("--tw-game-limit must be >= 1 when set")
    if args.tw_max_episode_steps < 1:
        raise ValueError("--tw-max-episode-steps must be >= 1")
    if args.tw_history_token_window < 1:
        raise ValueError("--tw-history-token-window must be >= 1")
    if args.tw_gamma < 0:
        raise ValueError("--tw-gamma must be >= 0")
    if args.max_length < args.tw_history_token_window:
        raise ValueError(
            "--max-length must be >= --tw-history-token-window when TextWorld token-window transcript mode is enabled"
        )
    if args.env == "textworld" and check_games:
        if not args.tw_game_dir:
            raise ValueError("--tw-game-dir is required with --env textworld")
        from ..env.textworld import load_game_files

        load_game_files(args.tw_game_dir, args.tw_game_pattern, args.seed, args.tw_game_limit)
    if args.grad_accum_steps < 1:
        raise ValueError("--grad-accum-steps must be >= 1")
    if args.max_steps < 1:
        raise ValueError("--max-steps must be >= 1")
    if args.learning_rate < 0:
        raise ValueError("--learning-rate must be >= 0")
    if args.lr_warmup_steps < 0:
        raise ValueError("--lr-warmup-steps must be >= 0")
    if args.batch_size < 1:
        raise ValueError("--batch-size must be >= 1")
    if args.train_pack_candidate_pool_size < 1:
        raise ValueError("--train-pack-candidate-pool-size must be >= 1")
    if args.train_packing == "varlen":
        if args.train_token_budget is None:
            raise ValueError("--train-token-budget is required with --train-packing varlen")
        if args.train_token_budget < args.max_length:
            raise ValueError(
                "--train-token-budget must be >= --max-length in varlen mode; "
                f"got {args.train_token_budget} < {args.max_length}"
            )
        if args.dtype == "float32":
            raise ValueError("varlen training requires float16, bfloat16, or auto dtype")
    elif args.train_token_budget is not None and args.train_token_budget < 1:
        raise ValueError("--train-token-budget must be >= 1 when set")
    if args.train_logprob_mode == "response_only_lm_head" and args.train_packing != "varlen":
        raise ValueError(
            "--train-logprob-mode response_only_lm_head requires --train-packing varlen so tensor "
            "logits_to_keep can address per-sample prediction positions"
        )
    if args.replay_capacity < 1:
        raise ValueError("--replay-capacity must be >= 1")
    if args.min_replay_size_per_rank < 1:
        raise ValueError("--min-replay-size-per-rank must be >= 1")
    if args.min_replay_size_per_rank > args.replay_capacity:
        raise ValueError(
            "--min-replay-size-per-rank must be <= --replay-capacity; "
            f"got {args.min_replay_size_per_rank} > {args.replay_capacity}"
        )
    if args.replay_wait_sleep_seconds <= 0:
        raise ValueError("--replay-wait-sleep-seconds must be > 0")
    if args.replay_sample_timeout_seconds < 0:
        raise ValueError("--replay-sample-timeout-seconds must be >= 0")
    if args.max_length < 1:
        raise ValueError("--max-length must be >= 1")
    if args.log_every < 1:
        raise ValueError("--log-every must be >= 1")
    if args.metrics_window_size < 1:
        raise ValueError("--metrics-window-size must be >= 1")
    if args.metrics_active_timeout_seconds <= 0:
        raise ValueError("--metrics-active-timeout-seconds must be > 0")
    if args.checkpoint_every_sync_rounds < 0:
        raise ValueError("--checkpoint-every-sync-rounds must be >= 0")
    if args.fsdp_world_size < 1:
        raise ValueError("--fsdp-world-size must be >= 1")
    if args.sync_every_optimizer_steps < 1:
        raise ValueError("--sync-every-optimizer-steps must be >= 1")
    if args.infer_size < 1:
        raise ValueError("--infer-size must be >= 1")
    if args.infer_tp_size < 1:
        raise ValueError("--infer-tp-size must be >= 1")
    if args.infer_max_tokens < 1:
        raise ValueError("--infer-max-tokens must be >= 1")
    if args.infer_temperature < 0.0:
        raise ValueError("--infer-temperature must be >= 0")
    if not 0.0 < args.infer_top_p <= 1.0:
        raise ValueError("--infer-top-p must be in (0, 1]")
    if args.num_rollout_workers < 1:
        raise ValueError("--num-rollout-workers must be >= 1")
    if args.num_rollout_workers < args.fsdp_world_size:
        raise ValueError(
            "TextWorld training requires --num-rollout-workers >= --fsdp-world-size so every trainer replay "
            f"buffer receives samples; got num_rollout_workers={args.num_rollout_workers}, "
            f"fsdp_world_size={args.fsdp_world_size}"
        )
    if args.rollout_batch_size < 1:
        raise ValueError("--rollout-batch-size must be >= 1")
    if args.grpo_group_size < 1:
        raise ValueError("--grpo-group-size must be >= 1")
    if args.grpo_adv_eps <= 0:
        raise ValueError("--grpo-adv-eps must be > 0")
    if args.ppo_adv_norm_eps <= 0:
        raise ValueError("--ppo-adv-norm-eps must be > 0")
    if args.tw_invalid_action_penalty < 0:
        raise ValueError("--tw-invalid-action-penalty must be >= 0")
    if args.tw_lost_penalty < 0:
        raise ValueError("--tw-lost-penalty must be >= 0")
    if args.rollout_stop_timeout <= 0:
        raise ValueError("--rollout-stop-timeout must be > 0")
    if args.vllm_max_num_seqs < 1:
        raise ValueError("--vllm-max-num-seqs must be >= 1")
    if args.vllm_max_num_batched_tokens < 1:
        raise ValueError("--vllm-max-num-batched-tokens must be >= 1")
    if args.vllm_max_model_len is not None and args.vllm_max_model_len < 1:
        raise ValueError("--vllm-max-model-len must be >= 1 when set")
    if args.max_sync_rounds is not None and args.max_sync_rounds < 0:
        raise ValueError("--max-sync-rounds must be >= 0 when set")


def make_args(**overrides) -> argparse.Namespace:
    """Programmatic construction with the CLI defaults (tests, benchmarks)."""
    argv: List[str] = ["--model-path", str(overrides.pop("model_path", "tiny-qwen2"))]
    args = build_parser().parse_args(argv)
    for k, v in overrides.items():
        if not hasattr(args, k):
            raise AttributeError(f"unknown option {k}")
        setattr(args, k, v)
    return finalize_args(args)
