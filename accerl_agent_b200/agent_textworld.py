"""Asynchronous online RL for text-game agents: the driver.

    python -m accerl_agent_b200.agent_textworld --model-path <hf dir | preset> [--env synthetic] ...

Same flags and loop as the reference entry point (agent_textworld.py:2931-3358):

1. start ``fsdp_world_size`` trainer processes (one GPU each, one replay shard each) and
   ``infer_size`` generation-engine processes on the following GPUs;
2. map trainer parameters into every engine (CUDA IPC) and run the initial full weight sync
   (scope ``all``, version stays 0); start the rollout workers (``worker_id % world`` picks the
   replay shard);
3. loop: every trainer runs ``train_until_next_sync(sync_every_optimizer_steps)`` while rollouts keep
   going; metrics go to TensorBoard and ``metrics.jsonl``; optional checkpoint; then every engine
   pauses (aborting in-flight requests, which resume later with their partial tokens), pulls the
   trainable parameter range straight from trainer memory, and resumes with the version incremented;
4. stop on ``max_steps`` / ``max_sync_rounds``; stop workers, final checkpoint, clean shutdown.

A rollout worker or engine process that dies is fatal, as in the reference.
"""

from __future__ import annotations

import os
import queue as pyqueue
import socket
import sys
import time
from typing import Dict, List, Optional

from .core.config import parse_args, validate_args
from .core.run_io import MetricsWriter, checkpoint_tag, save_run_config
from .replay import RolloutStats
from .runtime.actors import ActorDied, get, spawn_actor


def find_open_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def device_plan(args):
    """GPU indices of trainer ranks and engines (None entries mean CPU)."""
    import torch

    use_cuda = args.device != "cpu" and torch.cuda.is_available()
    world = args.fsdp_world_size
    n_engines = args.infer_size
    tp = args.infer_tp_size
    if not use_cuda:
        return [None] * world, [[None] * tp for _ in range(n_engines)]
    need = world + n_engines * tp
    have = torch.cuda.device_count()
    if have < need:
        raise RuntimeError(f"need {need} GPUs (fsdp_world_size + infer_tp_size * infer_size), found {have}")
    return list(range(world)), [[world + i * tp + j for j in range(tp)] for i in range(n_engines)]


def exchange_weight_handles(trainers, engines, followers, timeout: float = 600.0) -> None:
    """Hand every engine rank (leader and tensor-parallel followers) the weight-buffer handle of
    trainer ``i % world``, once at start-up; later syncs pull through the mapped buffers. A trainer
    or engine process that died before or during the exchange raises ``ActorDied`` here (the
    reference builds its NCCL weight-transfer group at this point, ``agent_textworld.py:3035-3057``)."""
    handles = None
    for i, e in enumerate(engines):
        handle = get(trainers[i % len(trainers)].export_weights_handle.remote(), timeout=timeout)
        if isinstance(handle, dict) and (handle.get("partition") or handle.get("zero3")):
            # expert-partitioned or layer-sharded trainers: every engine rank maps every trainer
            if handles is None:
                handles = get([t.export_weights_handle.remote() for t in trainers], timeout=timeout)
            handle = handles
        e.attach_trainer_weights(handle)
        for f in followers[i] if followers else ():
            f.attach_trainer_weights(handle)


def sync_weights(engines, trainers, scope: str) -> Dict[str, float]:
    numel = get(trainers[0].weight_numel.remote(scope))
    for t in trainers:
        t.synchronize()
    t0 = time.perf_counter()
    results = get([e.pull_weights.remote(scope) for e in engines])
    elapsed = time.perf_counter() - t0
    nbytes = sum(r["bytes"] for r in results)
    dev_ms = max(r["device_ms"] for r in results)
    print(f"[sync] {scope}: {numel * 2 / 1024**3:.3f} GiB per engine x {len(engines)} in {elapsed:.4f}s "
          f"(device max {dev_ms:.2f} ms, aggregate {nbytes / max(elapsed, 1e-9) / 1024**3:.2f} GiB/s)")
    return {"elapsed_s": elapsed, "device_ms": dev_ms, "bytes": nbytes}


def check_rollout_side(engines, followers) -> None:
    """Raise if a rollout worker, an engine process or a tensor-parallel engine rank has failed."""
    for e in engines:
        if not e.alive:
            raise RuntimeError("an inference engine process exited")
        err = get(e.check_workers.remote(), timeout=60)
        if err:
            raise RuntimeError(f"A rollout worker exited unexpectedly: {err}")
    for fs in followers:
        for f in fs:
            err = f.check()
            if err:
                raise RuntimeError(f"A tensor-parallel engine rank failed: {err}")


def _await_training(pending, engines, followers, poll_s: float = 5.0):
    """Results of the trainers' segment calls. While they run, the rollout side is checked every
    ``poll_s`` seconds: trainers waiting for samples from a dead engine would otherwise wait forever."""
    import concurrent.futures as cf

    while True:
        _, rest = cf.wait(pending, timeout=poll_s, return_when=cf.ALL_COMPLETED)
        if not rest:
            return get(pending)
        check_rollout_side(engines, followers)


def run_train(args) -> Dict[str, float]:
    import multiprocessing as mp

    save_run_config(args)
    writer = MetricsWriter(args.log_dir)
    trainer_devs, engine_devs = device_plan(args)
    world = args.fsdp_world_size
    ctx = mp.get_context("spawn")
    replay_queues = [ctx.Queue() for _ in range(world)]
    stats_queue = ctx.Queue()
    stats = RolloutStats(args.metrics_window_size, args.metrics_active_timeout_seconds)
    addr = args.fsdp_master_addr or "127.0.0.1"
    port = args.fsdp_master_port or find_open_port()
    trainers, engines = [], []
    followers: List[List] = []
    final: Dict[str, float] = {}
    try:
        trainers = [spawn_actor("accerl_agent_b200.trainer.actor:TrainerActor", args, r, world, addr, port,
                                replay_queues[r], trainer_devs[r], name=f"trainer{r}", ready_timeout=None)
                    for r in range(world)]
        for t in trainers:
            t.wait_ready(1800)
        print(f"[init] {world} trainer ranks ready.")
        assignment: List[List[int]] = [[] for _ in engine_devs]
        for wid in range(args.num_rollout_workers):
            assignment[wid % len(engine_devs)].append(wid)
        tp_ports = [find_open_port() for _ in engine_devs]
        engines = [spawn_actor("accerl_agent_b200.rollout.actor:InferenceActor", args, engine_devs[i][0], assignment[i],
                               replay_queues, stats_queue, tp_ports[i], name=f"engine{i}", ready_timeout=None)
                   for i in range(len(engine_devs))]
        followers = [[spawn_actor("accerl_agent_b200.rollout.actor:InferenceFollower", args, engine_devs[i][j], j,
                                  tp_ports[i], name=f"engine{i}-tp{j}", ready_timeout=None)
                      for j in range(1, args.infer_tp_size)] for i in range(len(engine_devs))]
        for e in engines + [f for fs in followers for f in fs]:
            e.wait_ready(1800)
        exchange_weight_handles(trainers, engines, followers)
        print("[sync] Initial full sync from trainers to engines...")
        get([e.pause_and_wait_idle.remote() for e in engines])
        sync_weights(engines, trainers, "all")
        get([e.resume_generation.remote(False) for e in engines])
        get([e.start_workers.remote() for e in engines])
        print(f"[rollout] {args.num_rollout_workers} rollout workers started on {len(engines)} engine(s).")

        sync_rounds = 0
        latest_step = 0
        last_ckpt = None
        reached_max = False
        while not reached_max:
            check_rollout_side(engines, followers)
            infer_start = sum(s["total_tokens"] for s in get([e.get_stats.remote() for e in engines]))
            t0 = time.perf_counter()
            pending = [t.train_until_next_sync.remote(args.sync_every_optimizer_steps) for t in trainers]
            summaries = _await_training(pending, engines, followers)
            elapsed = time.perf_counter() - t0
            infer_end = sum(s["total_tokens"] for s in get([e.get_stats.remote() for e in engines]))
            while True:
                try:
                    stats.add_record(*stats_queue.get_nowait())
                except pyqueue.Empty:
                    break
            r0 = next(s for s in summaries if s["rank"] == 0)
            reached_max = bool(r0["reached_max_steps"])
            latest_step = int(r0["optimizer_step"])
            if r0["optimizer_steps_run"] <= 0:
                break
            replay = get([t.get_replay_stats.remote() for t in trainers])
            rs = stats.get_stats()
            n = len(summaries)
            tokens = (float(r0["segment_valid_tokens"]) if args.train_packing == "varlen"
                      else sum(float(s["segment_valid_tokens"]) for s in summaries))
            if args.env == "gsm8k":
                env_scal = {
                    "Rollout/GlobalRewardSumMean": rs["global_reward_sum_mean"],
                    "Rollout/ResponseLengthMean": rs["response_length_mean"],
                    "Rollout/AbortRate": rs["abort_rate"],
                }
                score = rs["global_reward_sum_mean"]
            else:
                env_scal = {
                    "TextWorld/NormalizedScore": rs["tw_normalized_score"],
                    "TextWorld/WinRate": rs["tw_win_rate"],
                    "TextWorld/InvalidActionRate": rs["tw_invalid_action_rate"],
                    "TextWorld/EnvStepsMean": rs["tw_env_steps_mean"],
                }
                score = rs["tw_normalized_score"]
            scal = {
                **env_scal,
                "Train/OptimizerStep": latest_step,
                "Replay/FillRatio": sum(r["size"] for r in replay) / max(sum(r["capacity"] for r in replay), 1),
                "Replay/TrainSampleTrainerVersionLagMean": sum(s["segment_version_lag_mean"] for s in summaries) / n,
                "Rollout/ActiveWorkers": rs["active_workers"],
                "Train/Loss": sum(s["segment_loss_mean"] for s in summaries) / n,
                "Train/LossMeanAcrossRanks": sum(s["segment_loss_mean"] for s in summaries) / n,
                "KL/OldNewK3TokenMean": sum(s["segment_kl_mean"] for s in summaries) / n,
                "Train/LearningRate": r0["learning_rate"],
                "Train/TokensPerSec": tokens / max(elapsed, 1e-9),
                "Train/OptimizerStepsPerSec": r0["optimizer_steps_run"] / max(elapsed, 1e-9),
                "Infer/TokensPerSec": (infer_end - infer_start) / max(elapsed, 1e-9),
                "Train/PackTokenUtilization": r0.get("pack_token_utilization"),
                "Train/PackSampleCount": r0.get("pack_sample_count"),
                "Train/PackMaxSequenceLength": r0.get("pack_max_sequence_length"),
                "Train/PackCpuMilliseconds": r0.get("pack_cpu_ms"),
            }
            if args.clip_mode == "ppo":
                scal["Clip/PPOClipFrac"] = sum(s["segment_clip_frac"] for s in summaries) / n
            writer.add_scalars(scal, latest_step)
            print(f"[metrics] step={latest_step} loss={scal['Train/Loss']:.6f} kl={scal['KL/OldNewK3TokenMean']:.6f} "
                  f"train_tokens_per_sec={scal['Train/TokensPerSec']:.2f} "
                  f"infer_tokens_per_sec={scal['Infer/TokensPerSec']:.2f} score={score:.4f}")
            writer.flush()
            final = dict(scal)
            if args.save_checkpoint and args.checkpoint_every_sync_rounds > 0 and \
                    (sync_rounds + 1) % args.checkpoint_every_sync_rounds == 0:
                tag = args.checkpoint_name or checkpoint_tag(latest_step)
                get([t.save_checkpoint.remote(args.checkpoint_dir, tag) for t in trainers])
                last_ckpt = latest_step
            if args.max_sync_rounds is not None and sync_rounds >= args.max_sync_rounds:
                print("[sync] max_sync_rounds reached; letting inference finish without more trainable updates.")
                break
            sync_rounds += 1
            get([e.pause_and_wait_idle.remote() for e in engines])
            s = sync_weights(engines, trainers, "trainable")
            writer.add_scalars({"Sync/ElapsedSeconds": s["elapsed_s"], "Sync/DeviceMilliseconds": s["device_ms"]},
                               latest_step)
            final["Sync/ElapsedSeconds"] = s["elapsed_s"]
            version = get([e.resume_generation.remote(True) for e in engines])[0]
            print(f"[sync] Round {sync_rounds}: resumed generation with weight version {version}.")
        print("[rollout] Trainer finished or sync loop stopped; stopping rollout workers.")
        get([e.stop_workers.remote(args.rollout_stop_timeout) for e in engines])
        if args.save_checkpoint and latest_step > 0 and last_ckpt != latest_step:
            tag = args.checkpoint_name or checkpoint_tag(latest_step, "final")
            get([t.save_checkpoint.remote(args.checkpoint_dir, tag) for t in trainers])
    finally:
        for e in engines:
            try:
                get(e.method("shutdown").remote(), timeout=60)
            except Exception as exc:
                print(f"[cleanup] Ignoring engine shutdown error: {exc!r}")
            e.stop_process()
        for fs in followers:
            for f in fs:
                try:
                    get(f.shutdown.remote(30), timeout=60)
                except Exception as exc:
                    print(f"[cleanup] Ignoring engine follower shutdown error: {exc!r}")
                f.stop_process()
        # every trainer rank leaves its process group at the same time: destroying the group waits
        # for the other ranks, so closing them one after another would wait out each timeout
        try:
            get([t.close.remote() for t in trainers], timeout=60)
        except Exception as exc:
            print(f"[cleanup] Ignoring trainer close error: {exc!r}")
        for t in trainers:
            t.stop_process()
        writer.close()
    return final


def main(argv: Optional[List[str]] = None) -> None:
    args = parse_args(argv)
    validate_args(args, check_games=args.env == "textworld")
    run_train(args)


if __name__ == "__main__":
    main()
