"""Inference process actor: one generation engine (one GPU) plus the rollout workers it serves.

Rollout workers run in their own processes by default (``--rollout-worker-procs``, one per worker
as the reference's actors do) and send their requests over a Unix socket (``rollout/remote.py``);
with ``--rollout-worker-procs 0`` they are asyncio tasks inside the engine process. Either way they
push finished samples to the sample queue of trainer rank ``worker_id % fsdp_world_size`` and
episode records to the driver's statistics queue.
"""

from __future__ import annotations

import asyncio
import os
from typing import Any, Dict, List, Optional

import torch


class InferenceActor:
    def __init__(self, args, device_index: Optional[int], worker_ids: List[int], replay_queues, stats_queue,
                 tp_port: Optional[int] = None):
        """Rank 0 of an engine. With ``--infer-tp-size`` > 1 the other ranks are ``InferenceFollower``
        actors joined through ``tp_port``; this rank schedules and broadcasts every step."""
        from ..trainer.actor import _load_tokenizer
        from .inference import InferenceService

        if device_index is not None and torch.cuda.is_available():
            device = torch.device("cuda", device_index)
            torch.cuda.set_device(device)
        else:
            device = torch.device("cpu")
        self.args = args
        if args.env == "textworld":
            tokenizer = _load_tokenizer(args)
        elif args.env == "gsm8k":
            from ..core.tokenizer import load_tokenizer
            from ..models.config import resolve_model_config

            tokenizer = load_tokenizer(args.model_path, args.trust_remote_code,
                                       vocab_size=resolve_model_config(args.model_path).vocab_size, fallback=True)
        else:
            tokenizer = None
        tp_groups = None
        if getattr(args, "infer_tp_size", 1) > 1:
            from .inference import init_tp_groups

            tp_groups = init_tp_groups(0, args.infer_tp_size, tp_port, device)
        self.service = InferenceService(args, device, tokenizer=tokenizer, tp_groups=tp_groups)
        procs = getattr(args, "rollout_worker_procs", None)
        procs = len(worker_ids) if procs is None else int(procs)
        self.remote = None
        self.workers: List[Any] = []
        if procs > 0 and worker_ids:
            from .remote import WorkerProcesses

            self.remote = WorkerProcesses(args, self.service, list(worker_ids), replay_queues, stats_queue,
                                          min(procs, len(worker_ids)))
        else:
            from .remote import make_workers

            self.workers = make_workers(args, self.service, list(worker_ids), replay_queues, stats_queue, tokenizer)
        self.tasks: List[asyncio.Task] = []

    async def start_workers(self) -> int:
        if self.remote is not None:
            return await self.remote.start()
        self.tasks = [asyncio.create_task(w.run()) for w in self.workers]
        return len(self.tasks)

    async def check_workers(self) -> Optional[str]:
        """None while every worker runs; otherwise a description of the first one that exited."""
        if self.remote is not None:
            return self.remote.check()
        for w, t in zip(self.workers, self.tasks):
            if t.done():
                exc = t.exception()
                return f"rollout worker {w.worker_id} exited: {exc!r}" if exc else f"rollout worker {w.worker_id} exited"
        return None

    async def stop_workers(self, timeout: float) -> Dict[str, int]:
        if self.remote is not None:
            return await self.remote.stop(timeout)
        for w in self.workers:
            await w.stop()
        done, pending = await asyncio.wait(self.tasks, timeout=timeout) if self.tasks else (set(), set())
        for t in pending:
            t.cancel()
        return {"stopped": len(done), "cancelled": len(pending)}

    async def pause_and_wait_idle(self) -> None:
        await self.service.pause_and_wait_idle()

    async def resume_generation(self, increment_version: bool = False) -> int:
        return await self.service.resume_generation(increment_version)

    def attach_trainer_weights(self, handle) -> int:
        return self.service.attach_trainer_weights(handle)

    def pull_weights(self, scope: Any = "all") -> Dict[str, float]:
        return self.service.pull_weights(scope)

    def get_stats(self) -> Dict[str, Any]:
        return self.service.get_stats()

    async def shutdown(self) -> Dict[str, Any]:
        if self.remote is not None and self.remote.procs:
            await self.remote.stop(1.0)
        for w in self.workers:
            await w.stop()
        for t in self.tasks:
            if not t.done():
                t.cancel()
        return await self.service.shutdown()


class InferenceFollower:
    """Rank > 0 of a tensor-parallel engine: holds its weight and KV-cache shards and replays the
    steps, weight pulls and cache commands broadcast by rank 0 on a background thread."""

    def __init__(self, args, device_index: Optional[int], tp_rank: int, tp_port: int):
        import threading

        from .inference import build_engine, init_tp_groups

        if device_index is not None and torch.cuda.is_available():
            device = torch.device("cuda", device_index)
            torch.cuda.set_device(device)
        else:
            device = torch.device("cpu")
        self.args = args
        self.device = device
        groups = init_tp_groups(tp_rank, args.infer_tp_size, tp_port, device)
        self.engine = build_engine(args, device, tp_groups=groups)
        self._ipc_bases: List[int] = []
        self.error: Optional[str] = None
        self._thread = threading.Thread(target=self._serve, name="tp-follower", daemon=True)
        self._thread.start()

    def _serve(self) -> None:
        try:
            self.engine.serve_follower()
        except BaseException as exc:  # reported through check()
            self.error = repr(exc)

    def attach_trainer_weights(self, handle) -> int:
        from .inference import attach_weight_source

        return attach_weight_source(self.engine, self.args, self.device, handle, self._ipc_bases)

    def check(self) -> Optional[str]:
        if self.error:
            return self.error
        return None if self._thread.is_alive() else "follower loop exited"

    def shutdown(self, timeout: float = 60.0) -> bool:
        """Wait for the loop to end (rank 0 sends the stop command when it shuts down)."""
        self._thread.join(timeout)
        return not self._thread.is_alive()
