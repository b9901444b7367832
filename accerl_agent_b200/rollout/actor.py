"""Inference process actor: one generation engine (one GPU) plus the rollout workers it serves.

Rollout workers are asyncio tasks in the same process as the engine, so a request costs no
inter-process hop; they push finished samples to the sample queue of trainer rank
``worker_id % fsdp_world_size`` and episode records to the driver's statistics queue.
"""

from __future__ import annotations

import asyncio
import os
from typing import Any, Dict, List, Optional

import torch


class InferenceActor:
    def __init__(self, args, device_index: Optional[int], worker_ids: List[int], replay_queues, stats_queue):
        from ..trainer.actor import _load_tokenizer
        from .inference import InferenceService
        from .worker import RolloutWorker

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
        self.service = InferenceService(args, device, tokenizer=tokenizer)
        world = len(replay_queues)

        def sink_for(wid):
            q = replay_queues[wid % world]
            return lambda samples: q.put(samples)

        def stats_sink(*rec):
            stats_queue.put(rec)

        if args.env == "gsm8k":
            from .math_worker import MathRolloutWorker, load_math_examples

            examples = load_math_examples(args)
            self.workers = [MathRolloutWorker(args, self.service, wid, sink_for(wid), stats_sink, tokenizer=tokenizer,
                                              examples=examples) for wid in worker_ids]
        else:
            self.workers = [RolloutWorker(args, self.service, wid, sink_for(wid), stats_sink, tokenizer=tokenizer)
                            for wid in worker_ids]
        self.tasks: List[asyncio.Task] = []

    async def start_workers(self) -> int:
        self.tasks = [asyncio.create_task(w.run()) for w in self.workers]
        return len(self.tasks)

    async def check_workers(self) -> Optional[str]:
        """None while every worker runs; otherwise a description of the first one that exited."""
        for w, t in zip(self.workers, self.tasks):
            if t.done():
                exc = t.exception()
                return f"rollout worker {w.worker_id} exited: {exc!r}" if exc else f"rollout worker {w.worker_id} exited"
        return None

    async def stop_workers(self, timeout: float) -> Dict[str, int]:
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

    def pull_weights(self, numel: Optional[int] = None) -> Dict[str, float]:
        return self.service.pull_weights(numel)

    def get_stats(self) -> Dict[str, Any]:
        return self.service.get_stats()

    async def shutdown(self) -> Dict[str, Any]:
        for w in self.workers:
            await w.stop()
        for t in self.tasks:
            if not t.done():
                t.cancel()
        return await self.service.shutdown()
