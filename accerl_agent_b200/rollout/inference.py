"""Inference service: the reference's ``VLLMInferenceActor`` surface (agent_textworld.py:1916-2060)
over the native engine, plus the trainer->engine weight pull.

``request_batch(input_ids, infer_max_tokens)`` runs one interruptible request (stop on ``"\\n"``,
temperature / top-p from the flags, per-token logprobs and versions); ``pause_and_wait_idle`` pauses
the runner, aborts the engine's in-flight requests with their KV cache cleared and waits until every
attempt has drained; ``resume_generation(increment_version)`` bumps the policy version.

Weight sync: a trainer rank exports its flat bf16 parameter buffer once (a CUDA IPC handle, or a
shared-memory handle on CPU); ``attach_trainer_weights`` maps it into this process and
``pull_weights(scope_numel)`` copies the requested prefix (all parameters, or only the contiguous
trainable segment) straight from trainer memory into the engine's identical fused layout over NVLink,
timed with CUDA events.
"""

from __future__ import annotations

import asyncio
import time
from typing import Any, Dict, List, Optional

import torch

from ..models.config import resolve_model_config
from .engine import GenerationEngine
from .generation import InferenceResult, InterruptibleGenerationRunner, OnlineGenerationState


class InferenceService:
    def __init__(self, args, device: torch.device, tokenizer=None, dtype: Optional[torch.dtype] = None):
        self.args = args
        self.device = device
        if device.type == "cuda":
            torch.cuda.set_device(device)
        cfg = resolve_model_config(args.model_path)
        self.cfg = cfg
        dtype = dtype or (torch.bfloat16 if device.type == "cuda" else torch.float32)
        self.engine = GenerationEngine(
            cfg,
            device,
            dtype,
            max_num_seqs=args.vllm_max_num_seqs,
            max_num_batched_tokens=args.vllm_max_num_batched_tokens,
            max_model_len=args.vllm_max_model_len,
            block_size=getattr(args, "kv_block_size", 16),
            kv_cache_gb=getattr(args, "kv_cache_gb", None),
            enable_prefix_caching=not args.disable_vllm_prefix_caching,
            tokenizer=tokenizer,
        )
        if tokenizer is None:
            stop = None
        elif getattr(args, "env", "textworld") == "gsm8k":
            stop = ["</answer>"]  # R1-zero answers end at the closing tag (vllm_fsdp.py:1212-1217)
        else:
            stop = ["\n"]
        self.runner = InterruptibleGenerationRunner(
            self.engine, temperature=args.infer_temperature, top_p=args.infer_top_p, stop_sequences=stop,
            collect_logprobs=True,
        )
        if stop is None:
            self.runner.stop_sequences = None
        self.total_tokens = 0
        # bound on in-flight generation requests (the reference's actor max-concurrency knob)
        self._slots = asyncio.Semaphore(int(getattr(args, "infer_actor_max_concurrency", 1 << 20)))
        self.next_request_index = 0
        self.stopped = False
        self.active_generation_tasks = set()
        self._trainer_params: Optional[torch.Tensor] = None
        self.last_sync: Dict[str, float] = {}
        self.engine.start()

    # ------------------------------------------------------------------ generation
    async def request_batch(self, input_ids: List[int], infer_max_tokens: int) -> InferenceResult:
        async with self._slots:
            return await self._request(input_ids, infer_max_tokens)

    async def _request(self, input_ids: List[int], infer_max_tokens: int) -> InferenceResult:
        if self.stopped:
            raise RuntimeError("InferenceService is stopped.")
        index = self.next_request_index
        self.next_request_index += 1
        state = OnlineGenerationState(index=index, input_ids=list(input_ids), requested_max_tokens=int(infer_max_tokens))
        task = asyncio.create_task(self.runner.generate(state))
        self.active_generation_tasks.add(task)
        task.add_done_callback(self.active_generation_tasks.discard)
        try:
            done = await task
        except asyncio.CancelledError:
            if not task.done():
                task.cancel()
            await asyncio.gather(task, return_exceptions=True)
            raise
        result = InferenceResult(list(done.output_tokens), list(done.output_logprobs), list(done.output_versions),
                                 done.stop_reason)
        self.total_tokens += len(result.output_tokens)
        return result

    async def pause_and_wait_idle(self) -> None:
        self.runner.pause()
        await self.engine.pause_generation(mode="abort", clear_cache=True)
        await self.runner.wait_for_idle()

    async def resume_generation(self, increment_version: bool = False) -> int:
        if increment_version:
            self.runner.version += 1
        await self.engine.resume_generation()
        self.runner.resume()
        return self.runner.version

    @property
    def version(self) -> int:
        return self.runner.version

    # ------------------------------------------------------------------ weights
    def attach_trainer_weights(self, handle) -> int:
        """Map a trainer's exported flat parameter buffer into this process."""
        fn, fargs = handle
        self._trainer_params = fn(*fargs)
        if self._trainer_params.numel() < self.engine.layout.total_numel:
            raise ValueError("trainer parameter buffer is smaller than the engine layout")
        return int(self._trainer_params.numel())

    def pull_weights(self, numel: Optional[int] = None) -> Dict[str, float]:
        """Copy the first ``numel`` elements (default: everything) of the trainer's flat buffer into
        the engine. The engine must be paused. Returns timing and throughput."""
        if self._trainer_params is None:
            raise RuntimeError("attach_trainer_weights() was not called")
        n = self.engine.layout.total_numel if numel is None else int(numel)
        src = self._trainer_params[:n]
        t0 = time.perf_counter()
        if self.device.type == "cuda":
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            self.engine.load_flat_weights(src)
            end.record()
            torch.cuda.synchronize(self.device)
            dev_ms = start.elapsed_time(end)
        else:
            self.engine.load_flat_weights(src)
            dev_ms = (time.perf_counter() - t0) * 1e3
        wall = time.perf_counter() - t0
        nbytes = n * src.element_size()
        self.last_sync = {"device_ms": dev_ms, "wall_s": wall, "bytes": float(nbytes),
                          "gbs": nbytes / max(dev_ms, 1e-6) / 1e6}
        return self.last_sync

    def load_checkpoint(self, path: str) -> None:
        self.engine.reload_weights(path)

    # ------------------------------------------------------------------ misc
    def get_stats(self) -> Dict[str, Any]:
        s = {"total_tokens": self.total_tokens, "version": self.runner.version}
        s.update(self.engine.get_stats())
        return s

    async def shutdown(self) -> Dict[str, Any]:
        self.stopped = True
        self.runner.resume()
        for t in list(self.active_generation_tasks):
            if not t.done():
                t.cancel()
        if self.active_generation_tasks:
            await asyncio.gather(*self.active_generation_tasks, return_exceptions=True)
        await self.engine.shutdown()
        return self.get_stats()
