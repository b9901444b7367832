"""Inference service: the reference's ``VLLMInferenceActor`` surface (agent_textworld.py:1916-2060)
over the native engine, plus the trainer->engine weight pull.

``request_batch(input_ids, infer_max_tokens)`` runs one interruptible request (stop on ``"\\n"``,
temperature / top-p from the flags, per-token logprobs and versions); ``pause_and_wait_idle`` closes
the runner's gate and parks the engine's in-flight requests with their KV cache cleared once its last
step has completed; ``resume_generation(increment_version)`` bumps the policy version, which the
engine then stamps on every token it samples.

Weight sync: a trainer rank exports its flat bf16 parameter buffer once (a CUDA IPC handle, or a
shared-memory handle on CPU); ``attach_trainer_weights`` maps it into this process (opened on this
engine's device) together with the trainer's parameter layout, and ``pull_weights(scope)`` copies
the engine's slice of every parameter (``all``, or only the ``trainable`` ones) straight from trainer
memory into the engine's fused layout with one copy-plan kernel over NVLink, timed with CUDA events.
Tensor-parallel engines pull on every rank, each its own shard.
"""

from __future__ import annotations

import asyncio
import time
from typing import Any, Dict, List, Optional

import torch

from ..models.config import resolve_model_config
from .engine import GenerationEngine
from .generation import InferenceResult, InterruptibleGenerationRunner, OnlineGenerationState


def init_tp_groups(tp_rank: int, tp_size: int, port: int, device: torch.device):
    """Process groups of one tensor-parallel engine (its ranks only): the default group carries the
    activations' all-reduces (NCCL on GPUs), a gloo group carries the leader's step commands."""
    import datetime

    import torch.distributed as dist

    backend = "nccl" if device.type == "cuda" else "gloo"
    kw = {"device_id": device} if device.type == "cuda" else {}
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=tp_rank, world_size=tp_size,
                            timeout=datetime.timedelta(seconds=600), **kw)
    return dist.group.WORLD, dist.new_group(backend="gloo")


def build_engine(args, device: torch.device, tokenizer=None, dtype: Optional[torch.dtype] = None,
                 tp_groups=None) -> GenerationEngine:
    cfg = resolve_model_config(args.model_path)
    dtype = dtype or (torch.bfloat16 if device.type == "cuda" else torch.float32)
    tp_group, cmd_group = tp_groups if tp_groups else (None, None)
    return GenerationEngine(
        cfg,
        device,
        dtype,
        max_num_seqs=args.vllm_max_num_seqs,
        max_num_batched_tokens=args.vllm_max_num_batched_tokens,
        max_model_len=args.vllm_max_model_len,
        block_size=getattr(args, "kv_block_size", 16),
        kv_cache_gb=getattr(args, "kv_cache_gb", None),
        gpu_memory_utilization=getattr(args, "gpu_memory_utilization", None),
        enable_prefix_caching=not args.disable_vllm_prefix_caching,
        tokenizer=tokenizer,
        tp_group=tp_group,
        cmd_group=cmd_group,
    )


class InferenceService:
    def __init__(self, args, device: torch.device, tokenizer=None, dtype: Optional[torch.dtype] = None,
                 tp_groups=None):
        self.args = args
        self.device = device
        if device.type == "cuda":
            torch.cuda.set_device(device)
        self.engine = build_engine(args, device, tokenizer, dtype, tp_groups)
        self.cfg = self.engine.full_cfg
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
        self._ipc_bases: List[int] = []
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
        """Hold back new requests and park the engine's in-flight ones (their tokens are kept; they
        continue after ``resume_generation`` under the new weights). Returns once the engine has
        completed its last step, so the weights can be replaced."""
        self.runner.pause()
        await self.engine.pause_generation(mode="suspend", clear_cache=True)

    async def resume_generation(self, increment_version: bool = False) -> int:
        if increment_version:
            self.runner.version += 1
        await self.engine.resume_generation(version=self.runner.version)
        self.runner.resume()
        return self.runner.version

    @property
    def version(self) -> int:
        return self.runner.version

    # ------------------------------------------------------------------ weights
    def attach_trainer_weights(self, handle) -> int:
        """Map a trainer's exported flat parameter buffer into this process and register it (with the
        trainer's layout) as the engine's weight source. Returns the buffer's element count."""
        return attach_weight_source(self.engine, self.args, self.device, handle, self._ipc_bases)

    def pull_weights(self, scope: Any = "all") -> Dict[str, float]:
        """Copy this engine's slice of the trainer's parameters (``scope`` ``"all"`` or
        ``"trainable"``) into its weights. The engine must be paused. Returns timing and bytes."""
        if not isinstance(scope, str):
            scope = "all"
        t0 = time.perf_counter()
        if self.device.type == "cuda":
            with torch.cuda.device(self.device):
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                nbytes = self.engine.pull_weights(scope)
                end.record()
                torch.cuda.synchronize(self.device)
                dev_ms = start.elapsed_time(end)
        else:
            nbytes = self.engine.pull_weights(scope)
            dev_ms = (time.perf_counter() - t0) * 1e3
        wall = time.perf_counter() - t0
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
        await asyncio.to_thread(self.engine.stop_followers)
        return self.get_stats()


def _open_handle(handle, device: torch.device, opened: List[int]):
    """Map one exported trainer buffer on ``device``: returns ``(tensor, addr, numel)``."""
    if isinstance(handle, dict) and handle.get("kind") == "cuda-ipc":
        from .. import ops
        from ..ops._ext import native

        ext = native()
        with torch.cuda.device(device):
            if handle["device"] != device.index:
                ops.native().enable_peer_access(handle["device"])
            rc, base = ext.ipc_open(handle["handle"])
            if rc != 0:
                raise RuntimeError(f"cudaIpcOpenMemHandle of the trainer's parameters failed with code {rc}")
            opened.append(base)
            addr = base + handle["offset"]
            probe = handle.get("probe") or b""
            if probe:
                rc, got = ext.peer_read(addr, len(probe))
                if rc != 0 or bytes(got) != probe:
                    raise RuntimeError("the trainer's parameter mapping is not readable or holds other data")
        return None, addr, int(handle["numel"])
    fn, fargs = handle["reduce"] if isinstance(handle, dict) else handle
    tensor = fn(*fargs)
    return tensor, None, int(tensor.numel())


def _attach_sharded_sources(engine: GenerationEngine, cfg, device: torch.device, handles, opened: List[int]) -> int:
    """Layer-sharded trainers (``parallel/zero3.py``): map every trainer's shard buffer and pull each
    element from the trainer that stores it."""
    from ..parallel.zero3 import build_units, shard_pieces, sharded_layout
    from .weight_map import build_weight_map_sharded

    world = int(handles[0]["world"])
    handles = sorted(handles, key=lambda h: int(h["trainer_rank"]))
    if [int(h["trainer_rank"]) for h in handles] != list(range(world)):
        raise ValueError("layer-sharded weight sync needs the handle of every trainer rank")
    full = sharded_layout(cfg, handles[0].get("train_mode", "full"))
    pieces = shard_pieces(build_units(full, world, {n: s.trainable for n, s in full.slots.items()}), world)
    srcs, total = [], 0
    for h in handles:
        tensor, addr, numel = _open_handle(h, device, opened)
        srcs.append({"tensor": tensor, "addr": addr})
        total += numel
    plans = {scope: build_weight_map_sharded(cfg, full, pieces, world, engine.layout, engine.tp_rank, engine.tp, scope)
             for scope in ("all", "trainable")}
    engine.set_weight_plans(plans, srcs)
    return total


def attach_weight_source(engine: GenerationEngine, args, device: torch.device, handle, opened: List[int]) -> int:
    """Open a trainer's exported parameter handle on ``device`` and register it with ``engine``. A list
    of handles (one per trainer rank, from expert-partitioned trainers) registers every buffer: routed
    experts are pulled from their owner, the rest from trainer ``tp_rank % len(handles)``."""
    from ..models.transformer import ParamLayout

    handles = handle if isinstance(handle, list) else [handle]
    cfg = engine.full_cfg
    if isinstance(handles[0], dict) and handles[0].get("zero3"):
        return _attach_sharded_sources(engine, cfg, device, handles, opened)
    srcs, total = [], 0
    for h in handles:
        part = bool(isinstance(h, dict) and h.get("partition"))
        if part:
            from ..parallel.expert_parallel import expert_partition

            cfg_t = expert_partition(cfg, int(h["trainer_rank"]), int(h["world"]))
        else:
            cfg_t = cfg
        layout = ParamLayout.build(cfg_t, args.train_mode, pad_to=args.fsdp_world_size, experts_last=part)
        tensor, addr, numel = _open_handle(h, device, opened)
        if numel < layout.total_numel:
            raise ValueError("trainer parameter buffer is smaller than the trainer layout")
        srcs.append({"layout": layout, "tensor": tensor, "addr": addr,
                     "expert_lo": cfg_t.expert_offset if part else 0,
                     "expert_count": cfg_t.local_experts if part else cfg.num_experts})
        total += numel
    if len(srcs) == 1 and srcs[0]["expert_count"] == cfg.num_experts:
        engine.set_weight_source(srcs[0]["layout"], tensor=srcs[0]["tensor"], addr=srcs[0]["addr"])
    else:
        engine.set_weight_sources(srcs, primary=engine.tp_rank % len(srcs))
    return total
