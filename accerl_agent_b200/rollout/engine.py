"""Native paged-KV generation engine (continuous batching, chunked prefill, prefix caching,
temperature sampling, abort/pause/resume, in-place weight updates).

It is the rollout-side replacement of the vLLM ``AsyncLLMEngine`` that the reference drives
(agent_textworld.py:1916-2060) and exposes the same asynchronous surface:

* ``async for out in engine.generate({"prompt_token_ids": ids}, sampling_params, request_id=...)``
  yields cumulative ``RequestOutput`` objects (``.finished``, ``.outputs[0].token_ids``,
  ``.outputs[0].finish_reason``, ``.outputs[0].logprobs`` as ``[{token: logprob}]``);
* ``pause_generation(mode="abort", clear_cache=True)`` finishes every in-flight request with reason
  ``"abort"`` and frees (and optionally forgets) the KV cache; ``mode="suspend"`` instead parks every
  request (KV released, tokens kept) until ``resume_generation(version=v)``, after which it continues
  under the new weights; every sampled token is tagged with the engine's version
  (``CompletionOutput.token_versions``);
* ``collective_rpc("reload_weights", kwargs={"weights_path": ...})`` and ``load_flat_weights`` for
  in-place weight updates (the trainer and engine share the fused flat parameter layout).

One background thread runs the step loop. A step schedules decode tokens of running sequences first
and then prefill chunks of waiting ones under ``max_num_batched_tokens`` / ``max_num_seqs``, runs one
forward over the mixed batch (new K/V written straight into their paged slots, prefill queries over
their cached prefix with the varlen attention kernel, decode queries with the paged decode kernel),
applies the LM head only to rows that sample, and samples on the device (temperature, top-k,
top-p; ``csrc/sampler.cu``), which also returns each sampled token's log-probability. Sampled ids come back to the host once per step.
"""

from __future__ import annotations

import asyncio
import itertools
import math
import threading
import time
from collections import deque
from dataclasses import dataclass, field
from typing import Any, Deque, Dict, List, Optional

import numpy as np
import torch

from .. import ops
from ..utils import nvtx
from ..models.config import ModelConfig
from ..models.transformer import CausalLM, ParamLayout
from .generation import SamplingParams
from .kv_cache import BlockAllocator, block_hash


@dataclass
class CompletionOutput:
    index: int
    token_ids: List[int]
    finish_reason: Optional[str]
    logprobs: Optional[List[Dict[int, float]]]
    text: str = ""
    # policy version each token was sampled under (the engine's version at that step)
    token_versions: Optional[List[int]] = None


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: List[int]
    outputs: List[CompletionOutput]
    finished: bool


@dataclass
class _Seq:
    rid: str
    prompt: List[int]
    params: SamplingParams
    seed: int
    loop: Any
    queue: Any
    out: List[int] = field(default_factory=list)
    lps: List[float] = field(default_factory=list)
    versions: List[int] = field(default_factory=list)
    blocks: List[int] = field(default_factory=list)
    hashes: List[int] = field(default_factory=list)
    num_computed: int = 0
    finish_reason: Optional[str] = None
    arrival: float = 0.0
    toks: List[int] = field(default_factory=list)  # prompt + out, kept in step (no per-access concat)
    slot: int = -1     # row of the engine's device-side last-token table
    pending: int = 0   # 1 while a sampled token is on the device but not yet on the host

    def __post_init__(self) -> None:
        self.toks = list(self.prompt)

    def append(self, tok: int, lp: float, version: int) -> None:
        self.out.append(tok)
        self.lps.append(lp)
        self.versions.append(version)
        self.toks.append(tok)

    @property
    def tokens(self) -> List[int]:
        return self.toks

    @property
    def length(self) -> int:
        """Logical length: known tokens plus the one still on the device."""
        return len(self.toks) + self.pending


class GenerationEngine:
    def __init__(
        self,
        cfg: ModelConfig,
        device: torch.device,
        dtype: torch.dtype = torch.bfloat16,
        max_num_seqs: int = 128,
        max_num_batched_tokens: int = 8192,
        max_model_len: Optional[int] = None,
        block_size: int = 16,
        num_blocks: Optional[int] = None,
        kv_cache_gb: Optional[float] = None,
        enable_prefix_caching: bool = True,
        tokenizer=None,
        params: Optional[torch.Tensor] = None,
        gpu_memory_utilization: Optional[float] = None,
        seed: int = 0,
        decode_splits: Optional[int] = None,
        use_cuda_graphs: bool = True,
        layout: Optional[ParamLayout] = None,
        tp_group=None,
        cmd_group=None,
        async_steps: bool = True,
    ):
        """``layout``: flat parameter layout of the engine (default: the full-model layout); pass the
        trainer's layout to make weight syncs plain range copies. ``tp_group``/``cmd_group``: process
        groups of a tensor-parallel engine (NCCL for the activations' all-reduce, gloo for the step
        commands the leader, group rank 0, broadcasts); rank r then holds the r-th shard of every
        tensor-parallel weight and ranks > 0 run ``serve_follower``."""
        if device.type == "cuda" and device.index is None:  # the step thread selects this exact GPU
            device = torch.device("cuda", torch.cuda.current_device())
        self.full_cfg = cfg
        self.tp_group = tp_group
        self.cmd_group = cmd_group
        if tp_group is not None:
            import torch.distributed as dist

            self.tp = dist.get_world_size(tp_group)
            self.tp_rank = dist.get_rank(tp_group)
            self._cmd_src = dist.get_global_rank(cmd_group, 0)
        else:
            self.tp, self.tp_rank, self._cmd_src = 1, 0, 0
        self._followers_stopped = False
        if self.tp > 1:
            from .weight_map import tp_shard_config

            cfg = tp_shard_config(cfg, self.tp)
            if cfg.local_experts:
                cfg.expert_offset = self.tp_rank * cfg.local_experts
            layout = None
        self.cfg = cfg
        self.device = device
        self.dtype = dtype
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len or cfg.max_position_embeddings
        self.block_size = block_size
        # prefill attention reads keys from the paged cache in place (tensor-core kernel, head dim 128,
        # pages that divide its 128-token tiles); otherwise the context keys are gathered by slot
        self._paged_prefill = (device.type == "cuda" and cfg.head_dim == 128 and 8 <= block_size <= 128
                               and 128 % block_size == 0)
        self.tokenizer = tokenizer
        self.layout = layout or ParamLayout.build(cfg, "full")
        self._weight_src = None
        self._weight_maps: Dict[str, Any] = {}
        if params is None:
            params = torch.zeros(self.layout.total_numel, dtype=dtype, device=device)
        self.model = CausalLM(cfg, self.layout, params, None)
        L, Hkv, D = cfg.num_hidden_layers, cfg.num_key_value_heads, cfg.head_dim
        per_block = 2 * L * block_size * Hkv * D * torch.tensor([], dtype=dtype).element_size()
        if num_blocks is None:
            if kv_cache_gb is None:
                if device.type == "cuda":
                    free, total = torch.cuda.mem_get_info(device)
                    if gpu_memory_utilization:
                        # vLLM's rule: this process may hold `utilization` of the device; what the
                        # weights leave, minus a reserve for step workspaces, becomes KV cache
                        reserve = 10 * 1024**3
                        kv_cache_gb = max(1.0, (gpu_memory_utilization * total - (total - free) - reserve) / 1024**3)
                    else:
                        kv_cache_gb = 0.6 * free / 1024**3
                else:
                    kv_cache_gb = 0.25
            num_blocks = max(16, int(kv_cache_gb * 1024**3 // per_block))
        self.num_blocks = num_blocks
        self.k_cache = torch.zeros(L, num_blocks, block_size, Hkv, D, dtype=dtype, device=device)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.allocator = BlockAllocator(num_blocks, block_size, enable_prefix_caching)
        self._tp_ar = None
        self._ar_calls = 0
        if self.tp > 1 and device.type == "cuda":
            from ..parallel.symmetric import peer_access_available

            if peer_access_available(tp_group):
                from ..parallel.tp_allreduce import TPAllReduce

                rows = max(max_num_batched_tokens, max(self._BUCKETS))
                self._tp_ar = TPAllReduce(tp_group, device, rows * cfg.hidden_size, dtype)
        # block 0 is never handed to a sequence: padded rows of captured decode graphs point at it
        self.scratch_block = self.allocator.allocate()
        # MoE layers run the device-side routing layout (no host synchronisation), so single-GPU MoE
        # decode steps are captured like dense ones (tensor-parallel MoE engines stay eager);
        # tensor-parallel steps are captured only with the peer-memory all-reduce (no NCCL inside graphs)
        self.use_cuda_graphs = (use_cuda_graphs and device.type == "cuda"
                                and (not cfg.is_moe or (dtype == torch.bfloat16 and self.tp == 1))
                                and (self.tp == 1 or self._tp_ar is not None))
        self._graphs: Dict[Any, Any] = {}
        self._graph_pool = None
        # Asynchronous steps: step N+1 is launched before the tokens of step N reach the host. A decode
        # row reads its input token from a device table indexed by the sequence's slot (written by the
        # sampler), stop conditions are applied one step late, and a row launched for a sequence that
        # turned out to be finished is discarded.
        self.async_steps = async_steps
        n_slots = 2 * max_num_seqs + 1
        self._slot_tok = torch.zeros(n_slots, dtype=torch.long, device=device)
        self._dummy_slot = n_slots - 1
        self._free_slots = list(range(n_slots - 1))
        self._inflight = None
        self._pin_ring: List[torch.Tensor] = []
        self._pin_next = 0
        self._in_ring: List[List[Any]] = []
        self._in_next = 0
        self._res_rows = max(max_num_seqs, max(self._BUCKETS))
        self.waiting: Deque[_Seq] = deque()
        self.running: List[_Seq] = []
        self.by_id: Dict[str, _Seq] = {}
        self.paused = False
        self.version = 0  # policy version of the weights; tags every sampled token
        self._lock = threading.RLock()  # protects queues and sequence state
        self._step_lock = threading.Lock()  # held for the duration of one engine step
        self._wake = threading.Condition(self._lock)
        self._stop = False
        self._seed_counter = itertools.count(seed * 1_000_003 + 1)
        self.decode_splits = decode_splits
        self.stats = {"generated_tokens": 0, "prompt_tokens_computed": 0, "steps": 0, "preemptions": 0,
                      "aborted": 0, "suspended": 0, "finished": 0, "prefill_rows": 0, "decode_rows": 0,
                      # host wall time per step phase: scheduling, building and launching the step, and
                      # completing the previous one (waiting for its samples, appending, stop checks)
                      "t_schedule_s": 0.0, "t_launch_s": 0.0, "t_complete_s": 0.0}
        self._thread: Optional[threading.Thread] = None
        self.eos_ids = {cfg.eos_token_id}
        if tokenizer is not None and getattr(tokenizer, "eos_token_id", None) is not None:
            self.eos_ids.add(int(tokenizer.eos_token_id))

    # ------------------------------------------------------------------ lifecycle
    def start(self) -> None:
        if self._thread is None:
            self._thread = threading.Thread(target=self._run_loop, name="generation-engine", daemon=True)
            self._thread.start()

    async def shutdown(self) -> None:
        with self._lock:
            self._stop = True
            self._wake.notify_all()
        if self._thread is not None:
            await asyncio.to_thread(self._thread.join, 30)
            self._thread = None
        self._abort_all("abort")

    def _run_loop(self) -> None:
        # the CUDA current device is per thread: this thread launches on the engine's GPU
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        while True:
            with self._lock:
                while not self._stop and self._inflight is None and (
                        self.paused or (not self.waiting and not self.running)):
                    self._wake.wait(timeout=0.5)
                if self._stop:
                    return
            try:
                self.step()
            except Exception as exc:  # fail every request loudly instead of hanging callers
                import traceback

                traceback.print_exc()
                self._abort_all("abort", error=exc)

    # ------------------------------------------------------------------ public async API
    async def generate(self, prompt: Dict[str, List[int]], sampling_params: SamplingParams, request_id: str):
        if getattr(sampling_params, "frequency_penalty", 0.0):
            # accepted by the vLLM-shaped parameter object but not applied by this engine's sampler:
            # refuse instead of sampling without it
            raise ValueError("frequency_penalty is not supported by the native engine")
        if self._thread is None:
            self.start()
        loop = asyncio.get_running_loop()
        queue: asyncio.Queue = asyncio.Queue()
        ids = list(prompt["prompt_token_ids"])
        seed = sampling_params.seed if sampling_params.seed is not None else next(self._seed_counter)
        seq = _Seq(request_id, ids, sampling_params, int(seed) & ((1 << 62) - 1), loop, queue, arrival=time.time())
        with self._lock:
            if request_id in self.by_id:
                raise ValueError(f"duplicate request id {request_id}")
            self.by_id[request_id] = seq
            self.waiting.append(seq)
            self._wake.notify_all()
        finished = False
        try:
            while True:
                item = await queue.get()
                if isinstance(item, BaseException):
                    raise item
                yield item
                if item.finished:
                    finished = True
                    break
        finally:
            if not finished:
                self.abort(request_id)

    def abort(self, request_id: str) -> None:
        with self._step_lock, self._lock:
            seq = self.by_id.get(request_id)
            if seq is not None:
                self._finish(seq, "abort")

    async def pause_generation(self, mode: str = "abort", clear_cache: bool = True) -> None:
        """Stop scheduling once the step in flight has completed. ``mode='abort'``: every request
        ends with reason 'abort'. ``mode='suspend'``: every request is parked (its KV blocks are
        released, its tokens kept) and continues after ``resume_generation``, recomputing its prompt
        and tokens so far under whatever weights were loaded meanwhile."""
        def _pause():
            # one step-lock section: no step can launch between completing the one in flight and
            # parking the requests
            with self._step_lock, self._lock:
                self._flush()
                self.paused = True
                if mode == "abort":
                    self._abort_all("abort")
                elif mode == "suspend":
                    for seq in reversed(list(self.running)):
                        self._preempt(seq)
                    self.stats["suspended"] += len(self.waiting)
                if clear_cache:
                    self.allocator.clear_cache()

        await asyncio.to_thread(_pause)

    async def resume_generation(self, version: Optional[int] = None) -> None:
        """Resume scheduling; a given ``version`` tags the tokens sampled from now on."""
        with self._lock:
            if version is not None:
                self.version = int(version)
            self.paused = False
            self._wake.notify_all()

    async def collective_rpc(self, method: str, kwargs: Optional[Dict[str, Any]] = None, args=()):
        kwargs = kwargs or {}
        if method == "reload_weights":
            path = kwargs.get("weights_path") or (args[0] if args else None)
            await asyncio.to_thread(self.reload_weights, path)
            return [None]
        fn = getattr(self, method)
        res = fn(*args, **kwargs)
        if asyncio.iscoroutine(res):
            res = await res
        return [res]

    def report_cuda_memory(self, label: str, empty_cache: bool = False) -> Dict[str, Any]:
        """Memory of this engine's process (``collective_rpc("report_cuda_memory", args=(label,))``)."""
        from ..utils.memory import cuda_memory_report

        if self.device.type != "cuda":
            return {"label": label, "device": "cpu"}
        with torch.cuda.device(self.device):
            return cuda_memory_report(label, empty_cache)

    def reload_weights(self, path: str) -> None:
        from ..models.hf_io import load_hf_checkpoint

        with self._step_lock:
            self._flush()
            load_hf_checkpoint(self.model, path)
            self.allocator.clear_cache()

    def load_flat_weights(self, src: torch.Tensor, start: int = 0, stream=None) -> None:
        """Copy a fused-layout flat weight range (from a trainer, possibly a peer GPU's memory)."""
        with self._step_lock:
            self._flush()
            dst = self.model.params[start : start + src.numel()]
            if stream is not None:
                with torch.cuda.stream(stream):
                    dst.copy_(src, non_blocking=True)
            else:
                dst.copy_(src, non_blocking=True)

    def set_weight_source(self, src_layout: ParamLayout, tensor: Optional[torch.Tensor] = None,
                          addr: Optional[int] = None) -> None:
        """Register the trainer's flat bf16 buffer (a tensor, or a device address mapped by CUDA IPC)
        and precompute this rank's copy plans for the ``all`` and ``trainable`` scopes."""
        from .weight_map import build_weight_map, descs_tensor

        maps = {}
        for scope in ("all", "trainable"):
            descs = build_weight_map(self.full_cfg, src_layout, self.layout, self.tp_rank, self.tp, scope)
            maps[scope] = [(descs, descs_tensor(descs, self.device) if self.device.type == "cuda" else None)]
        self._weight_maps = maps
        self._weight_src = [(tensor, addr)]

    def set_weight_sources(self, sources, primary: int = 0) -> None:
        """Several trainer buffers, e.g. expert-partitioned trainers: ``sources`` lists dicts with
        ``layout``, ``expert_lo``, ``expert_count`` and ``tensor`` or ``addr``. Routed experts are pulled
        from their owner, everything else from ``sources[primary]``."""
        from .weight_map import build_weight_map_multi, descs_tensor

        srcs = [(src["layout"], int(src["expert_lo"]), int(src["expert_count"])) for src in sources]
        maps = {}
        for scope in ("all", "trainable"):
            plans = build_weight_map_multi(self.full_cfg, srcs, self.layout, self.tp_rank, self.tp, scope, primary)
            maps[scope] = [(pl, descs_tensor(pl, self.device) if self.device.type == "cuda" and pl else None)
                           for pl in plans]
        self._weight_maps = maps
        self._weight_src = [(src.get("tensor"), src.get("addr")) for src in sources]

    def set_weight_plans(self, plans_by_scope, sources) -> None:
        """Precomputed copy plans, one per source buffer and scope (layer-sharded trainers: every
        element is pulled from the trainer that stores it). ``sources`` lists dicts with ``tensor``
        or ``addr``."""
        from .weight_map import descs_tensor

        self._weight_maps = {scope: [(pl, descs_tensor(pl, self.device) if self.device.type == "cuda" and pl else None)
                                     for pl in plans] for scope, plans in plans_by_scope.items()}
        self._weight_src = [(src.get("tensor"), src.get("addr")) for src in sources]

    def pull_weights(self, scope: str = "all") -> int:
        """Copy this engine's slice of the registered trainer buffer into its weights (every TP rank
        pulls its own shard). Returns the bytes this rank copied."""
        with self._step_lock, nvtx.range("engine/pull_weights"):
            self._flush()
            if self.tp > 1 and self.tp_rank == 0:
                import torch.distributed as dist

                self._cmd(("pull", scope))
                n = self._pull_local(scope)
                dist.barrier(group=self.cmd_group)
                return n
            return self._pull_local(scope)

    def _pull_local(self, scope: str) -> int:
        from .weight_map import apply_map_torch, map_bytes

        if self._weight_src is None:
            raise RuntimeError("set_weight_source() was not called")
        dst = self.model.params
        nbytes = 0
        for (descs, descs_d), (tensor, addr) in zip(self._weight_maps[scope], self._weight_src):
            if not descs:
                continue
            if addr is not None:
                with torch.cuda.device(self.device):
                    ops.weight_pull(descs_d, addr, dst)
            else:
                apply_map_torch(tensor, dst, descs)
            nbytes += map_bytes(descs, dst.element_size())
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        return nbytes

    def get_stats(self) -> Dict[str, Any]:
        with self._lock:
            s = dict(self.stats)
            s.update(waiting=len(self.waiting), running=len(self.running), free_blocks=self.allocator.num_free,
                     prefix_cache_hit_rate=self.allocator.hits / max(self.allocator.queries, 1))
            return s

    # ------------------------------------------------------------------ request bookkeeping
    def _deliver(self, seq: _Seq, finished: bool, error: Optional[BaseException] = None) -> None:
        if error is not None:
            item: Any = error
        else:
            want_lp = seq.params.logprobs is not None
            comp = CompletionOutput(
                0, list(seq.out), seq.finish_reason if finished else None,
                [{t: lp} for t, lp in zip(seq.out, seq.lps)] if want_lp else None,
                token_versions=list(seq.versions),
            )
            item = RequestOutput(seq.rid, seq.prompt, [comp], finished)
        try:
            seq.loop.call_soon_threadsafe(seq.queue.put_nowait, item)
        except RuntimeError:
            pass  # the caller's event loop is gone

    def _finish(self, seq: _Seq, reason: str, error: Optional[BaseException] = None) -> None:
        seq.finish_reason = reason
        if seq.slot >= 0:
            # a row still in flight may write this slot; the next owner writes it later in stream order
            self._free_slots.append(seq.slot)
            seq.slot = -1
        if seq in self.running:
            self.running.remove(seq)
        try:
            self.waiting.remove(seq)
        except ValueError:
            pass
        self.allocator.free(seq.blocks)
        seq.blocks = []
        self.by_id.pop(seq.rid, None)
        self.stats["aborted" if reason == "abort" else "finished"] += 1
        self._deliver(seq, True, error)

    def _abort_all(self, reason: str, error: Optional[BaseException] = None) -> None:
        with self._lock:
            for seq in list(self.running) + list(self.waiting):
                self._finish(seq, reason, error)

    # ------------------------------------------------------------------ scheduling
    def _ensure_blocks(self, seq: _Seq, upto: int) -> bool:
        need = (upto + self.block_size - 1) // self.block_size
        while len(seq.blocks) < need:
            b = self.allocator.allocate()
            if b is None:
                return False
            seq.blocks.append(b)
        return True

    def _preempt(self, seq: _Seq) -> None:
        """Recompute-style preemption: drop the sequence's KV and requeue it first."""
        self.running.remove(seq)
        self.allocator.free(seq.blocks)
        seq.blocks, seq.hashes, seq.num_computed = [], [], 0
        self.waiting.appendleft(seq)
        self.stats["preemptions"] += 1

    def _admit(self, seq: _Seq) -> None:
        toks = seq.tokens
        blocks, hashes = self.allocator.match_prefix(toks)
        # always compute at least the last token so there is a row to sample from
        usable = min(len(blocks) * self.block_size, seq.length - 1)
        keep = usable // self.block_size
        self.allocator.free(blocks[keep:])
        seq.blocks = blocks[:keep]
        seq.hashes = hashes[:keep]
        seq.num_computed = keep * self.block_size

    def _schedule(self):
        budget = self.max_num_batched_tokens
        plan = []  # (seq, start, n_tokens, samples)
        with self._lock:
            if self.paused:
                return None
            for seq in list(self.running):
                if budget <= 0:
                    break
                n = min(seq.length - seq.num_computed, budget)
                if n <= 0:
                    continue
                while not self._ensure_blocks(seq, seq.num_computed + n):
                    victim = self.running[-1]
                    if victim is seq:
                        break
                    self._preempt(victim)
                    plan = [p for p in plan if p[0] is not victim]
                if len(seq.blocks) * self.block_size < seq.num_computed + n:
                    self._preempt(seq)
                    continue
                plan.append((seq, seq.num_computed, n, seq.num_computed + n == seq.length))
                budget -= n
            while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
                seq = self.waiting[0]
                if seq.pending:
                    break  # preempted with a token in flight: re-admit once it is on the host
                if seq.slot < 0:
                    if not self._free_slots:
                        break
                    seq.slot = self._free_slots.pop()
                if seq.num_computed == 0 and not seq.blocks:
                    self._admit(seq)
                n = min(seq.length - seq.num_computed, budget)
                if not self._ensure_blocks(seq, seq.num_computed + n):
                    self.allocator.free(seq.blocks)
                    seq.blocks, seq.hashes, seq.num_computed = [], [], 0
                    break
                self.waiting.popleft()
                self.running.append(seq)
                plan.append((seq, seq.num_computed, n, seq.num_computed + n == seq.length))
                budget -= n
        return plan or None

    # ------------------------------------------------------------------ execution
    def step(self) -> bool:
        with self._step_lock:
            t0 = time.perf_counter()
            with nvtx.range("engine/schedule"):
                plan = self._schedule()
            t1 = time.perf_counter()
            with nvtx.range("engine/launch"):
                launched = self._launch(plan) if plan else None
            t2 = time.perf_counter()
            prev, self._inflight = self._inflight, launched
            with nvtx.range("engine/complete"):
                if prev is not None:
                    self._complete(prev)
                if not self.async_steps and self._inflight is not None:
                    cur, self._inflight = self._inflight, None
                    self._complete(cur)
            t3 = time.perf_counter()
            if plan is None and prev is None:
                return False
            st = self.stats
            if plan:
                st["steps"] += 1
                st["prefill_rows"] += sum(p[2] for p in plan if p[2] > 1)
                st["decode_rows"] += sum(1 for p in plan if p[2] == 1)
            st["t_schedule_s"] += t1 - t0
            st["t_launch_s"] += t2 - t1
            st["t_complete_s"] += t3 - t2
            return True

    def _launch(self, plan) -> Dict[str, Any]:
        """Launch one step (prefill chunks eagerly, single-token rows from a decode graph when all of
        them sample) and commit its optimistic bookkeeping. Returns the handle ``_complete`` reads."""
        prefill = [p for p in plan if p[2] > 1]
        decode = [p for p in plan if p[2] == 1]
        parts = []
        if self.use_cuda_graphs and decode and all(p[3] for p in decode):
            if prefill:
                parts.append((prefill, self._execute(prefill, len(prefill))))
            parts.append((decode, self._execute_decode_graph(decode)))
        else:
            order = prefill + decode
            parts.append((order, self._execute(order, len(prefill))))
        for seq, start, n, samples in plan:
            seq.num_computed = start + n
            self.stats["prompt_tokens_computed"] += n
            if samples:
                seq.pending += 1
        return {"parts": parts}

    def _flush(self) -> None:
        """Complete the step in flight (callers hold the step lock)."""
        if self._inflight is not None:
            cur, self._inflight = self._inflight, None
            self._complete(cur)

    def _h2d(self, host: np.ndarray) -> torch.Tensor:
        """Copy an int64 host array to a fresh device tensor without blocking the host: it is staged in
        a pinned buffer from a ring whose entries are reused only after their previous copy has run."""
        n = host.size
        if self.device.type != "cuda":
            return torch.from_numpy(np.array(host, dtype=np.int64, copy=True))
        if not self._in_ring:
            self._in_ring = [[None, None] for _ in range(8)]
        entry = self._in_ring[self._in_next]
        self._in_next = (self._in_next + 1) % len(self._in_ring)
        if entry[1] is not None:
            entry[1].synchronize()
        if entry[0] is None or entry[0].numel() < n:
            entry[0] = torch.empty(max(n, 1 << 16), dtype=torch.int64).pin_memory()
        entry[0].numpy()[:n] = host
        out = torch.empty(n, dtype=torch.int64, device=self.device)
        out.copy_(entry[0][:n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        entry[1] = ev
        return out

    def _result_buffer(self) -> torch.Tensor:
        """Flat pinned float64 buffer for one step part's tokens and log-probs (a small ring: at most
        two steps, of at most two parts each, are alive)."""
        if not self._pin_ring:
            pin = self.device.type == "cuda"
            self._pin_ring = [torch.empty(2 * self._res_rows, dtype=torch.float64, pin_memory=pin) for _ in range(6)]
        buf = self._pin_ring[self._pin_next]
        self._pin_next = (self._pin_next + 1) % len(self._pin_ring)
        return buf

    def _stage_results(self, tokens: torch.Tensor, lps: torch.Tensor):
        """Start the device->host copy of a step part's samples; returns (view [2, n], n, event). The
        destination is a contiguous prefix of a pinned buffer, so the copy never blocks the host."""
        n = tokens.shape[0]
        buf = self._result_buffer()
        if 2 * n > buf.numel():
            buf = torch.empty(2 * n, dtype=torch.float64, pin_memory=self.device.type == "cuda")
        dst = buf[: 2 * n].view(2, n)
        res = torch.stack([tokens.double(), lps.double()])
        ev = None
        if self.device.type == "cuda":
            dst.copy_(res, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
        else:
            dst.copy_(res)
        return dst, n, ev

    # ------------------------------------------------------------------ model forward
    def _all_reduce(self, y: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            import torch.distributed as dist

            dist.all_reduce(y, group=self.tp_group)
        return y

    def _row_parallel(self, a: torch.Tensor, w: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """``residual + a @ w^T`` for a row-parallel weight: every rank multiplies its column slice
        and the partial sums are all-reduced. With peer access the GEMM writes its partial into the
        symmetric buffer and one P2P kernel sums the ranks and adds the residual; otherwise rank 0
        adds the residual in the GEMM epilogue and NCCL (gloo on CPU) all-reduces."""
        if self._tp_ar is not None:
            k = self._ar_calls
            self._ar_calls += 1
            part = self._tp_ar.slot(k, a.shape[0], w.shape[0])
            ops.linear(a, w, out=part)
            return self._tp_ar.reduce(k, part, residual)
        y = ops.linear(a, w, residual=residual if self.tp_rank == 0 else None)
        return self._all_reduce(y)

    def _reduce_partial(self, y: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        """``residual + sum over ranks of y`` (``y`` a partial computed outside the symmetric buffer)."""
        if self._tp_ar is not None:
            k = self._ar_calls
            self._ar_calls += 1
            part = self._tp_ar.slot(k, y.shape[0], y.shape[1])
            part.copy_(y)
            return self._tp_ar.reduce(k, part, residual)
        if self.tp_rank == 0:
            y = y + residual
        return self._all_reduce(y)

    def _forward_layers(self, x, pos_d, slots_d, attn_fn):
        """Decoder layers over rows ``x``; ``attn_fn(layer, q, k_cache, v_cache)`` returns the
        attention output rows. Returns the final hidden rows (before the last norm)."""
        cfg, m = self.cfg, self.model
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        self._ar_calls = 0
        for layer in range(cfg.num_hidden_layers):
            p = f"model.layers.{layer}."
            h1, _ = ops.rmsnorm(x, m.w(p + "input_layernorm.weight"), cfg.rms_norm_eps)
            bias = m.w(p + "self_attn.qkv_proj.bias") if cfg.qkv_bias else None
            qkv = ops.linear(h1, m.w(p + "self_attn.qkv_proj.weight"), bias=bias)
            kc, vc = self.k_cache[layer], self.v_cache[layer]
            qn = m.w(p + "self_attn.q_norm.weight") if cfg.qk_norm else None
            kn = m.w(p + "self_attn.k_norm.weight") if cfg.qk_norm else None
            # qk-norm, RoPE and the cache write in one kernel
            ops.qkv_rope_cache(qkv, pos_d, slots_d, kc, vc, Hq, Hkv, cfg.rope_theta, qn, kn, cfg.rms_norm_eps)
            attn = attn_fn(layer, qkv[:, : cfg.q_dim], kc, vc)
            x = self._row_parallel(attn, m.w(p + "self_attn.o_proj.weight"), x)
            h2, _ = ops.rmsnorm(x, m.w(p + "post_attention_layernorm.weight"), cfg.rms_norm_eps)
            if cfg.layer_is_moe(layer):
                from ..models.moe import moe_forward

                y, _ = moe_forward(m, layer, h2, torch.zeros_like(x), save=False)
                x = self._reduce_partial(y, x)
            else:
                act, _ = ops.linear_swiglu(h2, m.w(p + "mlp.gate_up_proj.weight"))
                x = self._row_parallel(act, m.w(p + "mlp.down_proj.weight"), x)
        return x

    # ------------------------------------------------------------------ CUDA-graph decode
    _BUCKETS = (8, 16, 32, 64, 128, 256, 512)

    def _decode_core(self, ids_d, pos_d, slots_d, table_d, lens_d, temps_d, seeds_d, offs_d, splits: int,
                     rowslot_d=None):
        """Forward of single-token rows (every row samples): returns (tokens, logprobs) on device.
        Rows whose id is negative read their input token from the slot table (``rowslot_d``), and the
        sampled tokens are written back into it."""
        cfg, m = self.cfg, self.model
        if rowslot_d is not None:
            ids_d = torch.where(ids_d >= 0, ids_d, self._slot_tok.index_select(0, rowslot_d))
        scale = 1.0 / math.sqrt(cfg.head_dim)
        Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads

        def attn_fn(layer, q, kc, vc):
            return ops.paged_decode(q, kc, vc, table_d, lens_d, Hq, Hkv, scale, num_splits=splits)

        x = ops.embedding(ids_d, m.w("model.embed_tokens.weight"))
        x = self._forward_layers(x, pos_d, slots_d, attn_fn)
        hN, _ = ops.rmsnorm(x, m.w("model.norm.weight"), cfg.rms_norm_eps)
        logits = ops.linear(hN, m.w(m.lm_head_name))
        tok, lp = ops.sample(logits, temps_d, seeds_d, offs_d)
        if rowslot_d is not None:
            self._slot_tok.index_copy_(0, rowslot_d, tok)
        return tok, lp

    def _graph_for(self, bucket: int, width: int):
        key = (bucket, width)
        g = self._graphs.get(key)
        if g is not None:
            return g
        dev = self.device
        meta = torch.zeros(bucket * (6 + width), dtype=torch.int64, device=dev)
        temps = torch.zeros(bucket, dtype=torch.float32, device=dev)

        def views():
            ids = meta[:bucket]
            pos = meta[bucket : 2 * bucket]
            slots = meta[2 * bucket : 3 * bucket].to(torch.int32)
            lens = meta[3 * bucket : 4 * bucket].to(torch.int32)
            seeds = meta[4 * bucket : 5 * bucket]
            rowslot = meta[5 * bucket : 6 * bucket]
            table = meta[6 * bucket :].view(bucket, width).to(torch.int32)
            return ids, pos, slots, table, lens, seeds, rowslot

        # a valid dummy batch: every row reads one token of the scratch block and writes nothing
        meta[2 * bucket : 3 * bucket] = -1
        meta[3 * bucket : 4 * bucket] = 1
        meta[5 * bucket : 6 * bucket] = self._dummy_slot
        meta[6 * bucket :] = self.scratch_block
        splits = self.decode_splits or _decode_splits(bucket * self.cfg.num_key_value_heads)
        offs = torch.zeros(bucket, dtype=torch.int64, device=dev)

        def run():
            ids, pos, slots, table, lens, seeds, rowslot = views()
            return self._decode_core(ids, pos, slots, table, lens, temps, seeds, offs, splits, rowslot)

        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(2):
                run()
        torch.cuda.current_stream(dev).wait_stream(side)
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self._graph_pool):
            out_tok, out_lp = run()
        g = {"graph": graph, "meta": meta, "temps": temps, "offs": offs, "tok": out_tok, "lp": out_lp}
        self._graphs[key] = g
        return g

    def _graph_meta(self, order) -> Optional[Dict[str, Any]]:
        """Host inputs of one decode-graph replay (None when the batch exceeds every bucket)."""
        bs = self.block_size
        B = len(order)
        bucket = next((b for b in self._BUCKETS if b >= B), None)
        if bucket is None:
            return None
        width = max(len(s.blocks) for s, *_ in order)
        width = (width + 63) // 64 * 64
        host = np.empty(bucket * (6 + width), dtype=np.int64)
        n = B
        starts = np.fromiter((st for _, st, _, _ in order), dtype=np.int64, count=n)
        # input token: known on the host, or -1 = the sequence's pending token in the slot table
        host[:n] = np.fromiter((s.toks[st] if st < len(s.toks) else -1 for s, st, _, _ in order), dtype=np.int64,
                               count=n)
        host[n:bucket] = 0
        host[bucket : bucket + n] = starts
        host[bucket + n : 2 * bucket] = 0
        last_blk = np.fromiter((s.blocks[st // bs] for s, st, _, _ in order), dtype=np.int64, count=n)
        host[2 * bucket : 2 * bucket + n] = last_blk * bs + starts % bs
        host[2 * bucket + n : 3 * bucket] = -1
        host[3 * bucket : 3 * bucket + n] = starts + 1
        host[3 * bucket + n : 4 * bucket] = 1
        host[4 * bucket : 4 * bucket + n] = np.fromiter((s.seed for s, *_ in order), dtype=np.int64, count=n)
        host[4 * bucket + n : 5 * bucket] = 0
        host[5 * bucket : 5 * bucket + n] = np.fromiter((s.slot for s, *_ in order), dtype=np.int64, count=n)
        host[5 * bucket + n : 6 * bucket] = self._dummy_slot
        table = host[6 * bucket :].reshape(bucket, width)
        table[:] = self.scratch_block
        for j, (seq, _, _, _) in enumerate(order):
            blk = seq.blocks
            table[j, : len(blk)] = blk
        temps = np.zeros(bucket, dtype=np.float32)
        temps[:n] = np.fromiter((float(s.params.temperature) for s, *_ in order), dtype=np.float32, count=n)
        offs = np.zeros(bucket, dtype=np.int64)
        offs[:n] = np.fromiter((len(s.out) + s.pending for s, *_ in order), dtype=np.int64, count=n)
        return {"kind": "graph", "B": B, "bucket": bucket, "width": width, "host": host, "temps": temps, "offs": offs}

    def _run_graph(self, meta):
        g = self._graph_for(meta["bucket"], meta["width"])
        n_meta = g["meta"].numel()
        bk = meta["bucket"]
        host = np.empty(n_meta + 2 * bk, dtype=np.int64)
        host[:n_meta] = meta["host"]
        host[n_meta : n_meta + bk] = meta["offs"]
        host[n_meta + bk :].view(np.float32)[:bk] = meta["temps"]
        d = self._h2d(host)
        g["meta"].copy_(d[:n_meta])
        g["offs"].copy_(d[n_meta : n_meta + bk])
        g["temps"].copy_(d[n_meta + bk :].view(torch.float32)[:bk])
        g["graph"].replay()
        B = meta["B"]
        return self._stage_results(g["tok"][:B], g["lp"][:B])

    def _execute_decode_graph(self, order):
        meta = self._graph_meta(order)
        if meta is None:
            return self._execute(order, 0)
        self._send_step(meta)
        return self._run_graph(meta)

    def _exec_meta(self, order, n_prefill: int) -> Dict[str, Any]:
        """Host inputs of one eager step over ``order`` (first ``n_prefill`` entries are prefill chunks)."""
        bs = self.block_size
        ids_l, pos_l, slots_l, ks_l = [], [], [], []
        sample_rows: List[int] = []
        cu_q = [0]
        cu_k = [0]
        max_q = 1
        rows = 0
        rs_l = []
        for i, (seq, start, n, samples) in enumerate(order):
            blocks = np.asarray(seq.blocks, dtype=np.int64)
            p = np.arange(start, start + n, dtype=np.int64)
            known = seq.toks[start : start + n]
            if len(known) < n:  # the pending token (decode rows only): read from the slot table
                known = known + [-1] * (n - len(known))
            ids_l.append(np.asarray(known, dtype=np.int64))
            rs_l.append(np.full(n, seq.slot if seq.slot >= 0 else self._dummy_slot, dtype=np.int64))
            pos_l.append(p)
            slots_l.append(blocks[p // bs] * bs + p % bs)
            rows += n
            if samples:
                sample_rows.append(rows - 1)
            if i < n_prefill:
                cu_q.append(cu_q[-1] + n)
                ctx = start + n
                cu_k.append(cu_k[-1] + ctx)
                if not self._paged_prefill:  # the CPU path gathers the context keys by slot
                    pk = np.arange(ctx, dtype=np.int64)
                    ks_l.append(blocks[pk // bs] * bs + pk % bs)
                max_q = max(max_q, n)
        empty = np.zeros(0, np.int64)
        ids = np.concatenate(ids_l) if ids_l else empty
        pos = np.concatenate(pos_l) if pos_l else empty
        slots = np.concatenate(slots_l) if slots_l else empty
        k_slots = np.concatenate(ks_l) if ks_l else empty
        row_slots = np.concatenate(rs_l) if rs_l else empty
        decode = order[n_prefill:]
        nd = len(decode)
        header = [len(ids), len(pos), len(slots), len(sample_rows), len(cu_q), len(cu_k), len(k_slots), len(row_slots)]
        flat = np.concatenate([ids, pos, slots, np.asarray(sample_rows, np.int64), np.asarray(cu_q, np.int64),
                               np.asarray(cu_k, np.int64), k_slots, row_slots])
        meta: Dict[str, Any] = {"kind": "exec", "header": header, "flat": flat, "Tp": cu_q[-1], "max_q": max_q,
                                "nd": nd}
        if nd:
            max_blocks = max(len(s.blocks) for s, *_ in decode)
            table = np.zeros((nd, max_blocks), np.int32)
            lens = np.zeros(nd, np.int32)
            for j, (sq, start, n, _) in enumerate(decode):
                table[j, : len(sq.blocks)] = sq.blocks
                lens[j] = start + n
            meta["table"], meta["lens"] = table, lens
        if n_prefill and self._paged_prefill:
            # prefill attention reads its keys from the pages in place: one block-table row per chunk
            pre = order[:n_prefill]
            ptable = np.zeros((n_prefill, max(len(s.blocks) for s, *_ in pre)), np.int32)
            for j, (sq, *_rest) in enumerate(pre):
                ptable[j, : len(sq.blocks)] = sq.blocks
            meta["ptable"] = ptable
        sampled = [e for e in order if e[3]]
        meta["temps"] = np.asarray([float(sq.params.temperature) for sq, *_ in sampled], np.float32)
        meta["seeds"] = np.asarray([sq.seed for sq, *_ in sampled], np.int64)
        meta["offs"] = np.asarray([len(sq.out) + sq.pending for sq, *_ in sampled], np.int64)
        if any(sq.params.top_p < 1.0 or (sq.params.top_k or -1) > 0 for sq, *_ in sampled):
            meta["filter_params"] = [sq.params for sq, *_ in sampled]
        return meta

    def _execute(self, order, n_prefill: int):
        meta = self._exec_meta(order, n_prefill)
        self._send_step(meta)
        return self._run_exec(meta)

    def _run_exec(self, meta):
        cfg = self.cfg
        dev = self.device
        header, Tp, max_q, nd = meta["header"], meta["Tp"], meta["max_q"], meta["nd"]
        ns = len(meta["seeds"])
        parts = [meta["flat"]]
        if nd:
            parts += [meta["table"].reshape(-1).astype(np.int64), meta["lens"].astype(np.int64)]
        ptable = meta.get("ptable")
        if ptable is not None:
            parts.append(ptable.reshape(-1).astype(np.int64))
        tail = np.empty(3 * ns, dtype=np.int64)
        tail[:ns] = meta["seeds"]
        tail[ns : 2 * ns] = meta["offs"]
        tail[2 * ns :].view(np.float32)[:ns] = meta["temps"]
        parts.append(tail)
        big = self._h2d(np.concatenate(parts))
        nflat = meta["flat"].size
        d = big[:nflat]
        rest = big[nflat:]
        off = np.cumsum([0] + header)
        ids_d = d[off[0] : off[1]]
        pos_d = d[off[1] : off[2]]
        slots_d = d[off[2] : off[3]].to(torch.int32)
        rows_d = d[off[3] : off[4]]
        cu_q_d = d[off[4] : off[5]].to(torch.int32)
        cu_k_d = d[off[5] : off[6]].to(torch.int32)
        kslots_d = d[off[6] : off[7]]
        rowslot_d = d[off[7] : off[8]]
        ids_d = torch.where(ids_d >= 0, ids_d, self._slot_tok.index_select(0, rowslot_d))
        if nd:
            max_blocks = meta["table"].shape[1]
            table_d = rest[: nd * max_blocks].view(nd, max_blocks).to(torch.int32)
            lens_d = rest[nd * max_blocks : nd * max_blocks + nd].to(torch.int32)
            rest = rest[nd * max_blocks + nd :]
        ptable_d = None
        if ptable is not None:
            ptable_d = rest[: ptable.size].view(ptable.shape).to(torch.int32)
            rest = rest[ptable.size :]
        seeds_d = rest[:ns]
        offs_d = rest[ns : 2 * ns]
        temps_d = rest[2 * ns :].view(torch.float32)[:ns]
        m = self.model
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        scale = 1.0 / math.sqrt(D)
        splits = self.decode_splits or _decode_splits(nd * Hkv)

        def attn_fn(layer, q, kc, vc):
            attn = torch.empty(q.shape[0], cfg.q_dim, dtype=q.dtype, device=dev)
            if Tp and ptable_d is not None:
                ops.attention_varlen(q[:Tp], kc, vc, cu_q_d, max_q, Hq, Hkv, D, scale=scale, out=attn[:Tp],
                                     cu_seqlens_k=cu_k_d, block_table=ptable_d)
            elif Tp:
                kctx = kc.view(-1, cfg.kv_dim).index_select(0, kslots_d)
                vctx = vc.view(-1, cfg.kv_dim).index_select(0, kslots_d)
                ops.attention_varlen(q[:Tp], kctx, vctx, cu_q_d, max_q, Hq, Hkv, D, scale=scale,
                                     out=attn[:Tp], cu_seqlens_k=cu_k_d)
            if nd:
                ops.paged_decode(q[Tp:], kc, vc, table_d, lens_d, Hq, Hkv, scale, num_splits=splits,
                                 out=attn[Tp:])
            return attn

        with torch.no_grad():
            x = ops.embedding(ids_d, m.w("model.embed_tokens.weight"))
            x = self._forward_layers(x, pos_d, slots_d, attn_fn)
            if header[3] == 0:
                return self._stage_results(torch.zeros(0, dtype=torch.long, device=dev),
                                           torch.zeros(0, dtype=torch.float32, device=dev))
            xs = x.index_select(0, rows_d)
            hN, _ = ops.rmsnorm(xs, m.w("model.norm.weight"), cfg.rms_norm_eps)
            logits = ops.linear(hN, m.w(m.lm_head_name))
            if "filter_params" in meta:
                fp = meta["filter_params"]
                top_k = torch.tensor([max(int(p.top_k or 0), 0) for p in fp], dtype=torch.int32)
                top_p = torch.tensor([float(p.top_p) for p in fp], dtype=torch.float32)
                tokens, lps = ops.sample(logits, temps_d, seeds_d, offs_d, top_k=top_k, top_p=top_p)
            else:
                tokens, lps = ops.sample(logits, temps_d, seeds_d, offs_d)
            self._slot_tok.index_copy_(0, rowslot_d.index_select(0, rows_d), tokens.to(torch.long))
            return self._stage_results(tokens, lps)  # the one device->host copy of the step

    # ------------------------------------------------------------------ tensor-parallel followers
    def _send_step(self, meta) -> None:
        """Leader: hand the step's host inputs to the follower ranks before running it."""
        if self.tp > 1 and self.tp_rank == 0:
            self._cmd(("step", meta))

    def _cmd(self, msg) -> None:
        import torch.distributed as dist

        obj = [msg]
        dist.broadcast_object_list(obj, src=self._cmd_src, group=self.cmd_group)

    def serve_follower(self) -> None:
        """Follower ranks: run every step, weight pull and cache command the leader broadcasts, until
        ``stop``. Sampled tokens are computed (the math is replicated) and discarded."""
        import torch.distributed as dist

        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        while True:
            obj = [None]
            dist.broadcast_object_list(obj, src=self._cmd_src, group=self.cmd_group)
            kind, payload = obj[0]
            if kind == "stop":
                return
            if kind == "step":
                if payload["kind"] == "graph":
                    _, _, ev = self._run_graph(payload)
                else:
                    _, _, ev = self._run_exec(payload)
                if ev is not None:
                    ev.synchronize()  # the result buffers are reused a few steps later
                if self._tp_ar is not None:
                    self._tp_ar.check()
            elif kind == "pull":
                self._pull_local(payload)
                dist.barrier(group=self.cmd_group)
            elif kind == "clear_graphs":
                self._graphs.clear()

    def stop_followers(self) -> None:
        with self._step_lock:
            if self.tp > 1 and self.tp_rank == 0 and not self._followers_stopped:
                self._followers_stopped = True
                self._cmd(("stop", None))

    def _complete(self, launched) -> None:
        """Apply the samples of a launched step: append tokens, register full prefix blocks, finish
        sequences that stop (rows of already-finished sequences are discarded)."""
        bs = self.block_size
        for order, (buf, n, ev) in launched["parts"]:
            if ev is not None:
                ev.synchronize()
            vals = buf.tolist()
            it = iter(zip(vals[0], vals[1]))
            with self._lock:
                for seq, start, nn, samples in order:
                    if samples:
                        tok, lp = next(it)
                    if seq.finish_reason is not None:
                        continue
                    # register newly completed full blocks (known tokens only) for prefix reuse
                    toks = seq.toks
                    while len(seq.hashes) < min(seq.num_computed, len(toks)) // bs and len(seq.hashes) < len(seq.blocks):
                        i = len(seq.hashes)
                        parent = seq.hashes[-1] if seq.hashes else None
                        h = block_hash(parent, toks[i * bs : (i + 1) * bs])
                        seq.hashes.append(h)
                        self.allocator.register(seq.blocks[i], h)
                    if not samples:
                        continue
                    seq.pending -= 1
                    seq.append(int(tok), float(lp), self.version)
                    self.stats["generated_tokens"] += 1
                    reason = self._stop_reason(seq, int(tok))
                    if reason is not None:
                        self._finish(seq, reason)
                    elif seq.params.output_kind != "final_only":
                        self._deliver(seq, False)
        if self._tp_ar is not None:
            self._tp_ar.check()

    def _stop_reason(self, seq: _Seq, tok: int) -> Optional[str]:
        p = seq.params
        if not p.ignore_eos and tok in self.eos_ids:
            return "stop"
        if p.stop_token_ids and tok in p.stop_token_ids:
            return "stop"
        if p.stop and self.tokenizer is not None:
            window = max(8, max(len(x) for x in p.stop) + 2)
            tail = self.tokenizer.decode(seq.out[-window:], skip_special_tokens=p.skip_special_tokens)
            if any(s in tail for s in p.stop):
                return "stop"
        if len(seq.out) >= p.max_tokens or seq.length >= self.max_model_len:
            return "length"
        return None


def _decode_splits(ctas_per_split: int) -> int:
    """Sequence splits of the paged decode kernel: about 4 CTAs per SM (148 SMs), at most 16."""
    return max(1, min(16, -(-4 * 148 // max(ctas_per_split, 1))))
