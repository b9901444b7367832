"""Reusable rollout front-end with latency metrics: ``LocalRolloutEngine.agenerate(RolloutRequest)``.

Behaviour being provided (accerl_agent/vllm_local_rollout_engine.py:135-326): one sample per call,
prompt + partial continuation after a pause, per-token policy versions, never more than
``max_new_tokens`` tokens, time to first token, inter-token latencies and total latency, an optional
``metadata["on_token_update"](request, output_len, version)`` progress callback (sync or async), and
the ``pause_generation -> update_weights(path) -> continue_generation`` lifecycle, where
``update_weights`` asks the engine to ``reload_weights`` from an HF checkpoint directory.

The submission loop is ``generation.ResumableFrontEnd.drive``; this class only maps a
``GenerationConfig`` onto sampling arguments, reads log-probabilities leniently (a missing entry
counts as 0.0 instead of voiding the submission) and keeps the per-request metrics. Inter-token
latencies are measured between token arrivals of the stream: tokens that arrive in one output are
0 s apart.
"""

from __future__ import annotations

import asyncio
import inspect
import time
import uuid
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

from .generation import OnlineGenerationState, ResumableFrontEnd, SamplingParams, StopReason, _entry_logprob


@dataclass
class GenerationConfig:
    n_samples: int = 1
    max_new_tokens: int = 16384
    min_new_tokens: int = 0
    max_tokens: int = 32768
    greedy: bool = False
    top_p: float = 1.0
    top_k: int = int(1e8)
    temperature: float = 1.0
    stop_token_ids: List[int] = field(default_factory=list)
    ignore_eos: bool = False
    skip_special_tokens: bool = True
    stop: Optional[List[str]] = None
    frequency_penalty: float = 0.0
    use_beam_search: bool = False

    def new(self, **kwargs) -> "GenerationConfig":
        return GenerationConfig(**{**asdict(self), **kwargs})


@dataclass
class RolloutRequest:
    rid: str = field(default_factory=lambda: str(uuid.uuid4()))
    input_ids: List[int] = field(default_factory=list)
    gconfig: GenerationConfig = field(default_factory=GenerationConfig)
    metadata: Dict[str, Any] = field(default_factory=dict)
    tokenizer: Any = None

    def copy(self) -> "RolloutRequest":
        return RolloutRequest(rid=self.rid, input_ids=list(self.input_ids), gconfig=self.gconfig.new(),
                              metadata=dict(self.metadata), tokenizer=self.tokenizer)


@dataclass
class RolloutResponse:
    input_tokens: List[int] = field(default_factory=list)
    output_tokens: List[int] = field(default_factory=list)
    output_logprobs: List[float] = field(default_factory=list)
    output_versions: List[int] = field(default_factory=list)
    stop_reason: StopReason = "stop"
    tokenizer: Any = None
    latency: float = float("inf")
    ttft: float = float("inf")
    itl: List[float] = field(default_factory=list)


@dataclass
class _Clock:
    """Per-request timing: arrival times of streamed tokens."""

    request: RolloutRequest
    start: float
    seen: int = 0  # tokens of the current submission already timed
    first: Optional[float] = None
    last: Optional[float] = None
    gaps: List[float] = field(default_factory=list)

    def arrived(self, n_new: int, now: float) -> None:
        if n_new <= 0:
            return
        if self.first is None:
            self.first = now - self.start
        if self.last is not None:
            self.gaps.append(now - self.last)
        self.gaps += [0.0] * (n_new - 1)
        self.last = now


class LocalRolloutEngine(ResumableFrontEnd):
    budget_overrides_reason = False  # keep the engine's own terminal reason at the budget
    def __init__(self, async_llm_engine, max_resubmit_retries: int = 20, resubmit_wait: float = 0.0,
                 sampling_params_cls=None):
        super().__init__(async_llm_engine, max_resubmit_retries, sampling_params_cls or SamplingParams)
        self.resubmit_wait = resubmit_wait
        self.paused = asyncio.Event()  # set while generation is paused

    # ---- lifecycle
    async def pause_generation(self) -> None:
        self.paused.set()
        self.pause()
        await self.engine.pause_generation(mode="abort", clear_cache=True)

    async def update_weights(self, path: str) -> None:
        await self.engine.collective_rpc("reload_weights", kwargs={"weights_path": path, "is_checkpoint_format": True})
        self.version += 1

    async def continue_generation(self) -> None:
        await self.engine.resume_generation()
        self.paused.clear()
        self.resume()

    # ---- hooks of the submission loop
    def sampling_kwargs(self, budget: int, clock: "_Clock") -> Dict[str, Any]:
        g = clock.request.gconfig
        kw: Dict[str, Any] = {
            "temperature": 0.0 if g.greedy else g.temperature, "top_p": g.top_p, "top_k": g.top_k,
            "max_tokens": budget, "stop_token_ids": g.stop_token_ids, "ignore_eos": g.ignore_eos,
            "skip_special_tokens": g.skip_special_tokens, "frequency_penalty": g.frequency_penalty, "logprobs": 0,
        }
        if g.stop:
            kw["stop"] = g.stop
        if g.use_beam_search:
            kw["use_beam_search"] = True
        return kw

    def read_logprobs(self, done, tokens: List[int]) -> List[float]:
        raw = done.raw_logprobs
        vals = []
        for i, t in enumerate(tokens):
            v = None
            if i < len(raw) and raw[i] is not None:
                e = raw[i]
                v = _entry_logprob(e, t)
                if v is None and isinstance(e, dict) and e:
                    v = _entry_logprob(next(iter(e.values())), t)
            vals.append(0.0 if v is None else v)
        return vals

    async def on_stream(self, clock: _Clock, request_output, already: int, budget: int, version: int) -> None:
        outs = getattr(request_output, "outputs", None) or []
        n = min(len(getattr(outs[0], "token_ids", None) or []), budget) if outs else 0
        clock.arrived(n - clock.seen, time.perf_counter())
        clock.seen = max(clock.seen, n)
        callback = clock.request.metadata.get("on_token_update")
        if callback is not None:
            result = callback(clock.request, already + n, version)
            if inspect.isawaitable(result):
                await result

    def on_absorbed(self, clock: _Clock, n_new: int) -> None:
        clock.seen = 0  # the next submission streams from zero again

    async def between_attempts(self) -> None:
        await asyncio.sleep(self.resubmit_wait)

    # ---- public call
    async def agenerate(self, request: RolloutRequest) -> RolloutResponse:
        req = request.copy() if hasattr(request, "copy") else request
        g = req.gconfig
        if g.n_samples != 1:
            raise ValueError("LocalRolloutEngine only supports n_samples=1; call agenerate once per sample.")
        budget = min(g.max_tokens - len(req.input_ids), g.max_new_tokens)
        if budget <= 0:
            raise RuntimeError(
                f"max_new_tokens ({budget}) is non-positive: max_tokens={g.max_tokens}, "
                f"input_len={len(req.input_ids)}, configured_max_new_tokens={g.max_new_tokens}."
            )
        clock = _Clock(req, time.perf_counter())
        state = OnlineGenerationState(index=0, input_ids=list(req.input_ids), requested_max_tokens=budget)
        state = await self.drive(state, str(req.rid), clock)
        return RolloutResponse(
            input_tokens=list(request.input_ids), output_tokens=state.output_tokens,
            output_logprobs=state.output_logprobs, output_versions=state.output_versions,
            stop_reason=state.stop_reason or "abort", tokenizer=getattr(request, "tokenizer", None),
            latency=time.perf_counter() - clock.start, ttft=clock.first if clock.first is not None else float("inf"),
            itl=clock.gaps,
        )
