"""Reusable rollout front-end with token-level abort/resubmit handling and latency metrics.

``LocalRolloutEngine.agenerate(RolloutRequest) -> RolloutResponse`` has the behaviour of the
reference's ``vllm_local_rollout_engine.py:135-326``: prompt + partial continuation after aborts,
per-token versions, never more than ``max_new_tokens`` tokens, TTFT / inter-token latency / total
latency, an optional ``on_token_update(req, output_len, version)`` progress callback, and the
``pause_generation -> update_weights(path) -> continue_generation`` lifecycle (``update_weights``
asks the engine to ``reload_weights`` from an HF checkpoint directory and bumps the version).

The engine is any object with the async surface described in ``rollout/generation.py``; the sampling
parameter class is injectable so tests can record the arguments.
"""

from __future__ import annotations

import asyncio
import inspect
import time
import uuid
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional

from .generation import (
    SamplingParams,
    StopReason,
    finish_reason_from_output,
    normalize_stop_reason,
    tokens_from_output,
)


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
        values = asdict(self)
        values.update(kwargs)
        return GenerationConfig(**values)


@dataclass
class RolloutRequest:
    rid: str = field(default_factory=lambda: str(uuid.uuid4()))
    input_ids: List[int] = field(default_factory=list)
    gconfig: GenerationConfig = field(default_factory=GenerationConfig)
    metadata: Dict[str, Any] = field(default_factory=dict)
    tokenizer: Any = None

    def copy(self) -> "RolloutRequest":
        return RolloutRequest(
            rid=self.rid,
            input_ids=list(self.input_ids),
            gconfig=self.gconfig.new(),
            metadata=dict(self.metadata),
            tokenizer=self.tokenizer,
        )


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


def _stream_logprobs(request_output, token_ids: List[int]) -> List[float]:
    """Lenient logprob extraction: missing entries become 0.0 (vllm_local_rollout_engine.py:105-132)."""
    if not getattr(request_output, "outputs", None):
        return []
    raw = getattr(request_output.outputs[0], "logprobs", None)
    if not raw:
        return [0.0] * len(token_ids)
    parsed: List[float] = []
    for token_id, entry in zip(token_ids, raw):
        value = 0.0
        if isinstance(entry, dict):
            item = entry.get(token_id)
            if item is None and entry:
                item = next(iter(entry.values()))
            if item is not None:
                value = float(getattr(item, "logprob", item))
        elif entry is not None:
            value = float(getattr(entry, "logprob", entry))
        parsed.append(value)
    if len(parsed) < len(token_ids):
        parsed.extend([0.0] * (len(token_ids) - len(parsed)))
    return parsed[: len(token_ids)]


class LocalRolloutEngine:
    def __init__(self, async_llm_engine, max_resubmit_retries: int = 20, resubmit_wait: float = 0.0, sampling_params_cls=None):
        self.engine = async_llm_engine
        self.version = 0
        self.paused = asyncio.Event()
        self.max_resubmit_retries = max_resubmit_retries
        self.resubmit_wait = resubmit_wait
        self._sampling_params_cls = sampling_params_cls or SamplingParams

    async def agenerate(self, request: RolloutRequest) -> RolloutResponse:
        req = request.copy() if hasattr(request, "copy") else request
        g = req.gconfig
        if g.n_samples != 1:
            raise ValueError("LocalRolloutEngine only supports n_samples=1; call agenerate once per sample.")
        max_new = min(g.max_tokens - len(req.input_ids), g.max_new_tokens)
        if max_new <= 0:
            raise RuntimeError(
                f"max_new_tokens ({max_new}) is non-positive: max_tokens={g.max_tokens}, "
                f"input_len={len(req.input_ids)}, configured_max_new_tokens={g.max_new_tokens}."
            )
        start = time.perf_counter()
        last_token_time: Optional[float] = None
        ttft = float("inf")
        itl: List[float] = []
        tokens: List[int] = []
        logprobs: List[float] = []
        versions: List[int] = []
        stop_reason: Optional[StopReason] = None
        for attempt in range(1, self.max_resubmit_retries + 1):
            while self.paused.is_set():
                await asyncio.sleep(self.resubmit_wait)
            remaining = max_new - len(tokens)
            if remaining <= 0:
                stop_reason = "length"
                break
            version = self.version
            params = self._make_sampling_params(g, remaining)
            request_id = f"{req.rid}-v{version}-try{attempt}-{uuid.uuid4()}"
            final = None
            finished = False
            async for out in self.engine.generate(
                {"prompt_token_ids": list(req.input_ids) + tokens}, params, request_id=request_id
            ):
                final = out
                finished = bool(getattr(out, "finished", False))
                streamed = tokens_from_output(out)[:remaining]
                await self._notify_progress(req, len(tokens) + len(streamed), version)
            if final is None:
                stop_reason = "abort"
                continue
            new_tokens = tokens_from_output(final)[:remaining]
            new_logprobs = _stream_logprobs(final, new_tokens)
            now = time.perf_counter()
            if new_tokens:
                if ttft == float("inf"):
                    ttft = now - start
                if last_token_time is not None:
                    itl.append(now - last_token_time)
                if len(new_tokens) > 1:
                    itl.extend([0.0] * (len(new_tokens) - 1))
                last_token_time = now
            tokens.extend(new_tokens)
            logprobs.extend(new_logprobs)
            versions.extend([version] * len(new_tokens))
            stop_reason = normalize_stop_reason(finish_reason_from_output(final))
            if stop_reason in ("stop", "tool_calls", "length"):
                break
            if len(tokens) >= max_new:
                stop_reason = "length"
                break
            if not finished or stop_reason == "abort":
                await asyncio.sleep(self.resubmit_wait)
                continue
            break
        else:
            stop_reason = "length" if len(tokens) >= max_new else "abort"
        if stop_reason == "abort" and len(tokens) >= max_new:
            stop_reason = "length"
        if stop_reason is None:
            stop_reason = "length" if len(tokens) >= max_new else "abort"
        return RolloutResponse(
            input_tokens=list(request.input_ids),
            output_tokens=tokens,
            output_logprobs=logprobs,
            output_versions=versions,
            stop_reason=stop_reason,
            tokenizer=getattr(request, "tokenizer", None),
            latency=time.perf_counter() - start,
            ttft=ttft,
            itl=itl,
        )

    async def _notify_progress(self, req: RolloutRequest, output_len: int, version: int) -> None:
        callback = getattr(req, "metadata", {}).get("on_token_update")
        if callback is None:
            return
        result = callback(req, output_len, version)
        if inspect.isawaitable(result):
            await result

    async def pause_generation(self) -> None:
        self.paused.set()
        await self.engine.pause_generation(mode="abort", clear_cache=True)

    async def update_weights(self, path: str) -> None:
        await self.engine.collective_rpc("reload_weights", kwargs={"weights_path": path, "is_checkpoint_format": True})
        self.version += 1

    async def continue_generation(self) -> None:
        await self.engine.resume_generation()
        self.paused.clear()

    def _make_sampling_params(self, g: GenerationConfig, max_tokens: int):
        kwargs = {
            "temperature": 0.0 if g.greedy else g.temperature,
            "top_p": g.top_p,
            "top_k": g.top_k,
            "max_tokens": max_tokens,
            "stop_token_ids": g.stop_token_ids,
            "ignore_eos": g.ignore_eos,
            "skip_special_tokens": g.skip_special_tokens,
            "frequency_penalty": g.frequency_penalty,
            "logprobs": 0,
        }
        if g.stop:
            kwargs["stop"] = g.stop
        if g.use_beam_search:
            kwargs["use_beam_search"] = True
        return self._sampling_params_cls(**kwargs)
