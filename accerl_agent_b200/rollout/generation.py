"""Interruptible, versioned generation on top of any async token engine.

An engine exposes ``async generate({"prompt_token_ids": ids}, sampling_params, request_id=...)``
yielding request outputs (``.finished``, ``.outputs[0].token_ids / .finish_reason / .logprobs``),
``pause_generation(mode="abort", clear_cache=True)`` and ``resume_generation()``. The native paged-KV
engine (``rollout/engine.py``) and the test fakes implement exactly that surface.

``InterruptibleGenerationRunner`` (agent_textworld.py:1773-1913) keeps per-request token state across
weight-update pauses: every attempt waits for the resume event, resubmits ``prompt + partial output``
with ``max_tokens = remaining`` and tags each new token with the policy version current at attempt
start. Aborted attempts are resubmitted up to ``max_resubmit_retries`` times; exceptions raised while
paused count as aborts. An active-attempt counter under a condition lets ``wait_for_idle`` drain.
"""

from __future__ import annotations

import asyncio
import uuid
from dataclasses import dataclass, field
from typing import Any, List, Literal, Optional

StopReason = Literal["length", "stop", "tool_calls", "abort"]


@dataclass
class SamplingParams:
    """Sampling controls understood by the native engine (a subset of vLLM's ``SamplingParams``)."""

    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = -1
    max_tokens: int = 16
    stop: Optional[List[str]] = None
    stop_token_ids: Optional[List[int]] = None
    ignore_eos: bool = False
    logprobs: Optional[int] = None
    skip_special_tokens: bool = True
    frequency_penalty: float = 0.0
    seed: Optional[int] = None
    # "cumulative": a RequestOutput after every step (streaming); "final_only": only the finished
    # (or aborted) output, which saves the per-step hand-off for callers that use only the last one
    output_kind: str = "cumulative"

    def __init__(self, **kwargs: Any):
        for name, default in (
            ("temperature", 1.0), ("top_p", 1.0), ("top_k", -1), ("max_tokens", 16), ("stop", None),
            ("stop_token_ids", None), ("ignore_eos", False), ("logprobs", None), ("skip_special_tokens", True),
            ("frequency_penalty", 0.0), ("seed", None), ("output_kind", "cumulative"),
        ):
            setattr(self, name, kwargs.pop(name, default))
        kwargs.pop("use_beam_search", None)
        if kwargs:
            raise TypeError(f"Unsupported sampling parameters: {sorted(kwargs)}")
        if self.top_k is not None and self.top_k >= 10**7:
            self.top_k = -1


@dataclass
class OnlineGenerationState:
    """Token-level state of one request across weight-update interruptions."""

    index: int
    input_ids: List[int]
    requested_max_tokens: int
    output_tokens: List[int] = field(default_factory=list)
    output_logprobs: List[float] = field(default_factory=list)
    output_versions: List[int] = field(default_factory=list)
    stop_reason: Optional[StopReason] = None

    @property
    def remaining_max_tokens(self) -> int:
        return max(0, self.requested_max_tokens - len(self.output_tokens))

    @property
    def restart_prompt_token_ids(self) -> List[int]:
        return self.input_ids + self.output_tokens


@dataclass
class InferenceResult:
    output_tokens: List[int]
    output_logprobs: List[float]
    output_versions: List[int]
    stop_reason: Optional[StopReason]


def tokens_from_output(request_output) -> List[int]:
    if not getattr(request_output, "outputs", None):
        return []
    return list(getattr(request_output.outputs[0], "token_ids", []) or [])


def logprobs_from_output(request_output, token_ids: List[int]) -> List[float]:
    """Sampled-token logprobs; returns ``[]`` when any is missing (the attempt then counts as aborted)."""
    if not getattr(request_output, "outputs", None):
        return []
    raw = getattr(request_output.outputs[0], "logprobs", None) or []
    out: List[float] = []
    for token_id, entry in zip(token_ids, raw):
        value = entry
        if isinstance(entry, dict):
            value = entry.get(token_id)
            if value is None:
                value = entry.get(str(token_id))
        if hasattr(value, "logprob"):
            value = value.logprob
        if value is None:
            return []
        out.append(float(value))
    return out


def finish_reason_from_output(request_output):
    if not getattr(request_output, "outputs", None):
        return None
    return getattr(request_output.outputs[0], "finish_reason", None)


def normalize_stop_reason(reason) -> StopReason:
    if reason in ("length", "stop", "tool_calls", "abort"):
        return reason
    if reason in ("eos", "stop_token", "stop_sequence"):
        return "stop"
    return "abort"


class InterruptibleGenerationRunner:
    def __init__(
        self,
        engine,
        temperature: float = 0.7,
        top_p: float = 0.9,
        stop_sequences: Optional[List[str]] = None,
        collect_logprobs: bool = False,
        max_resubmit_retries: int = 200,
        sampling_params_cls=SamplingParams,
    ):
        self.engine = engine
        self.temperature = temperature
        self.top_p = top_p
        self.stop_sequences = stop_sequences or ["</answer>"]
        self.collect_logprobs = collect_logprobs
        self.max_resubmit_retries = max_resubmit_retries
        self.sampling_params_cls = sampling_params_cls
        self.version = 0
        self.resume_event = asyncio.Event()
        self.resume_event.set()
        self._active_attempts = 0
        self._active_changed = asyncio.Condition()

    def pause(self) -> None:
        self.resume_event.clear()

    def resume(self) -> None:
        self.resume_event.set()

    async def _change_active(self, delta: int) -> None:
        async with self._active_changed:
            self._active_attempts += delta
            self._active_changed.notify_all()

    async def wait_for_idle(self) -> None:
        async with self._active_changed:
            await self._active_changed.wait_for(lambda: self._active_attempts == 0)

    @property
    def active_attempts(self) -> int:
        return self._active_attempts

    async def generate(self, state: OnlineGenerationState) -> OnlineGenerationState:
        for attempt in range(1, self.max_resubmit_retries + 1):
            await self.resume_event.wait()
            remaining = state.remaining_max_tokens
            if remaining <= 0:
                state.stop_reason = "length"
                return state
            attempt_version = self.version
            kwargs = {
                "temperature": self.temperature,
                "top_p": self.top_p,
                "max_tokens": remaining,
                "stop": self.stop_sequences,
            }
            if self.collect_logprobs:
                kwargs["logprobs"] = 1
            if self.sampling_params_cls is SamplingParams:
                kwargs["output_kind"] = "final_only"  # only the last output of an attempt is used
            params = self.sampling_params_cls(**kwargs)
            request_id = f"online-sync-{state.index}-v{attempt_version}-try{attempt}-{uuid.uuid4()}"
            final_output = None
            finished = False
            await self._change_active(+1)
            try:
                async for out in self.engine.generate(
                    {"prompt_token_ids": state.restart_prompt_token_ids}, params, request_id=request_id
                ):
                    final_output = out
                    finished = bool(getattr(out, "finished", False))
            except asyncio.CancelledError:
                raise
            except Exception:
                if self.resume_event.is_set():
                    raise
                final_output = None
            finally:
                await self._change_active(-1)

            if final_output is None:
                state.stop_reason = "abort"
                continue
            tokens = tokens_from_output(final_output)[:remaining]
            if tokens:
                logprobs: List[float] = []
                if self.collect_logprobs:
                    logprobs = logprobs_from_output(final_output, tokens)[: len(tokens)]
                    if len(logprobs) != len(tokens):
                        state.stop_reason = "abort"
                        continue
                state.output_tokens.extend(tokens)
                state.output_logprobs.extend(logprobs)
                state.output_versions.extend([attempt_version] * len(tokens))
            reason = normalize_stop_reason(finish_reason_from_output(final_output))
            if len(state.output_tokens) >= state.requested_max_tokens:
                reason = "length"
            state.stop_reason = reason
            if reason in ("stop", "tool_calls", "length"):
                return state
            if not finished or reason == "abort":
                await asyncio.sleep(0)
                continue
            return state
        state.stop_reason = "length" if state.remaining_max_tokens <= 0 else "abort"
        print(
            f"[generate] Request {state.index} reached max_resubmit_retries={self.max_resubmit_retries}; "
            "keeping partial output."
        )
        return state
