"""Versioned generation that survives weight-update pauses.

Behaviour being provided (the reference's ``InterruptibleGenerationRunner``,
accerl_agent/agent_textworld.py:1773-1913, and ``LocalRolloutEngine``,
accerl_agent/vllm_local_rollout_engine.py:135-326): a request keeps every token it has produced
across a trainer->engine weight sync, each token is tagged with the policy version that sampled it,
no request ever gets more than its token budget, and the trainer can pause generation and wait until
no submission is in flight.

Two kinds of engines are served by one submission loop (``ResumableFrontEnd.drive``):

* The native paged-KV engine (``rollout/engine.py``) *suspends*: ``pause_generation(mode="suspend")``
  parks its sequences (KV blocks released, tokens kept) and ``resume_generation(version=v)``
  re-admits them, recomputing prompt + tokens so far under the new weights; the engine tags every
  sampled token with its version (``CompletionOutput.token_versions``). A request is then a single
  submission.
* vLLM-shaped engines (and the test fakes) *abort*: a pause ends in-flight submissions with finish
  reason ``abort``. The loop keeps the partial tokens, waits for the gate to reopen and submits
  ``prompt + tokens so far`` for the remaining budget, tagging the new tokens with the version current
  at that submission.

Both front-ends, ``InterruptibleGenerationRunner`` (the inference service's, strict about
log-probabilities) and ``LocalRolloutEngine`` in ``local_engine.py`` (lenient, with latency metrics
and a progress callback), are thin subclasses that choose sampling arguments and log-probability
handling.
"""

from __future__ import annotations

import asyncio
import logging
import uuid
from dataclasses import dataclass, field
from typing import Any, Dict, List, Literal, Optional

StopReason = Literal["length", "stop", "tool_calls", "abort"]
_TERMINAL = ("stop", "tool_calls", "length")

log = logging.getLogger(__name__)


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

    def absorb(self, tokens: List[int], logprobs: List[float], versions: List[int]) -> None:
        self.output_tokens += tokens
        self.output_logprobs += logprobs
        self.output_versions += versions


@dataclass
class InferenceResult:
    output_tokens: List[int]
    output_logprobs: List[float]
    output_versions: List[int]
    stop_reason: Optional[StopReason]


def normalize_stop_reason(reason) -> StopReason:
    """Map an engine finish reason onto the four reasons a sample records."""
    if reason in ("length", "stop", "tool_calls", "abort"):
        return reason
    return "stop" if reason in ("eos", "stop_token", "stop_sequence") else "abort"


def _entry_logprob(entry, token: int) -> Optional[float]:
    """One sampled-token log-probability from a vLLM-style entry: a float, an object with
    ``.logprob``, or a ``{token: value}`` dict (keys may be ints or strings)."""
    if isinstance(entry, dict):
        entry = entry[token] if token in entry else entry.get(str(token))
    if entry is None:
        return None
    return float(getattr(entry, "logprob", entry))


@dataclass
class _Completion:
    """What one submission left behind: its last output, reduced to the fields the loop uses."""

    tokens: List[int]
    raw_logprobs: List[Any]
    finish: StopReason
    versions: Optional[List[int]]

    @staticmethod
    def of(request_output) -> "_Completion":
        outs = getattr(request_output, "outputs", None) or []
        if not outs:
            return _Completion([], [], "abort", None)
        o = outs[0]
        versions = getattr(o, "token_versions", None)
        return _Completion(list(getattr(o, "token_ids", None) or []), list(getattr(o, "logprobs", None) or []),
                           normalize_stop_reason(getattr(o, "finish_reason", None)),
                           list(versions) if versions is not None else None)


class ResumableFrontEnd:
    """Submission loop shared by the generation front-ends (see the module docstring).

    A gate (``pause``/``resume``) holds back new submissions; ``wait_for_idle`` returns once no
    submission is in flight. Subclasses provide ``sampling_kwargs`` and ``read_logprobs`` and may
    observe streamed outputs with ``on_stream``."""

    # a request whose budget is spent reports "length" even when the engine said "stop"
    budget_overrides_reason = True

    def __init__(self, engine, max_attempts: int, sampling_params_cls=None):
        self.engine = engine
        self.max_attempts = max_attempts
        self.sampling_params_cls = sampling_params_cls or SamplingParams
        self.version = 0
        self._open = asyncio.Event()
        self._open.set()
        self._idle = asyncio.Event()
        self._idle.set()
        self._in_flight = 0

    # ---- gate
    def pause(self) -> None:
        self._open.clear()

    def resume(self) -> None:
        self._open.set()

    async def wait_for_idle(self) -> None:
        await self._idle.wait()

    @property
    def active_attempts(self) -> int:
        return self._in_flight

    # ---- hooks
    def sampling_kwargs(self, budget: int, ctx) -> Dict[str, Any]:
        raise NotImplementedError

    def read_logprobs(self, done: _Completion, tokens: List[int]) -> Optional[List[float]]:
        """Log-probabilities of ``tokens``; None voids the submission (it then counts as aborted)."""
        raise NotImplementedError

    async def on_stream(self, ctx, request_output, already: int, budget: int, version: int) -> None:
        return None

    def on_absorbed(self, ctx, n_new: int) -> None:
        return None

    async def between_attempts(self) -> None:
        await asyncio.sleep(0)

    # ---- loop
    def _params(self, budget: int, ctx):
        kwargs = self.sampling_kwargs(budget, ctx)
        if self.sampling_params_cls is SamplingParams:
            kwargs["output_kind"] = "final_only"  # only the last output of a submission is used
        return self.sampling_params_cls(**kwargs)

    async def _submit(self, state: OnlineGenerationState, budget: int, version: int, request_id: str, ctx):
        already = len(state.output_tokens)
        last = None
        self._in_flight += 1
        self._idle.clear()
        try:
            async for out in self.engine.generate({"prompt_token_ids": state.restart_prompt_token_ids},
                                                  self._params(budget, ctx), request_id=request_id):
                last = out
                await self.on_stream(ctx, out, already, budget, version)
        except asyncio.CancelledError:
            raise
        except Exception:
            if self._open.is_set():
                raise
            last = None  # the engine failed the submission while paused: same as an abort
        finally:
            self._in_flight -= 1
            if self._in_flight == 0:
                self._idle.set()
        return None if last is None else _Completion.of(last)

    async def drive(self, state: OnlineGenerationState, tag: str, ctx=None) -> OnlineGenerationState:
        for attempt in range(1, self.max_attempts + 1):
            await self._open.wait()
            budget = state.remaining_max_tokens
            if budget <= 0:
                state.stop_reason = "length"
                return state
            version = self.version
            done = await self._submit(state, budget, version, f"{tag}-v{version}-a{attempt}-{uuid.uuid4().hex[:10]}",
                                      ctx)
            lps = None
            if done is not None:
                tokens = done.tokens[:budget]
                lps = self.read_logprobs(done, tokens) if tokens else []
            if lps is None:
                state.stop_reason = "abort"
                await self.between_attempts()
                continue
            versions = done.versions[: len(tokens)] if done.versions is not None else [version] * len(tokens)
            state.absorb(tokens, lps, versions)
            self.on_absorbed(ctx, len(tokens))
            spent = state.remaining_max_tokens <= 0
            if spent and (self.budget_overrides_reason or done.finish not in _TERMINAL):
                state.stop_reason = "length"
            else:
                state.stop_reason = done.finish
            if state.stop_reason in _TERMINAL:
                return state
            await self.between_attempts()
        state.stop_reason = "length" if state.remaining_max_tokens <= 0 else "abort"
        log.warning("request %s: no completion after %d submissions; returning the %d tokens produced",
                    tag, self.max_attempts, len(state.output_tokens))
        return state


class InterruptibleGenerationRunner(ResumableFrontEnd):
    """The inference service's front-end: fixed temperature / top-p / stop strings for every
    request, and, with ``collect_logprobs``, a submission whose log-probabilities do not cover every
    token counts as aborted (so every trained token has its behaviour log-probability)."""

    def __init__(self, engine, temperature: float = 0.7, top_p: float = 0.9,
                 stop_sequences: Optional[List[str]] = None, collect_logprobs: bool = False,
                 max_resubmit_retries: int = 200, sampling_params_cls=SamplingParams):
        super().__init__(engine, max_resubmit_retries, sampling_params_cls)
        self.temperature = temperature
        self.top_p = top_p
        self.stop_sequences = stop_sequences or ["</answer>"]
        self.collect_logprobs = collect_logprobs

    @property
    def max_resubmit_retries(self) -> int:
        return self.max_attempts

    def sampling_kwargs(self, budget: int, ctx=None) -> Dict[str, Any]:
        kw: Dict[str, Any] = {"temperature": self.temperature, "top_p": self.top_p, "max_tokens": budget,
                              "stop": self.stop_sequences}
        if self.collect_logprobs:
            kw["logprobs"] = 1
        return kw

    def read_logprobs(self, done: _Completion, tokens: List[int]) -> Optional[List[float]]:
        if not self.collect_logprobs:
            return []
        if len(done.raw_logprobs) < len(tokens):
            return None
        out = [_entry_logprob(e, t) for e, t in zip(done.raw_logprobs, tokens)]
        return None if any(v is None for v in out) else out

    async def generate(self, state: OnlineGenerationState) -> OnlineGenerationState:
        return await self.drive(state, f"req{state.index}")
