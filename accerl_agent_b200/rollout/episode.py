"""Episode transcripts to ``RLSample`` (the sample format of agent_textworld.py:2488-2588).

An episode is a chain of requests whose prompts extend one another: each request's prompt is the
previous prompt plus the previous response plus the new observation. The builder turns the chain
into a list of segments of the final transcript,

    context   -- prompt tokens nobody sampled here (the new observation), and the tokens of an
                 aborted generation: not trained;
    response  -- a completed generation: trained on its own tokens with the behaviour
                 log-probabilities and weight versions the engine reported,

checks that every prompt starts with the transcript so far (an episode whose history was re-rendered
cannot be trained on token by token and is dropped), and lays the segments out as the sample's
per-token arrays. The n-th response segment has response index n. Advantages: PPO places each
step's reward on the last token of its response and turns the token rewards into Monte-Carlo
returns; GRPO gives every trained token the episode's group advantage. A transcript longer than
the history window, or one with nothing to train, yields no sample.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

from ..algo.advantages import token_level_returns
from ..core.sample import IGNORE_INDEX, RLSample
from .generation import InferenceResult


@dataclass
class StepRecord:
    training_result: InferenceResult
    prompt_ids: List[int]
    reward: float


@dataclass
class _Segment:
    tokens: Sequence[int]
    trained: bool
    logprobs: Sequence[float] = ()
    versions: Sequence[int] = ()
    reward: float = 0.0  # PPO: the step reward, on the segment's last token


def _segments(records: List[StepRecord]) -> Optional[List[_Segment]]:
    """The transcript as segments, or None when a prompt does not extend it or a response's
    log-probabilities / versions do not cover its tokens."""
    segs: List[_Segment] = []
    length = 0
    transcript: List[int] = []
    for rec in records:
        prompt = rec.prompt_ids
        if len(prompt) < length or prompt[:length] != transcript:
            return None
        if len(prompt) > length:
            segs.append(_Segment(prompt[length:], trained=False))
            transcript.extend(prompt[length:])
            length = len(prompt)
        res = rec.training_result
        toks = list(res.output_tokens)
        if not toks:
            continue
        if res.stop_reason != "abort":
            if len(res.output_logprobs) != len(toks) or len(res.output_versions) != len(toks):
                return None
            segs.append(_Segment(toks, True, [float(x) for x in res.output_logprobs], list(res.output_versions),
                                 float(rec.reward)))
        else:  # an interrupted generation stays in the transcript as context
            segs.append(_Segment(toks, trained=False))
        transcript.extend(toks)
        length += len(toks)
    return segs


def _lay_out(segs: List[_Segment], algorithm: str) -> Tuple[List[int], List[int], List[float], List[float], List[int],
                                                            List[int]]:
    ids: List[int] = []
    labels: List[int] = []
    logprobs: List[float] = []
    rewards: List[float] = []
    resp_idx: List[int] = []
    versions: List[int] = []
    n_resp = 0
    for seg in segs:
        n = len(seg.tokens)
        ids += seg.tokens
        if not seg.trained:
            labels += [IGNORE_INDEX] * n
            logprobs += [0.0] * n
            rewards += [0.0] * n
            resp_idx += [-1] * n
            continue
        if algorithm not in ("ppo", "grpo"):
            raise ValueError(f"Unsupported rl_algorithm: {algorithm}")
        labels += seg.tokens
        logprobs += seg.logprobs
        rewards += [0.0] * (n - 1) + [seg.reward if algorithm == "ppo" else 0.0]
        resp_idx += [n_resp] * n
        versions += seg.versions
        n_resp += 1
    return ids, labels, logprobs, rewards, resp_idx, versions


def build_episode_rl_sample(
    step_records: List[StepRecord],
    algorithm: str,
    history_window: int,
    gamma: float = 1.0,
    sample_advantage: Optional[float] = None,
) -> Optional[RLSample]:
    segs = _segments(step_records)
    if segs is None or not any(s.trained for s in segs):
        return None
    ids, labels, logprobs, rewards, resp_idx, versions = _lay_out(segs, algorithm)
    if len(ids) > history_window:
        return None
    if algorithm == "ppo":
        advantage = 0.0
        token_adv = token_level_returns(labels, rewards, gamma)
    else:
        if sample_advantage is None:
            raise ValueError("GRPO samples require a sample advantage.")
        advantage = float(sample_advantage)
        token_adv = [0.0 if lab == IGNORE_INDEX else advantage for lab in labels]
    return RLSample(
        algorithm=algorithm,  # type: ignore[arg-type]
        input_ids=ids,
        attention_mask=[1] * len(ids),
        labels=labels,
        old_logprobs=logprobs,
        advantage=advantage,
        token_advantages=token_adv,
        response_indices=resp_idx,
        output_versions=versions,
    )
