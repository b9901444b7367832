"""Episode transcripts to ``RLSample`` (agent_textworld.py:2488-2588).

Every step record holds the prompt token ids the request was made with, the generation result and
the step reward. The builder walks the records and checks that each prompt extends the running
transcript; the new prompt tokens are context (label -100). Aborted outputs are kept as context too.
Trained response tokens carry their own ids as labels, the behaviour logprobs and versions, and a
response index that counts up per action. PPO puts the step reward on the response's last token and
turns token rewards into Monte-Carlo returns; GRPO broadcasts the group advantage to every response
token. Samples longer than the history window are rejected.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

from ..algo.advantages import token_level_returns
from ..core.sample import IGNORE_INDEX, RLSample
from .generation import InferenceResult


@dataclass
class StepRecord:
    training_result: InferenceResult
    prompt_ids: List[int]
    reward: float


def build_episode_rl_sample(
    step_records: List[StepRecord],
    algorithm: str,
    history_window: int,
    gamma: float = 1.0,
    sample_advantage: Optional[float] = None,
) -> Optional[RLSample]:
    input_ids: List[int] = []
    labels: List[int] = []
    old_logprobs: List[float] = []
    token_rewards: List[float] = []
    response_indices: List[int] = []
    output_versions: List[int] = []
    next_response = 0
    for record in step_records:
        prompt = record.prompt_ids
        if len(input_ids) > len(prompt) or prompt[: len(input_ids)] != input_ids:
            return None
        delta = prompt[len(input_ids):]
        if delta:
            n = len(delta)
            input_ids.extend(delta)
            labels.extend([IGNORE_INDEX] * n)
            old_logprobs.extend([0.0] * n)
            token_rewards.extend([0.0] * n)
            response_indices.extend([-1] * n)
        result = record.training_result
        if not result.output_tokens:
            continue
        out = list(result.output_tokens)
        n = len(out)
        if result.stop_reason == "abort":
            input_ids.extend(out)
            labels.extend([IGNORE_INDEX] * n)
            old_logprobs.extend([0.0] * n)
            token_rewards.extend([0.0] * n)
            response_indices.extend([-1] * n)
            continue
        if len(result.output_logprobs) != n or len(result.output_versions) != n:
            return None
        input_ids.extend(out)
        labels.extend(out)
        old_logprobs.extend(float(x) for x in result.output_logprobs)
        rewards = [0.0] * n
        if algorithm == "ppo":
            rewards[-1] = float(record.reward)
        elif algorithm != "grpo":
            raise ValueError(f"Unsupported rl_algorithm: {algorithm}")
        token_rewards.extend(rewards)
        response_indices.extend([next_response] * n)
        output_versions.extend(result.output_versions)
        next_response += 1
    if not labels or all(label == IGNORE_INDEX for label in labels):
        return None
    if len(input_ids) > history_window:
        return None
    if algorithm == "ppo":
        token_advantages = token_level_returns(labels, token_rewards, gamma)
        advantage = 0.0
    else:
        if sample_advantage is None:
            raise ValueError("GRPO samples require a sample advantage.")
        advantage = float(sample_advantage)
        token_advantages = [advantage if label != IGNORE_INDEX else 0.0 for label in labels]
    return RLSample(
        algorithm=algorithm,  # type: ignore[arg-type]
        input_ids=input_ids,
        attention_mask=[1] * len(input_ids),
        labels=labels,
        old_logprobs=old_logprobs,
        advantage=advantage,
        token_advantages=token_advantages,
        response_indices=response_indices,
        output_versions=output_versions,
    )
