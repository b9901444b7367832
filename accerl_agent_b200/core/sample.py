"""The per-episode training sample contract shared by rollout, replay and trainer.

Field semantics follow the reference contract (accerl_agent/agent_textworld.py:60-70, README.md:307-322):

* ``input_ids``      full token transcript (prompt deltas, responses, aborted outputs)
* ``labels``         token id where the position is trained, ``-100`` otherwise
* ``old_logprobs``   behaviour-policy log-probability of each trained token (0.0 elsewhere)
* ``advantage``      scalar GRPO advantage of the whole trajectory
* ``token_advantages`` per-token PPO advantage (Monte-Carlo reward-to-go); GRPO broadcasts ``advantage``
* ``response_indices`` index of the action response each trained token belongs to, -1 elsewhere
* ``output_versions`` policy version that produced every trained token, in order
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Literal

import torch

Algorithm = Literal["ppo", "grpo"]

IGNORE_INDEX = -100

VARLEN_TOKEN_STAT_NAMES = (
    "policy_token_sum",
    "old_new_kl_k3_sum",
    "ppo_clip_count",
)


@dataclass
class RLSample:
    algorithm: Algorithm
    input_ids: List[int]
    attention_mask: List[int]
    labels: List[int]
    old_logprobs: List[float]
    advantage: float
    token_advantages: List[float]
    response_indices: List[int]
    output_versions: List[int]

    def __len__(self) -> int:
        return len(self.input_ids)

    @property
    def num_targets(self) -> int:
        return sum(1 for label in self.labels if label != IGNORE_INDEX)

    def validate(self) -> None:
        """Raise ``ValueError`` when per-token fields disagree in length."""
        n = len(self.input_ids)
        for name in ("attention_mask", "labels", "old_logprobs", "token_advantages", "response_indices"):
            if len(getattr(self, name)) != n:
                raise ValueError(f"RLSample.{name} has length {len(getattr(self, name))}, expected {n}")


@dataclass
class PreparedVarlenPack:
    """One CPU-resident pack of a varlen optimizer window (agent_textworld.py:73-81)."""

    batch: Dict[str, torch.Tensor]
    valid_token_count: int
    max_seqlen: int
    version_lag_sum: float
    sample_count: int
    total_tokens: int = 0
    pack_cpu_ms: float = 0.0
    extra: Dict[str, float] = field(default_factory=dict)
