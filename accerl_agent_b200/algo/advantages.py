"""Advantage estimators.

* ``token_level_returns`` – Monte-Carlo reward-to-go over trained tokens only (prompt tokens are
  skipped, not discounted), agent_textworld.py:2590-2607.
* ``grpo_group_advantages`` – ``(R_i - mean)/(std + eps)`` with the population std; all zeros when the
  group has at most one member or ``std <= eps`` (agent_textworld.py:2609-2623).
* ``compute_gae`` – generalised advantage estimation ``delta = r + gamma*V' - V``,
  ``A = delta + gamma*lambda*A'`` (accerl_agent/scripts/compute_GAE.py:14-54); not wired into training,
  as in the reference, since no critic exists.
"""

from __future__ import annotations

import math
from typing import List, Sequence, Tuple

import torch

from ..core.sample import IGNORE_INDEX


def token_level_returns(labels: Sequence[int], token_rewards: Sequence[float], gamma: float) -> List[float]:
    if len(labels) != len(token_rewards):
        raise ValueError("labels and token_rewards must have the same length.")
    out = [0.0] * len(labels)
    running = 0.0
    for i in range(len(labels) - 1, -1, -1):
        if labels[i] == IGNORE_INDEX:
            continue
        running = float(token_rewards[i]) + gamma * running
        out[i] = running
    return out


def grpo_group_advantages(rewards: Sequence[float], eps: float) -> Tuple[float, float, List[float]]:
    if not rewards:
        return 0.0, 0.0, []
    n = len(rewards)
    mean = sum(rewards) / n
    std = math.sqrt(sum((r - mean) ** 2 for r in rewards) / n)
    if n <= 1 or std <= eps:
        return mean, std, [0.0] * n
    return mean, std, [(r - mean) / (std + eps) for r in rewards]


def compute_gae(
    rewards: torch.Tensor,
    values: torch.Tensor,
    gamma: float = 0.99,
    gae_lambda: float = 0.95,
    bootstrap: float | torch.Tensor = 0.0,
) -> Tuple[torch.Tensor, torch.Tensor]:
    if rewards.ndim != 1 or values.ndim != 1 or rewards.shape != values.shape:
        raise ValueError(f"rewards and values must be 1-D with equal shapes, got {rewards.shape} and {values.shape}")
    boot = torch.as_tensor(bootstrap, dtype=values.dtype, device=values.device).reshape(1)
    next_values = torch.cat((values[1:], boot))
    deltas = rewards + gamma * next_values - values
    gae = torch.empty_like(deltas)
    running = torch.zeros((), dtype=deltas.dtype, device=deltas.device)
    for i in range(rewards.numel() - 1, -1, -1):
        running = deltas[i] + gamma * gae_lambda * running
        gae[i] = running
    return gae, deltas
