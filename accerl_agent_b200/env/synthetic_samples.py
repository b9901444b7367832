"""RLSamples with the token layout of synthetic text-game episodes, produced without a model.

Each episode follows ``SyntheticTextGame`` (observations of U[obs_min, obs_max] random tokens, actions of
``action_tokens`` sampled tokens, Bernoulli rewards, end after ``max_steps`` or with ``end_prob``),
truncated at the history window. Groups of ``group_size`` episodes of one game get GRPO advantages
from their returns. Old log-probabilities are drawn around ``-log(vocab)`` (a random-init policy).
The benchmark and tests use these to feed the trainer with exactly the shapes rollouts produce.
"""

from __future__ import annotations

import math
import random
from typing import List

from ..algo.advantages import grpo_group_advantages
from ..core.sample import IGNORE_INDEX, RLSample
from .synthetic import SyntheticGameConfig, SyntheticTextGame


def synthetic_episode_sample(rng: random.Random, game_seed: int, cfg: SyntheticGameConfig, action_tokens: int,
                             window: int, algorithm: str = "grpo", version: int = 0, gamma: float = 1.0):
    env = SyntheticTextGame(game_seed * 1000003 + rng.randrange(1 << 30), cfg)
    obs, _ = env.reset()
    ids: List[int] = list(obs)
    labels: List[int] = [IGNORE_INDEX] * len(obs)
    rewards_tok: List[float] = [0.0] * len(obs)
    resp: List[int] = [-1] * len(obs)
    old: List[float] = [0.0] * len(obs)
    versions: List[int] = []
    total_reward = 0.0
    r_idx = 0
    base_lp = -math.log(cfg.vocab_size)
    while len(ids) < window:
        n = min(action_tokens, window - len(ids))
        act = [rng.randrange(cfg.vocab_size) for _ in range(n)]
        ids.extend(act)
        labels.extend(act)
        old.extend(base_lp + rng.gauss(0.0, 0.5) for _ in range(n))
        resp.extend([r_idx] * n)
        versions.extend([version] * n)
        obs, reward, done, _ = env.step(act)
        tr = [0.0] * n
        tr[-1] = reward
        rewards_tok.extend(tr)
        total_reward += reward
        r_idx += 1
        if done:
            break
        obs = obs[: max(0, window - len(ids))]
        ids.extend(obs)
        labels.extend([IGNORE_INDEX] * len(obs))
        old.extend([0.0] * len(obs))
        rewards_tok.extend([0.0] * len(obs))
        resp.extend([-1] * len(obs))
    return ids, labels, old, rewards_tok, resp, versions, total_reward


def synthetic_rl_samples(num_groups: int, group_size: int = 8, seed: int = 0, window: int = 8192,
                         action_tokens: int = 16, cfg: SyntheticGameConfig = SyntheticGameConfig(),
                         algorithm: str = "grpo", gamma: float = 1.0, version: int = 0) -> List[RLSample]:
    from ..algo.advantages import token_level_returns

    rng = random.Random(seed)
    out: List[RLSample] = []
    for g in range(num_groups):
        eps = [synthetic_episode_sample(rng, seed * 7919 + g, cfg, action_tokens, window, algorithm, version, gamma)
               for _ in range(group_size)]
        _, _, advs = grpo_group_advantages([e[6] for e in eps], 1e-8)
        for (ids, labels, old, rtok, resp, versions, _), a in zip(eps, advs):
            if algorithm == "ppo":
                tok_adv = token_level_returns(labels, rtok, gamma)
                adv = 0.0
            else:
                adv = a
                tok_adv = [a if lab != IGNORE_INDEX else 0.0 for lab in labels]
            out.append(RLSample(algorithm=algorithm, input_ids=ids, attention_mask=[1] * len(ids), labels=labels,
                                old_logprobs=old, advantage=float(adv), token_advantages=tok_adv,
                                response_indices=resp, output_versions=versions))
    return out


def benchmark_pool(rank: int, samples: int, window: int) -> List[RLSample]:
    """The trainer benchmark's per-rank replay pool: seeded synthetic text-game episodes in GRPO
    groups of 8 with 16-token actions and a ``window``-token history (seed 1000 + rank)."""
    groups = (samples + 7) // 8
    return synthetic_rl_samples(groups, group_size=8, seed=1000 + rank, window=window, action_tokens=16)
