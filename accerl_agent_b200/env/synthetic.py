"""Seeded synthetic text game for benchmarking the RL loop without TextWorld game files.

Each step emits an observation of uniform-random token ids whose length is drawn from
``U[obs_min, obs_max]`` (64..256 by default). Any generated action is accepted; the step reward is
Bernoulli(``reward_prob``) in {0, 1}. An episode ends after ``max_steps`` steps (50) or, after each
step, with probability ``end_prob`` (0.02). The environment works on token ids directly, so rollouts
need no tokenizer: the transcript is the initial observation followed by alternating action and
observation tokens, the same growing-prefix layout the TextWorld transcript has.
"""

from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Dict, List, Tuple


@dataclass(frozen=True)
class SyntheticGameConfig:
    vocab_size: int = 151936
    obs_min: int = 64
    obs_max: int = 256
    reward_prob: float = 0.1
    end_prob: float = 0.02
    max_steps: int = 50
    token_low: int = 0  # lowest token id emitted in observations


class SyntheticTextGame:
    def __init__(self, seed: int, cfg: SyntheticGameConfig = SyntheticGameConfig()):
        self.cfg = cfg
        self.seed = int(seed)
        self._rng = random.Random(self.seed)
        self.steps = 0
        self.score = 0.0
        self.done = False

    def _observation(self) -> List[int]:
        n = self._rng.randint(self.cfg.obs_min, self.cfg.obs_max)
        hi = self.cfg.vocab_size - 1
        lo = self.cfg.token_low
        return [self._rng.randint(lo, hi) for _ in range(n)]

    def _infos(self) -> Dict:
        return {
            "score": self.score,
            "max_score": float(self.cfg.max_steps),
            "won": False,
            "lost": False,
            "moves": self.steps,
            "admissible_commands": None,
        }

    def reset(self) -> Tuple[List[int], Dict]:
        self._rng = random.Random(self.seed)
        self.steps = 0
        self.score = 0.0
        self.done = False
        return self._observation(), self._infos()

    def step(self, action_tokens: List[int]) -> Tuple[List[int], float, bool, Dict]:
        if self.done:
            raise RuntimeError("step() called on a finished episode")
        self.steps += 1
        reward = 1.0 if self._rng.random() < self.cfg.reward_prob else 0.0
        self.score += reward
        self.done = self.steps >= self.cfg.max_steps or self._rng.random() < self.cfg.end_prob
        obs = [] if self.done else self._observation()
        return obs, reward, self.done, self._infos()

    def close(self) -> None:
        pass


def synthetic_episode_lengths(seed: int, cfg: SyntheticGameConfig, action_tokens: int, window: int) -> List[Tuple[int, int]]:
    """Token layout of one episode played with fixed-length actions: a list of
    ``(observation_len, action_len)`` steps, cut where the transcript reaches ``window`` tokens.
    The synthetic sample generator of the benchmark and tests uses it to mirror real rollouts."""
    env = SyntheticTextGame(seed, cfg)
    obs, _ = env.reset()
    total = len(obs)
    layout: List[Tuple[int, int]] = []
    pending_obs = len(obs)
    while True:
        if total >= window:
            break
        act = min(action_tokens, window - total)
        layout.append((pending_obs, act))
        total += act
        obs, _, done, _ = env.step([0] * act)
        if done:
            break
        pending_obs = len(obs)
        total += pending_obs
    return layout
