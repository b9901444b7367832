"""Replay shards and rollout statistics.

``ReplayBuffer`` keeps a FIFO ring of ``RLSample`` with ``capacity`` entries; ``sample(n)`` draws
uniformly *without removal*, so samples are reused until evicted (agent_textworld.py:1689-1727).
One shard exists per trainer rank and rollout worker ``i`` feeds shard ``i % world``.

``RolloutStats`` keeps sliding windows of episode outcomes and an active-worker count based on a
last-seen timeout (agent_textworld.py:1634-1686).
"""

from __future__ import annotations

import random
import threading
import time
from collections import deque
from typing import Dict, List, Optional

from ..core.sample import RLSample


class ReplayBuffer:
    def __init__(self, capacity: int, seed: Optional[int] = None):
        if capacity < 1:
            raise ValueError("capacity must be >= 1")
        self.samples: deque = deque(maxlen=capacity)
        self.total_samples_added = 0
        self.total_samples_sampled = 0
        self.total_samples_evicted = 0
        self._rng = random.Random(seed)
        self._lock = threading.Lock()

    def add_samples(self, samples: List[RLSample]) -> Dict[str, int]:
        with self._lock:
            capacity = self.samples.maxlen or 0
            if capacity > 0:
                self.total_samples_evicted += max(0, len(self.samples) + len(samples) - capacity)
            self.samples.extend(samples)
            self.total_samples_added += len(samples)
            return self._stats_locked()

    def sample(self, batch_size: int) -> List[RLSample]:
        with self._lock:
            if batch_size < 1:
                return []
            count = min(batch_size, len(self.samples))
            if count == 0:
                return []
            out = self._rng.sample(list(self.samples), count)
            self.total_samples_sampled += len(out)
            return out

    def _stats_locked(self) -> Dict[str, int]:
        return {
            "size": len(self.samples),
            "capacity": self.samples.maxlen or 0,
            "total_samples_added": self.total_samples_added,
            "total_samples_sampled": self.total_samples_sampled,
            "total_samples_evicted": self.total_samples_evicted,
        }

    def get_stats(self) -> Dict[str, int]:
        with self._lock:
            return self._stats_locked()

    def __len__(self) -> int:
        return len(self.samples)


class RolloutStats:
    def __init__(self, window_size: int, active_timeout_seconds: float, clock=time.time):
        self.clock = clock
        self.active_timeout_seconds = active_timeout_seconds
        self.worker_last_active: Dict[int, float] = {}
        self.scores: deque = deque(maxlen=window_size)
        self.max_scores: deque = deque(maxlen=window_size)
        self.wins: deque = deque(maxlen=window_size)
        self.steps: deque = deque(maxlen=window_size)
        self.invalid_actions: deque = deque(maxlen=window_size)
        # math variant (per generated answer)
        self.rewards: deque = deque(maxlen=window_size)
        self.response_lengths: deque = deque(maxlen=window_size)
        self.abort_flags: deque = deque(maxlen=window_size)
        self.total_answers = 0
        self._lock = threading.Lock()

    def add_textworld_episode(
        self, worker_id: int, score: float, max_score: float, won: bool, steps: int, invalid_actions: int
    ) -> None:
        with self._lock:
            self.scores.append(float(score))
            self.max_scores.append(float(max_score))
            self.wins.append(bool(won))
            self.steps.append(int(steps))
            self.invalid_actions.append(int(invalid_actions))
            self.worker_last_active[int(worker_id)] = self.clock()

    add_episode = add_textworld_episode

    def add_rollout_batch(self, worker_id: int, rewards, response_lengths, abort_flags) -> None:
        """One group of answers of the math variant (``vllm_fsdp.py:1013-1030``)."""
        if not (len(rewards) == len(response_lengths) == len(abort_flags)):
            raise ValueError(f"Rollout metric batch lengths must match: rewards={len(rewards)} "
                             f"response_lengths={len(response_lengths)} abort_flags={len(abort_flags)}")
        with self._lock:
            self.rewards.extend(float(r) for r in rewards)
            self.response_lengths.extend(int(n) for n in response_lengths)
            self.abort_flags.extend(bool(f) for f in abort_flags)
            self.total_answers += len(rewards)
            self.worker_last_active[int(worker_id)] = self.clock()

    def add_record(self, *rec) -> None:
        """Dispatch a statistics record from a rollout worker: ``("math", ...)`` or a TextWorld episode."""
        if rec and rec[0] == "math":
            self.add_rollout_batch(*rec[1:])
        else:
            self.add_textworld_episode(*rec)

    def get_stats(self) -> Dict[str, float]:
        with self._lock:
            cutoff = self.clock() - self.active_timeout_seconds
            active = sum(1 for t in self.worker_last_active.values() if t >= cutoff)
            n = len(self.scores)
            total_steps = sum(self.steps)
            total_max = sum(self.max_scores)
            return {
                "active_workers": active,
                "tw_win_rate": (sum(1 for w in self.wins if w) / n) if n else 0.0,
                "tw_normalized_score": (sum(self.scores) / total_max) if total_max > 0 else 0.0,
                "tw_invalid_action_rate": (sum(self.invalid_actions) / total_steps) if total_steps else 0.0,
                "tw_env_steps_mean": (total_steps / n) if n else 0.0,
                "episodes": n,
                "global_reward_sum_mean": (sum(self.rewards) / len(self.rewards)) if self.rewards else 0.0,
                "response_length_mean": (sum(self.response_lengths) / len(self.response_lengths))
                if self.response_lengths else 0.0,
                "abort_rate": (sum(1 for f in self.abort_flags if f) / len(self.abort_flags)) if self.abort_flags else 0.0,
                "total_episodes": self.total_answers,
            }
