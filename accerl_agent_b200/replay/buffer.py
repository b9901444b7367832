"""Replay shards and rollout statistics.

``ReplayBuffer`` is one trainer rank's replay shard: a fixed ring of ``capacity`` sample slots with a
write cursor. New samples overwrite the oldest ones once the ring is full, and ``sample(n)`` returns
``min(n, size)`` distinct samples chosen uniformly while leaving them in place, so a sample keeps
being reused until it is overwritten (the replay semantics of accerl_agent/agent_textworld.py:1689-1727;
its ``get_stats`` keys are kept so dashboards and logs read the same). Rollout worker ``i`` feeds
shard ``i % world``.

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
        self._ring: List[Optional[RLSample]] = [None] * capacity
        self._cursor = 0  # slot the next sample is written to
        self._filled = 0  # occupied slots
        self._counts = {"added": 0, "drawn": 0, "overwritten": 0}
        self._rng = random.Random(seed)
        self._mu = threading.Lock()

    @property
    def capacity(self) -> int:
        return len(self._ring)

    def add_samples(self, samples: List[RLSample]) -> Dict[str, int]:
        """Append ``samples`` in order; returns the stats after the write."""
        cap = len(self._ring)
        with self._mu:
            n = len(samples)
            self._counts["added"] += n
            self._counts["overwritten"] += max(0, self._filled + n - cap)
            # only the newest `cap` of this call can survive it
            for s in samples[max(0, n - cap):]:
                self._ring[self._cursor] = s
                self._cursor = (self._cursor + 1) % cap
            self._filled = min(cap, self._filled + n)
            return self._stats()

    def sample(self, batch_size: int) -> List[RLSample]:
        """Up to ``batch_size`` distinct stored samples, uniformly at random, without removing them."""
        with self._mu:
            k = min(max(batch_size, 0), self._filled)
            if k == 0:
                return []
            cap = len(self._ring)
            oldest = (self._cursor - self._filled) % cap
            picks = self._rng.sample(range(self._filled), k)
            self._counts["drawn"] += k
            return [self._ring[(oldest + i) % cap] for i in picks]

    def snapshot(self) -> List[RLSample]:
        """The stored samples, oldest first."""
        with self._mu:
            cap = len(self._ring)
            oldest = (self._cursor - self._filled) % cap
            return [self._ring[(oldest + i) % cap] for i in range(self._filled)]

    def _stats(self) -> Dict[str, int]:
        return {
            "size": self._filled,
            "capacity": len(self._ring),
            "total_samples_added": self._counts["added"],
            "total_samples_sampled": self._counts["drawn"],
            "total_samples_evicted": self._counts["overwritten"],
        }

    def get_stats(self) -> Dict[str, int]:
        with self._mu:
            return self._stats()

    def __len__(self) -> int:
        return self._filled


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
