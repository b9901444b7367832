"""Rollout worker of the math (GSM8K) variant: one prompt, ``rollout_batch_size`` sampled answers,
R1-zero rewards and a group advantage, every answer one training sample.

Behaviour of the reference's ``RolloutWorkerActor`` (``vllm_fsdp.py:1546-1743``): an aborted or
empty generation gets reward 0; the group advantage is ``(r - mean) / (std + 1e-6)`` (population
std) and is zero for the whole group unless at least two answers earned a positive reward and the
rewards are not all equal. Samples use the shared ``RLSample`` contract (``algorithm="grpo"``,
prompt positions masked with -100, behaviour log-probs on the answer tokens).
"""

from __future__ import annotations

import asyncio
import math
import os
import random
from typing import Any, Callable, Dict, List, Optional, Tuple

from ..core.sample import IGNORE_INDEX, RLSample
from ..env.gsm8k import format_r1_zero_prompt, load_gsm8k, synthetic_arithmetic_problems
from ..rewards import r1_zero_reward_fn


def group_advantages(rewards: List[float]) -> List[float]:
    if not rewards:
        return []
    if sum(1 for r in rewards if r > 0.0) <= 1 or max(rewards) - min(rewards) < 1e-6:
        return [0.0] * len(rewards)
    mean = sum(rewards) / len(rewards)
    std = math.sqrt(sum((r - mean) ** 2 for r in rewards) / len(rewards))
    if std < 1e-6:
        return [0.0] * len(rewards)
    return [(r - mean) / (std + 1e-6) for r in rewards]


def load_math_examples(args) -> List[Tuple[str, str]]:
    path = getattr(args, "gsm8k_train_path", None)
    if path and path != "synthetic" and os.path.isfile(path):
        return load_gsm8k(path, getattr(args, "gsm8k_limit", None))
    n = getattr(args, "gsm8k_limit", None) or 4096
    return synthetic_arithmetic_problems(n, seed=args.seed)


class MathRolloutWorker:
    def __init__(self, args, infer, worker_id: int, replay_sink: Callable[[list], Any],
                 stats_sink: Callable[..., Any], tokenizer=None, examples: Optional[List[Tuple[str, str]]] = None):
        if tokenizer is None:
            raise ValueError("math rollouts need a tokenizer")
        self.args = args
        self.infer = infer
        self.worker_id = int(worker_id)
        self.replay_sink = replay_sink
        self.stats_sink = stats_sink
        self.tokenizer = tokenizer
        self.examples = examples if examples is not None else load_math_examples(args)
        self.rng = random.Random(args.seed * 100003 + self.worker_id)
        self.batch_id = 0
        self.episodes = 0
        self.stopped = False

    async def stop(self) -> None:
        self.stopped = True

    def reward_info(self, text: str, ground_truth: str, result) -> Dict[str, float]:
        if result.stop_reason == "abort" or not result.output_tokens:
            return {"format_reward": 0.0, "answer_reward": 0.0, "reward": 0.0}
        return r1_zero_reward_fn(text, ground_truth)

    def build_samples(self, input_ids: List[int], ground_truth: str, results) -> Tuple[List[RLSample], List[float]]:
        texts = [self.tokenizer.decode(r.output_tokens, skip_special_tokens=True) for r in results]
        rewards = [self.reward_info(t, ground_truth, r)["reward"] for t, r in zip(texts, results)]
        advs = group_advantages(rewards)
        samples = []
        n_prompt = len(input_ids)
        for r, adv in zip(results, advs):
            out = list(r.output_tokens)
            n = n_prompt + len(out)
            samples.append(RLSample(
                algorithm="grpo",
                input_ids=list(input_ids) + out,
                attention_mask=[1] * n,
                labels=[IGNORE_INDEX] * n_prompt + out,
                old_logprobs=[0.0] * n_prompt + [float(x) for x in r.output_logprobs],
                advantage=float(adv),
                token_advantages=[0.0] * n_prompt + [float(adv)] * len(out),
                response_indices=[-1] * n_prompt + [0] * len(out),
                output_versions=list(r.output_versions),
            ))
        return samples, rewards

    def next_prompt(self) -> Tuple[str, str, List[int]]:
        question, answer = self.rng.choice(self.examples)
        ids = list(self.tokenizer.encode(format_r1_zero_prompt(question)))
        return question, answer, ids

    async def run(self) -> Dict[str, int]:
        a = self.args
        while not self.stopped:
            _, answer, ids = self.next_prompt()
            self.batch_id += 1
            results = await asyncio.gather(*[self.infer.request_batch(ids, a.infer_max_tokens)
                                             for _ in range(a.rollout_batch_size)])
            if self.stopped and all(r.stop_reason == "abort" for r in results):
                break
            samples, rewards = self.build_samples(ids, answer, results)
            self.replay_sink(samples)
            self.episodes += len(samples)
            self.stats_sink("math", self.worker_id, rewards, [len(r.output_tokens) for r in results],
                            [r.stop_reason == "abort" for r in results])
        return {"worker_id": self.worker_id, "batches": self.batch_id, "episodes": self.episodes}
