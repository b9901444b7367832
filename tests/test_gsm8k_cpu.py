"""Math (GSM8K) variant: the R1-zero grader, the group-advantage rule, sample construction of the
math rollout worker, the REINFORCE-style objective, and the whole loop on CPU ranks."""

import asyncio
import json
import types

import pytest
import torch

from accerl_agent_b200.algo.objectives import ObjectiveConfig, token_objective
from accerl_agent_b200.core.tokenizer import ByteTokenizer
from accerl_agent_b200.env.gsm8k import extract_gsm8k_final_answer, format_r1_zero_prompt, synthetic_arithmetic_problems
from accerl_agent_b200.rewards import extract_boxed, grade_answer, r1_zero_reward_fn
from accerl_agent_b200.rollout.math_worker import MathRolloutWorker, group_advantages


@pytest.mark.parametrize("response,gt,expected", [
    ("a </think> <answer>42</answer>", "42", (1.0, 1.0)),
    ("a </think> <answer> 1,234 </answer>", "1234", (1.0, 1.0)),
    ("a </think> <answer>$18.00</answer>", "18", (1.0, 1.0)),
    ("a </think> <answer>\\boxed{\\frac{3}{4}}</answer>", "0.75", (1.0, 1.0)),
    ("a </think> <answer>The answer is 7 dollars.</answer>", "7", (1.0, 1.0)),
    ("a </think> <answer>41</answer>", "42", (1.0, 0.0)),
    ("a </think> <answer>\\boxed{</answer>", "42", (1.0, 0.0)),
    ("a </think><answer>42</answer>", "42", (0.0, 0.0)),   # strict separator
    ("a </think> <answer>42", "42", (0.0, 0.0)),           # no closing tag
])
def test_r1_zero_reward(response, gt, expected):
    r = r1_zero_reward_fn(response, gt)
    assert (r["format_reward"], r["answer_reward"]) == expected
    assert r["reward"] == r["answer_reward"]


def test_grader_equivalences():
    assert grade_answer("x = 12", "12")
    assert not grade_answer("12", "13")
    assert grade_answer("2x+1", "1+2*x", fast=True)  # symbolic match is part of the fast path
    assert extract_boxed("so \\boxed{a{b}c} done") == "a{b}c"
    assert r1_zero_reward_fn("x </think> <answer>5</answer>", ["4", "5"])["reward"] == 1.0
    assert extract_gsm8k_final_answer("steps...\n#### 1,250") == "1250"


def test_group_advantage_rule():
    assert group_advantages([1.0, 0.0, 0.0, 0.0]) == [0.0] * 4        # a single right answer: no signal
    assert group_advantages([1.0, 1.0, 1.0]) == [0.0] * 3             # all equal
    adv = group_advantages([1.0, 1.0, 0.0, 0.0])
    assert adv[0] == pytest.approx(1.0, abs=1e-5) and adv[2] == pytest.approx(-1.0, abs=1e-5)


def test_reinforce_objective_has_no_ratio():
    lp = torch.tensor([-1.0, -2.0], requires_grad=True)
    obj, _, _ = token_objective(lp, torch.tensor([-5.0, 0.0]), torch.tensor([2.0, -1.0]), ObjectiveConfig(clip_mode="none"))
    obj.sum().backward()
    assert torch.allclose(obj, torch.tensor([-2.0, 2.0])) and torch.allclose(lp.grad, torch.tensor([2.0, -1.0]))


class _FakeInfer:
    def __init__(self, tok, texts):
        self.tok, self.texts, self.i = tok, texts, 0

    async def request_batch(self, ids, max_tokens):
        text = self.texts[self.i % len(self.texts)]
        self.i += 1
        out = self.tok.encode(text)
        return types.SimpleNamespace(output_tokens=out, output_logprobs=[-0.5] * len(out), output_versions=[3] * len(out),
                                     stop_reason="stop")


def test_math_worker_builds_grpo_samples():
    tok = ByteTokenizer(4096)
    args = types.SimpleNamespace(seed=1, infer_max_tokens=64, rollout_batch_size=4)
    texts = [" ok </think> <answer>7</answer>", " no </think> <answer>8</answer>"]
    sunk, stats = [], []
    w = MathRolloutWorker(args, _FakeInfer(tok, texts), 0, sunk.append, lambda *r: stats.append(r), tokenizer=tok,
                          examples=[("q?", "7")])
    _, gt, ids = w.next_prompt()
    assert tok.decode(ids).startswith("A conversation between User and Assistant.")
    async def four():
        return await asyncio.gather(*[w.infer.request_batch(ids, 64) for _ in range(4)])

    results = asyncio.run(four())
    samples, rewards = w.build_samples(ids, gt, results)
    assert rewards == [1.0, 0.0, 1.0, 0.0]
    for s, r in zip(samples, results):
        s.validate()
        n = len(ids)
        assert s.labels[:n] == [-100] * n and s.labels[n:] == list(r.output_tokens)
        assert s.old_logprobs[n:] == [-0.5] * len(r.output_tokens)
        assert s.algorithm == "grpo" and s.output_versions == [3] * len(r.output_tokens)
    assert samples[0].advantage > 0 > samples[1].advantage


def test_synthetic_problems_are_seeded_and_answerable():
    a = synthetic_arithmetic_problems(20, seed=3)
    assert a == synthetic_arithmetic_problems(20, seed=3)
    assert all(int(ans) >= 0 for _, ans in a)
    assert "<think>" in format_r1_zero_prompt(a[0][0])


def test_gsm8k_loop_end_to_end_cpu(tmp_path):
    from accerl_agent_b200.gsm8k_fsdp import main

    log = tmp_path / "run"
    main([
        "--model-path", "tiny-qwen2", "--device", "cpu", "--fsdp-world-size", "1", "--infer-size", "1",
        "--num-rollout-workers", "2", "--rollout-batch-size", "2", "--batch-size", "2", "--grad-accum-steps", "1",
        "--max-steps", "2", "--sync-every-optimizer-steps", "1", "--infer-max-tokens", "8", "--max-length", "1024",
        "--gsm8k-limit", "16", "--train-mode", "full", "--dtype", "float32", "--log-dir", str(log),
        "--learning-rate", "1e-4",
    ])
    recs = [json.loads(l) for l in open(log / "metrics.jsonl")]
    steps = [r for r in recs if "Train/Loss" in r]
    assert [r["step"] for r in steps] == [1, 2]
    for r in steps:
        assert "Rollout/GlobalRewardSumMean" in r and "Rollout/AbortRate" in r
    assert steps[0]["Infer/TokensPerSec"] > 0


@pytest.mark.parametrize("pred,gt,want", [
    ("50%", "50", True),             # the percent sign is dropped, not converted
    ("50%", "0.5", False),
    ("2/4", "1/2", False),           # an unreduced fraction does not match the reduced one
    (r"\frac{1}{2}", "0.5", True),
    ("5.0", "5", True),
    ("5.5", "5", False),             # an integer answer needs an integer
    ("0.333", "1/3", False),         # exact, no tolerance
    ("(1, 2)", "(1,2)", True),
    ("(1.0, 2)", "(1,2)", True),
    ("(1,2)", "[1,2]", False),       # a tuple's brackets must match
    ("(1,2)", "(2,1)", False),
    (r"\$1,250", "1250", True),
    (r"10\text{ cm}", "10", True),
    (r"\frac12", "1/2", True),
    (r"\frac{\sqrt{3}}{2}", r"\sqrt{3}/2", True),
    ("x^{100}+1", "1+x^{100}", False),  # braced exponents are not evaluated
])
def test_grader_fast_rules(pred, gt, want):
    """The fast path's decision rules (normalised match, then element-wise exact / symbolic match with
    the reference's fraction, integer, bracket and evaluation guards)."""
    assert grade_answer(pred, gt, fast=True) is want


def test_question_only_reward_and_repeatness():
    from accerl_agent_b200.rewards.math_grader import question_only_reward_fn, repeatness

    assert question_only_reward_fn("so it is \\boxed{7}.", 7)["reward"] == 1.0
    assert question_only_reward_fn("so it is \\boxed{8}.", 7) == {"format_reward": 1.0, "answer_reward": 0.0,
                                                                  "reward": 0.0}
    assert question_only_reward_fn("7", 7)["format_reward"] == 0.0
    assert repeatness("abc" * 40) and not repeatness("the quick brown fox jumps over the lazy dog")
    assert not repeatness("a")


@pytest.mark.parametrize("pred,gt,want", [
    (r"\frac{\sqrt{3}}{2}", r"\dfrac{\sqrt3}{2}", True),
    (r"\frac{1}{\frac{1}{2}}", "2", True),
    (r"2\frac{1}{2}", "5/2", True),
    (r"\sqrt[3]{8}", "2", True),
    (r"x^{2}+2x+1", "(x+1)^2", True),
    (r"\pi/2", r"\frac{\pi}{2}", True),
    (r"3 \pm \sqrt{2}", r"3-\sqrt2, 3+\sqrt2", True),
    (r"\{1, 2, 3\}", r"\{3,1,2\}", True),
    (r"(1, 2)", r"(2, 1)", False),
    (r"[0, 1)", r"[0,1)", True),
    (r"[0, 1)", r"[0,1]", False),
    (r"x = 5", "5", True),
    (r"2\sqrt{2}", r"\sqrt{8}", True),
    (r"\frac{3}{4}", "0.76", False),
])
def test_grader_latex_equivalence(pred, gt, want):
    from accerl_agent_b200.rewards.math_grader import grade_answer

    assert grade_answer(pred, gt, fast=False) is want
