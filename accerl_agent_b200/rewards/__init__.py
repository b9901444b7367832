"""Reward functions for the math (GSM8K) variant of the RL loop."""

from .math_grader import (extract_boxed, grade_answer, normalize_answer, question_only_reward_fn, r1_zero_reward_fn,
                          repeatness)

__all__ = ["extract_boxed", "grade_answer", "normalize_answer", "question_only_reward_fn", "r1_zero_reward_fn",
           "repeatness"]
