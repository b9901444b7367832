"""GSM8K data and the R1-zero prompt of the math variant of the RL loop.

``load_gsm8k`` reads the GSM8K ``jsonl`` layout (``question`` and ``answer`` with the final answer
after ``####``; ``vllm_fsdp.py:123-148`` of the reference reads the same layout). Offline runs without
the dataset use ``synthetic_arithmetic_problems``: seeded word problems with integer answers in the
same (question, answer) form.
"""

from __future__ import annotations

import json
import random
from typing import List, Optional, Tuple

# The R1-zero prompt format (public; the reward parser depends on the "<think>"/"<answer>" tags).
R1_ZERO_PROMPT = (
    "A conversation between User and Assistant. The User asks a question, and the Assistant solves it. "
    "The Assistant first thinks about the reasoning process in the mind and then provides the User with the "
    "answer. The reasoning process is enclosed within <think> </think> and answer is enclosed within "
    "<answer> </answer> tags, respectively, i.e., <think> reasoning process here </think> <answer> answer here "
    "</answer>.\nUser: {question}\nAssistant: <think>"
)


def format_r1_zero_prompt(question: str) -> str:
    return R1_ZERO_PROMPT.replace("{question}", question)


def extract_gsm8k_final_answer(answer: str) -> str:
    if "####" in answer:
        answer = answer.rsplit("####", 1)[-1]
    return answer.strip().replace(",", "")


def load_gsm8k(path: str, limit: Optional[int] = None) -> List[Tuple[str, str]]:
    out: List[Tuple[str, str]] = []
    with open(path, "r", encoding="utf-8") as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            item = json.loads(line)
            out.append((item["question"], extract_gsm8k_final_answer(item["answer"])))
            if limit is not None and len(out) >= limit:
                break
    if not out:
        raise ValueError(f"No GSM8K examples loaded from {path!r}.")
    return out


_NAMES = ("Ava", "Ben", "Chen", "Dana", "Eli", "Fatima", "Gus", "Hana", "Ivan", "Jia")
_ITEMS = ("apples", "marbles", "stickers", "books", "coins", "pencils", "cards", "shells")


def synthetic_arithmetic_problems(n: int, seed: int = 0) -> List[Tuple[str, str]]:
    """``n`` seeded two-step word problems (buy/give/split) with integer answers."""
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        name, item = rng.choice(_NAMES), rng.choice(_ITEMS)
        a, b, c = rng.randint(2, 60), rng.randint(2, 12), rng.randint(2, 9)
        kind = rng.randrange(3)
        if kind == 0:
            q = (f"{name} has {a} {item}. {name} buys {b} packs with {c} {item} in each pack. "
                 f"How many {item} does {name} have now?")
            ans = a + b * c
        elif kind == 1:
            total = b * c * rng.randint(1, 5)
            q = (f"{name} has {total + a} {item} and gives away {a}. The rest are shared equally among {b} "
                 f"friends. How many {item} does each friend get?")
            ans = total // b
        else:
            q = (f"A box holds {c} {item}. {name} fills {b} boxes and has {a} {item} left over. "
                 f"How many {item} did {name} start with?")
            ans = b * c + a
        out.append((q, str(ans)))
    return out
