"""R1-zero style math reward: strict ``</think> <answer>...</answer>`` format, then answer equivalence.

Same contract as the reference's grader entry point (``scripts/drgrpo_grader.py:1008-1047``): a
response earns ``format_reward`` 1 when it contains ``"</think> <answer>"`` and ``"</answer>"``; the
text after the last ``<answer>`` (``\\boxed{...}`` content when present) is graded against the ground
truth (a string, a number or a list of accepted answers); ``reward = answer_reward`` and a
well-formatted wrong answer gets no reward (no reward for format alone).

Equivalence is decided here, in order:
  1. normalised strings are equal (LaTeX wrappers, units words, ``$``, thousands separators,
     trailing periods and spacing removed; ``\\frac{a}{b}`` -> ``a/b``);
  2. both sides parse as numbers (integers, decimals, fractions, percentages, scientific notation)
     and agree to a relative tolerance of 1e-4 (percent answers also match their fraction);
  3. with ``fast=False``: both sides parse as sympy expressions whose difference simplifies to 0.
``math_verify`` (when installed) is consulted last in slow mode, like the reference's fallback chain.
"""

from __future__ import annotations

import re
from typing import Dict, Iterable, Optional, Union

_UNIT_WORDS = (
    "dollars", "dollar", "cents", "cent", "percent", "units", "unit", "meters", "meter", "miles", "mile",
    "hours", "hour", "minutes", "minute", "seconds", "second", "days", "day", "weeks", "week", "years", "year",
    "feet", "foot", "inches", "inch", "pounds", "pound", "kg", "km", "cm", "mm", "degrees", "degree",
)


def extract_boxed(text: str) -> Optional[str]:
    """Content of the last ``\\boxed{...}`` (or ``\\fbox{...}``) with balanced braces, else None."""
    start = max(text.rfind("\\boxed"), text.rfind("\\fbox"))
    if start < 0:
        return None
    i = text.find("{", start)
    if i < 0:
        # \boxed 5  (no braces): the token after the command
        rest = text[start:].split(None, 1)
        return rest[1].strip() if len(rest) == 2 else None
    depth = 0
    for j in range(i, len(text)):
        if text[j] == "{":
            depth += 1
        elif text[j] == "}":
            depth -= 1
            if depth == 0:
                return text[i + 1 : j]
    return None


def _strip_wrappers(s: str) -> str:
    for cmd in ("\\text", "\\textbf", "\\mathrm", "\\mbox", "\\mathbf"):
        while cmd + "{" in s:
            k = s.find(cmd + "{")
            depth, j = 0, k + len(cmd)
            end = -1
            for j in range(k + len(cmd), len(s)):
                if s[j] == "{":
                    depth += 1
                elif s[j] == "}":
                    depth -= 1
                    if depth == 0:
                        end = j
                        break
            if end < 0:
                break
            s = s[:k] + s[k + len(cmd) + 1 : end] + s[end + 1 :]
    return s


def _frac_to_slash(s: str) -> str:
    pat = re.compile(r"\\[dt]?frac\s*\{([^{}]*)\}\s*\{([^{}]*)\}")
    while True:
        t = pat.sub(lambda m: f"({m.group(1)})/({m.group(2)})", s)
        if t == s:
            break
        s = t
    # \frac12 shorthand
    s = re.sub(r"\\[dt]?frac(\d)(\d)", r"(\1)/(\2)", s)
    return s


def normalize_answer(ans: str) -> str:
    s = str(ans).strip()
    s = s.replace("\n", " ")
    s = _strip_wrappers(s)
    for tok in ("\\left", "\\right", "\\!", "\\,", "\\;", "\\:", "\\ ", "$", "\\displaystyle"):
        s = s.replace(tok, "")
    s = s.replace("^\\circ", "").replace("^{\\circ}", "").replace("\\circ", "")
    s = s.replace("\\%", "%").replace("\\$", "")
    s = _frac_to_slash(s)
    s = s.replace("\\cdot", "*").replace("\\times", "*").replace("\\div", "/")
    s = s.replace("{", "(").replace("}", ")")
    low = s.lower().strip()
    # leading "x =" / "answer:" style prefixes
    low = re.sub(r"^(the\s+)?(final\s+)?answer\s*(is|:)\s*", "", low)
    low = re.sub(r"^[a-z]\s*=\s*", "", low)
    words = r"\b(" + "|".join(_UNIT_WORDS) + r")\b"
    low = re.sub(words, "", low)
    low = re.sub(r"(?<=\d),(?=\d{3}\b)", "", low)  # thousands separators
    low = low.replace(" ", "")
    low = low.rstrip(".")
    if low.startswith("(") and low.endswith(")") and low.count("(") == 1:
        low = low[1:-1]
    return low


_NUM = re.compile(r"^[+-]?(\d+(\.\d*)?|\.\d+)(e[+-]?\d+)?$")


def _to_number(s: str) -> Optional[float]:
    s = s.strip()
    pct = s.endswith("%")
    if pct:
        s = s[:-1]
    s = s.replace("(", "").replace(")", "")
    val: Optional[float] = None
    if _NUM.match(s):
        val = float(s)
    elif s.count("/") == 1:
        a, b = s.split("/")
        if _NUM.match(a) and _NUM.match(b) and float(b) != 0.0:
            val = float(a) / float(b)
    if val is None:
        return None
    return val / 100.0 if pct else val


def _close(a: float, b: float) -> bool:
    return abs(a - b) <= 1e-4 * max(1.0, abs(a), abs(b))


def _numbers_equal(pred: str, gt: str) -> bool:
    a, b = _to_number(pred), _to_number(gt)
    if a is None or b is None:
        return False
    if _close(a, b):
        return True
    # "25%" vs "25" and "0.25" vs "25%" are both accepted
    if pred.endswith("%") and _close(a * 100.0, b):
        return True
    if gt.endswith("%") and _close(a, b * 100.0):
        return True
    return False


def _sympy_equal(pred: str, gt: str) -> bool:
    try:
        import sympy
        from sympy.parsing.sympy_parser import (implicit_multiplication_application, parse_expr,
                                                standard_transformations)
    except Exception:
        return False
    tr = standard_transformations + (implicit_multiplication_application,)
    try:
        a = parse_expr(pred.replace("^", "**"), transformations=tr, evaluate=True)
        b = parse_expr(gt.replace("^", "**"), transformations=tr, evaluate=True)
        return bool(sympy.simplify(a - b) == 0)
    except Exception:
        return False


def _math_verify_equal(pred: str, gt: str) -> bool:
    try:
        from math_verify import parse, verify
    except Exception:
        return False
    try:
        return bool(verify(parse(gt), parse(pred)))
    except Exception:
        return False


def grade_answer(pred: str, gt: str, fast: bool = True) -> bool:
    if pred is None:
        return False
    p, g = normalize_answer(pred), normalize_answer(gt)
    if not p:
        return False
    if p == g or _numbers_equal(p, g):
        return True
    if fast:
        return False
    return _sympy_equal(p, g) or _math_verify_equal(pred, gt)


def r1_zero_reward_fn(response: str, ground_truth: Union[str, int, float, Iterable], fast: bool = True) -> Dict[str, float]:
    zero = {"format_reward": 0.0, "answer_reward": 0.0, "reward": 0.0}
    if "</think> <answer>" not in response or "</answer>" not in response:
        return zero
    answer = response.split("<answer>")[-1].replace("</answer>", "")
    if "\\boxed" in answer or "\\fbox" in answer:
        answer = extract_boxed(answer)
        if answer is None:
            return {"format_reward": 1.0, "answer_reward": 0.0, "reward": 0.0}
    if isinstance(ground_truth, (int, float)):
        gts = [str(ground_truth)]
    elif isinstance(ground_truth, str):
        gts = [ground_truth]
    else:
        gts = [str(g) for g in ground_truth]
    ok = any(grade_answer(answer, g, fast) for g in gts)
    return {"format_reward": 1.0, "answer_reward": 1.0 if ok else 0.0, "reward": 1.0 if ok else 0.0}
