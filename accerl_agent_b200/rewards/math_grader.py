"""R1-zero style math reward: strict ``</think> <answer>...</answer>`` format, then answer equivalence.

Same contract as the reference's grader entry point (``scripts/drgrpo_grader.py:1008-1047``): a
response earns ``format_reward`` 1 when it contains ``"</think> <answer>"`` and ``"</answer>"``; the
text after the last ``<answer>`` (``\\boxed{...}`` content when present) is graded against the ground
truth (a string, a number or a list of accepted answers); ``reward = answer_reward`` and a
well-formatted wrong answer gets no reward (no reward for format alone). ``question_only_reward_fn``
grades the last ``\\boxed{}`` of a free-form response (``drgrpo_grader.py:1050-1080``).

Equivalence follows the reference's decision rules (``grade``: normalised match or symbolic match,
``drgrpo_grader.py:936-1005``), implemented here:
  1. normalised strings are equal (LaTeX wrappers, unit words, ``$``, ``%``, thousands separators,
     trailing periods, spacing and a short ``x =`` prefix removed; ``\\frac{a}{b}`` -> ``a/b``;
     ``million`` / ``billion`` / ``trillion`` as powers of ten);
  2. otherwise, element by element (a bracketed tuple or interval splits at its commas, and both
     sides must use the same brackets): two fractions of integers must be written identically (an
     unreduced fraction is not accepted for a reduced one), an integer answer needs an integer, and
     everything else must be exactly equal as a number or, for expressions that are safe to evaluate
     (at most two unknown letters, no braced or multi-digit exponents), under sympy simplification;
  3. with ``fast=False`` also: the LaTeX is rewritten into sympy syntax (nested fractions, roots,
     powers, constants, mixed numbers) and compared symbolically, then numerically; ``\\pm`` answers
     and ``\\{...\\}`` sets compare as unordered lists, tuples in order, intervals with their
     brackets; ``math_verify`` (when installed) is consulted last, like the reference's fallback.
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
    """``\\frac{a}{b}`` (and ``\\dfrac`` / ``\\tfrac``, nested, or the ``\\frac12`` shorthand) ->
    ``(a)/(b)``, arguments matched by balanced braces."""
    out, i = [], 0
    while i < len(s):
        m = re.match(r"\\[dt]?frac", s[i:])
        if not m:
            out.append(s[i])
            i += 1
            continue
        num, j = _arg(s, i + len(m.group(0)))
        den, j = _arg(s, j)
        out.append(f"({_frac_to_slash(num)})/({_frac_to_slash(den)})")
        i = j
    return "".join(out)


def normalize_answer(ans: str) -> str:
    s = str(ans).strip()
    s = s.replace("\n", " ")
    s = _strip_wrappers(s)
    s = s.replace("\\%", "%").replace("\\$", "").replace("%", "")
    for tok in ("\\left", "\\right", "\\!", "\\,", "\\;", "\\:", "\\ ", "$", "\\displaystyle"):
        s = s.replace(tok, "")
    s = s.replace("^\\circ", "").replace("^{\\circ}", "").replace("\\circ", "")
    s = re.sub(r"\s*\b(million|billion|trillion)\b", lambda m: {"million": "*10^6", "billion": "*10^9",
                                                                 "trillion": "*10^12"}[m.group(1)], s)
    s = re.sub(r"\s+(or|and)\s+", ",", s)
    s = _frac_to_slash(s)
    for word in ("sqrt", "pi", "infty"):
        s = s.replace("\\" + word, word)
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
    if low.startswith("(") and low.endswith(")") and low.count("(") == 1 and "," not in low:
        low = low[1:-1]
    low = re.sub(r"(?<![a-z])\((-?\d+(?:\.\d+)?)\)", r"\1", low)  # "(1)/(2)" -> "1/2", not "sqrt(3)"
    if re.fullmatch(r"-?\d+\.0*", low):  # "5.0" -> "5"
        low = low.split(".")[0]
    return low


_NUM = re.compile(r"^[+-]?(\d+(\.\d*)?|\.\d+)(e[+-]?\d+)?$")


_INT_FRAC = re.compile(r"^-?\d+/0*[1-9]\d*$")


def _exact_number(s: str):
    """The exact rational value of a decimal or a fraction of decimals, else None."""
    from fractions import Fraction

    s = s.replace("(", "").replace(")", "")
    try:
        if _NUM.match(s):
            return Fraction(s)
        if s.count("/") == 1:
            a, b = s.split("/")
            if _NUM.match(a) and _NUM.match(b) and float(b) != 0.0:
                return Fraction(a) / Fraction(b)
    except (ValueError, ZeroDivisionError):
        return None
    return None


def _is_integer_text(s: str) -> bool:
    v = _exact_number(s)
    return v is not None and v.denominator == 1


def _tuple_elements(s: str):
    """Elements of a bracketed tuple or interval written without nested brackets, else [s]."""
    if len(s) > 2 and s[0] in "([" and s[-1] in ")]" and not any(c in s[1:-1] for c in "()[]"):
        return [e.strip() for e in s[1:-1].split(",")]
    return [s]


def _safe_to_evaluate(expr: str) -> bool:
    """Expressions sympy may simplify without hanging: at most two unknown letters, no braced or
    parenthesised exponents, no exponent of two or more digits and no power towers."""
    body = expr
    for word in ("sqrt", "frac", "pi"):
        body = body.replace(word, "")
    if len({c for c in body if c.isalpha()}) > 2 or len(expr) > 200:
        return False
    if "^{" in expr or "^(" in expr or "**(" in expr:
        return False
    return re.search(r"\^\d+\^", expr) is None and re.search(r"\^\d\d+", expr) is None


def _symbolic_zero(a: str, b: str) -> bool:
    try:
        import sympy
        from sympy.parsing.sympy_parser import (convert_xor, implicit_multiplication_application, parse_expr,
                                                standard_transformations)
    except Exception:
        return False
    tr = standard_transformations + (implicit_multiplication_application, convert_xor)
    try:
        return sympy.simplify(parse_expr(f"({a})-({b})", transformations=tr)) == 0
    except Exception:
        return False


def _element_equal(pred: str, gt: str) -> bool:
    if _INT_FRAC.match(pred) and _INT_FRAC.match(gt):
        return pred == gt  # an unreduced fraction does not match the reduced one
    if _is_integer_text(pred) != _is_integer_text(gt):
        return False  # an integer answer needs an integer
    a, b = _exact_number(pred), _exact_number(gt)
    if a is not None and b is not None:
        return a == b
    expr = f"({gt})-({pred})"
    return _safe_to_evaluate(expr) and _symbolic_zero(gt, pred)


def _normalised_equal(pred: str, gt: str) -> bool:
    """Rule 2 of the module docstring on normalised strings."""
    ge, pe = _tuple_elements(gt), _tuple_elements(pred)
    if len(ge) > 1 and (gt[0] != pred[0] or gt[-1] != pred[-1]):
        return False
    if len(ge) != len(pe):
        return False
    return all(_element_equal(p, g) for p, g in zip(pe, ge))


def _braced(s: str, i: int):
    """(content, index after the closing brace) of the brace group opening at s[i] == '{'."""
    depth = 0
    for j in range(i, len(s)):
        if s[j] == "{":
            depth += 1
        elif s[j] == "}":
            depth -= 1
            if depth == 0:
                return s[i + 1 : j], j + 1
    return s[i + 1 :], len(s)


def _arg(s: str, i: int):
    """One LaTeX macro argument starting at s[i] (after spaces): a brace group or a single token."""
    while i < len(s) and s[i] == " ":
        i += 1
    if i >= len(s):
        return "", i
    if s[i] == "{":
        return _braced(s, i)
    if s[i] == "\\":
        m = re.match(r"\\[a-zA-Z]+", s[i:])
        if m:
            return m.group(0), i + len(m.group(0))
    return s[i], i + 1


_LATEX_WORDS = {
    "\\pi": "pi", "\\infty": "oo", "\\cdot": "*", "\\times": "*", "\\div": "/", "\\ln": "log",
    "\\log": "log", "\\sin": "sin", "\\cos": "cos", "\\tan": "tan", "\\exp": "exp", "\\e": "E",
}


def latex_to_sympy_text(s: str) -> str:
    """Rewrite a LaTeX math answer into text that sympy's parser reads: nested ``\\frac`` /
    ``\\dfrac`` / ``\\tfrac``, ``\\sqrt[n]{x}``, braces after ``^``, ``\\pi``, ``\\infty``, products,
    ``\\left`` / ``\\right`` sizing, and mixed numbers (``2\\frac{1}{2}`` = 5/2)."""
    s = _strip_wrappers(str(s))
    for tok in ("\\left", "\\right", "\\!", "\\,", "\\;", "\\:", "\\displaystyle", "$"):
        s = s.replace(tok, "")
    s = s.replace("\\{", "{").replace("\\}", "}")
    out = []
    i = 0
    while i < len(s):
        if s.startswith("\\sqrt", i):
            i += 5
            index = None
            if i < len(s) and s[i] == "[":
                k = s.index("]", i)
                index, i = s[i + 1 : k], k + 1
            body, i = _arg(s, i)
            body = latex_to_sympy_text(body)
            out.append(f"(({body})**(1/({latex_to_sympy_text(index)})))" if index else f"sqrt({body})")
            continue
        m = re.match(r"\\[dt]?frac", s[i:])
        if m:
            num, j = _arg(s, i + len(m.group(0)))
            den, j = _arg(s, j)
            num_t, den_t = latex_to_sympy_text(num), latex_to_sympy_text(den)
            # mixed number: an integer written right before a fraction of integers
            prev = "".join(out).rstrip()
            lead = re.search(r"(?:^|[^\w.)])(\d+)$", prev)
            if lead and num_t.strip().isdigit() and den_t.strip().isdigit():
                out = [prev[: len(prev) - len(lead.group(1))], f"({lead.group(1)}+({num_t})/({den_t}))"]
            else:
                out.append(f"(({num_t})/({den_t}))")
            i = j
            continue
        if s[i] == "^":
            body, i = _arg(s, i + 1)
            out.append(f"**({latex_to_sympy_text(body)})")
            continue
        m = re.match(r"\\[a-zA-Z]+", s[i:])
        if m:
            word = m.group(0)
            out.append(_LATEX_WORDS.get(word, word[1:]))
            i += len(word)
            continue
        out.append(s[i])
        i += 1
    text = "".join(out).replace("{", "(").replace("}", ")")
    return text


def _split_top(s: str, sep: str = ","):
    parts, depth, cur = [], 0, ""
    for ch in s:
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        if ch == sep and depth == 0:
            parts.append(cur)
            cur = ""
        else:
            cur += ch
    parts.append(cur)
    return [p.strip() for p in parts]


def _parse_sympy(text: str):
    import sympy
    from sympy.parsing.sympy_parser import (convert_xor, implicit_multiplication_application, parse_expr,
                                            standard_transformations)

    tr = standard_transformations + (implicit_multiplication_application, convert_xor)
    text = text.strip()
    if "=" in text:  # "x = 3" -> 3; an equation of expressions compares as lhs - rhs
        lhs, rhs = text.split("=", 1)
        if re.fullmatch(r"\s*[a-zA-Z]\s*", lhs):
            text = rhs
        else:
            return sympy.simplify(parse_expr(lhs, transformations=tr) - parse_expr(rhs, transformations=tr))
    return parse_expr(text, transformations=tr, evaluate=True)


def _expr_equal(a_text: str, b_text: str) -> bool:
    import sympy

    a, b = _parse_sympy(a_text), _parse_sympy(b_text)
    try:
        if sympy.simplify(a - b) == 0:
            return True
    except Exception:
        pass
    try:
        fa, fb = complex(sympy.N(a)), complex(sympy.N(b))
        return abs(fa - fb) <= 1e-6 * max(1.0, abs(fa), abs(fb))
    except Exception:
        return False


def _plus_minus(text: str):
    if "\\pm" not in text:
        return None
    lhs, rhs = text.split("\\pm", 1)
    return [f"{lhs}+{rhs}", f"{lhs}-{rhs}"]


def _sympy_equal(pred: str, gt: str) -> bool:
    """LaTeX-aware symbolic comparison: single expressions, ``\\pm`` pairs, ordered tuples, unordered
    sets (``\\{...\\}`` or bare comma lists) and intervals (bracket types must match)."""
    try:
        import sympy  # noqa: F401
    except Exception:
        return False
    try:
        pm_p, pm_g = _plus_minus(pred), _plus_minus(gt)
        if pm_p or pm_g:
            ps = pm_p or _split_top(pred)
            gs = pm_g or _split_top(gt)
            return _lists_equal(ps, gs, ordered=False)
        p, g = latex_to_sympy_text(pred).strip(), latex_to_sympy_text(gt).strip()
        interval = re.compile(r"^([\[(])(.*)([\])])$")
        mp, mg = interval.match(p), interval.match(g)
        if mp and mg and len(_split_top(mp.group(2))) == 2 and len(_split_top(mg.group(2))) == 2:
            if mp.group(1) + mp.group(3) != mg.group(1) + mg.group(3) and "(" not in (mp.group(1) + mg.group(1)):
                return False
            ordered = True
            return (mp.group(1) == mg.group(1) and mp.group(3) == mg.group(3)
                    and _lists_equal(_split_top(mp.group(2)), _split_top(mg.group(2)), ordered))
        is_set = pred.strip().startswith("\\{") or gt.strip().startswith("\\{")
        if is_set:
            p, g = p.strip("() "), g.strip("() ")
        ps, gs = _split_top(p), _split_top(g)
        if len(ps) > 1 or len(gs) > 1:
            return _lists_equal(ps, gs, ordered=not is_set and not (len(ps) > 1 and len(gs) > 1 and
                                                                    not p.startswith("(")))
        return _expr_equal(p, g)
    except Exception:
        return False


def _lists_equal(ps, gs, ordered: bool) -> bool:
    if len(ps) != len(gs):
        return False
    ps = [latex_to_sympy_text(x) for x in ps]
    gs = [latex_to_sympy_text(x) for x in gs]
    if ordered:
        return all(_expr_equal(a, b) for a, b in zip(ps, gs))
    left = list(gs)
    for a in ps:
        hit = next((k for k, b in enumerate(left) if _expr_equal(a, b)), None)
        if hit is None:
            return False
        left.pop(hit)
    return True


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
    if p == g or _normalised_equal(p, g):
        return True
    if fast:
        return False
    return _sympy_equal(pred, gt) or _math_verify_equal(pred, gt)


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


def question_only_reward_fn(response: str, ground_truth: Union[str, int, float, Iterable],
                            fast: bool = True) -> Dict[str, float]:
    """Reward of a free-form response: its last ``\\boxed{}`` graded against the ground truth (no
    ``<answer>`` tags needed); nothing boxed earns nothing, a boxed wrong answer earns the format
    reward only."""
    answer = extract_boxed(response)
    if answer is None:
        return {"format_reward": 0.0, "answer_reward": 0.0, "reward": 0.0}
    if isinstance(ground_truth, (int, float)):
        gts = [str(ground_truth)]
    elif isinstance(ground_truth, str):
        gts = [ground_truth]
    else:
        gts = [str(g) for g in ground_truth]
    ok = any(grade_answer(answer, g, fast) for g in gts)
    return {"format_reward": 1.0, "answer_reward": 1.0 if ok else 0.0, "reward": 1.0 if ok else 0.0}


def repeatness(text: str, threshold: float = 0.2) -> bool:
    """Whether ``text`` repeats itself: the summed longest-common-prefix lengths of its adjacent sorted
    suffixes, as a fraction of the ``n (n + 1) / 2`` characters of all its suffixes, exceed
    ``threshold`` (the reference's degenerate-output check, ``drgrpo_grader.py:452-492``).
    Suffixes are sorted by prefix doubling; the LCPs come from Kasai's algorithm."""
    n = len(text)
    if n <= 1:
        return False
    rank = [ord(c) for c in text]
    sa = list(range(n))
    k = 1
    while True:
        key = lambda i: (rank[i], rank[i + k] if i + k < n else -1)  # noqa: E731
        sa.sort(key=key)
        new = [0] * n
        for j in range(1, n):
            new[sa[j]] = new[sa[j - 1]] + (key(sa[j]) != key(sa[j - 1]))
        rank = new
        if rank[sa[-1]] == n - 1 or k >= n:
            break
        k <<= 1
    lcp_sum, h = 0, 0
    for i in range(n):  # Kasai: h drops by at most one from suffix i to suffix i + 1
        if rank[i] == n - 1:
            h = 0
            continue
        j = sa[rank[i] + 1]
        while i + h < n and j + h < n and text[i + h] == text[j + h]:
            h += 1
        lcp_sum += h
        if h:
            h -= 1
    return lcp_sum * 2 / (n * (n + 1)) > threshold
