"""TextWorld adapter: prompting, incremental transcripts, the action parser and the step reward.

The prompt and parser behaviour matches agent_textworld.py:2122-2271:

* the initial prompt is the chat template over a fixed system prompt and a user message with the
  objective, observation, inventory and admissible commands;
* after each action only the Qwen suffix ``<|im_end|>\\n<|im_start|>user\\n...<|im_end|>\\n<|im_start|>assistant\\n``
  is tokenized and appended, so each request's prompt is a token prefix of the next one (prefix caching
  hits); a chat template without ``<|im_start|>``/``<|im_end|>`` is rejected;
* the parser keeps the first line, strips ``>`` and ``action:``-style prefixes (up to four times),
  trailing dots, quotes and backticks, lower-cases, collapses whitespace and matches the normalised
  admissible commands exactly;
* step reward ``score_after - score_before - step_penalty (+win_bonus) (-lost_penalty)``.

``textworld`` itself is imported lazily: it is only needed to load ``.z8`` games.
"""

from __future__ import annotations

import glob
import os
import random
from dataclasses import dataclass
from typing import Dict, List, Optional

TEXTWORLD_SYSTEM_PROMPT = (
    "You are a TextWorld action selector. Reply with exactly one command "
    "from the admissible commands. Do not add explanations, punctuation, "
    "quotes, or a leading prompt marker."
)

_ACTION_PREFIXES = ("action:", "command:", "assistant:", "answer:", "output:", "input:")


@dataclass
class ParsedAction:
    normalized: str
    action: Optional[str]


def clean_action_text(text: str) -> str:
    lines = text.splitlines()
    cleaned = (lines[0] if lines else text).strip()
    for _ in range(4):
        cleaned = cleaned.strip().lstrip(">").strip()
        lower = cleaned.lower()
        for prefix in _ACTION_PREFIXES:
            if lower.startswith(prefix):
                cleaned = cleaned[len(prefix):]
                break
        else:
            break
    cleaned = cleaned.strip()
    for _ in range(2):
        cleaned = cleaned.rstrip(".")
        cleaned = cleaned.strip("'\"`")
    return " ".join(cleaned.lower().split())


def parse_model_action(raw_text: str, admissible_commands: List[str]) -> ParsedAction:
    normalized = clean_action_text(raw_text)
    by_norm = {" ".join(c.lower().split()): c for c in admissible_commands}
    return ParsedAction(normalized=normalized, action=by_norm.get(normalized))


def format_user_content(obs: str, infos: Dict) -> str:
    objective = infos.get("objective") or ""
    inventory = infos.get("inventory") or ""
    commands = infos.get("admissible_commands", []) or []
    lines = "\n".join(f"- {c}" for c in commands)
    return (
        "Objective:\n"
        f"{objective}\n\n"
        "Observation:\n"
        f"{obs}\n\n"
        "Inventory:\n"
        f"{inventory}\n\n"
        "Admissible commands:\n"
        f"{lines}\n\n"
        "Return one command only."
    )


def format_illegal_action_feedback(action: str, obs: str, infos: Dict) -> str:
    return f'Illegal action: "{action}" is not an admissible command.\n\n' + format_user_content(obs, infos)


def encode_fragment(tokenizer, text: str) -> List[int]:
    try:
        return list(tokenizer.encode(text, add_special_tokens=False))
    except TypeError:
        return list(tokenizer.encode(text))


def transcript_user_suffix(user_content: str, tokenizer=None) -> str:
    if tokenizer is not None and hasattr(tokenizer, "apply_chat_template"):
        template = getattr(tokenizer, "chat_template", "") or ""
        if "<|im_start|>" not in template or "<|im_end|>" not in template:
            raise ValueError(
                "--tw-history-token-window requires a Qwen-style <|im_start|>/<|im_end|> chat template "
                "when using apply_chat_template."
            )
        return f"<|im_end|>\n<|im_start|>user\n{user_content}<|im_end|>\n<|im_start|>assistant\n"
    return f"\n\nUser:\n{user_content}\n\nAssistant:"


def encode_transcript_user_suffix(user_content: str, tokenizer) -> List[int]:
    return encode_fragment(tokenizer, transcript_user_suffix(user_content, tokenizer=tokenizer))


def format_initial_prompt(obs: str, infos: Dict, tokenizer=None) -> str:
    user = format_user_content(obs, infos)
    if tokenizer is not None and hasattr(tokenizer, "apply_chat_template"):
        return tokenizer.apply_chat_template(
            [{"role": "system", "content": TEXTWORLD_SYSTEM_PROMPT}, {"role": "user", "content": user}],
            tokenize=False,
            add_generation_prompt=True,
        )
    return f"System: {TEXTWORLD_SYSTEM_PROMPT}\n\nUser:\n{user}\n\nAssistant:"


def step_reward(
    score_before: float, score_after: float, won: bool, lost: bool, step_penalty: float, win_bonus: float, lost_penalty: float
) -> float:
    reward = score_after - score_before - step_penalty
    if won:
        reward += win_bonus
    if lost:
        reward -= lost_penalty
    return float(reward)


def textworld_score(step_score, infos: Dict) -> float:
    try:
        return float(infos.get("score", step_score))
    except (TypeError, ValueError):
        return 0.0


def textworld_max_score(infos: Dict) -> float:
    try:
        return float(infos.get("max_score", 0))
    except (TypeError, ValueError):
        return 0.0


def load_game_files(game_dir: str, pattern: str, seed: int, limit: Optional[int]) -> List[str]:
    files = sorted(p for p in glob.glob(os.path.join(game_dir, pattern)) if os.path.isfile(p))
    random.Random(seed).shuffle(files)
    if limit is not None:
        files = files[:limit]
    if not files:
        raise ValueError(f"No TextWorld game files found: tw_game_dir={game_dir!r} tw_game_pattern={pattern!r}")
    return files


def make_textworld_env(game_file: str, max_episode_steps: int, policy_commands: bool = False):
    """Register and build one TextWorld gym env (imports ``textworld`` on demand). ``policy_commands``
    also requests the game's walkthrough (debugging only: it reveals the solution)."""
    try:
        import textworld
        import textworld.gym
    except ImportError as exc:  # pragma: no cover - depends on the optional package
        raise RuntimeError("TextWorld games need the 'textworld' package; use --env synthetic otherwise") from exc
    infos = textworld.EnvInfos(
        objective=True, inventory=True, admissible_commands=True, score=True,
        max_score=True, won=True, lost=True, moves=True, policy_commands=policy_commands,
    )
    env_id = textworld.gym.register_game(game_file, request_infos=infos, max_episode_steps=max_episode_steps)
    return textworld.gym.make(env_id)
