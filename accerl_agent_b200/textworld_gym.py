"""Rule-based TextWorld sanity run: plays one game without a model and prints every step.

    python -m accerl_agent_b200.textworld_gym --game-file data/tw_games/coin_l1_seed0.z8 [--max-steps 20]

Use it to check that the games load and that the environment plumbing (observations, admissible
commands, scores, win / loss flags) behaves before spending GPU time (the reference's
accerl_agent/run_textworld_gym.py:8-100). The rule picks, in order: the next walkthrough command when
the game provides one (``--walkthrough``, which requests ``policy_commands``), an admissible command
that takes a coin, the first admissible movement, ``look``, or else the first admissible command.
"""

from __future__ import annotations

import argparse
from typing import Callable, Dict, List, Optional, Sequence

from .env.textworld import make_textworld_env


def rule_action(infos: Dict) -> str:
    walkthrough = infos.get("policy_commands") or []
    if walkthrough:
        return walkthrough[0]
    admissible: Sequence[str] = infos.get("admissible_commands") or []
    if not admissible:
        return "look"
    preferred = ([c for c in admissible if "take coin" in c] + [c for c in admissible if c.startswith("go ")]
                 + [c for c in admissible if c == "look"])
    return preferred[0] if preferred else admissible[0]


def play(env, max_steps: int, log: Callable[[str], None] = print) -> Dict:
    """Step ``env`` with ``rule_action`` until it is done or ``max_steps`` actions were taken."""
    obs, infos = env.reset()
    log("=" * 80 + f"\nInitial observation:\n{obs}\n\nObjective:\n{infos.get('objective')}")
    log("\nAdmissible commands:\n" + "\n".join(f"- {c}" for c in infos.get("admissible_commands") or []))
    score, done, steps = 0, False, 0
    actions: List[str] = []
    while not done and steps < max_steps:
        action = rule_action(infos)
        obs, score, done, infos = env.step(action)
        actions.append(action)
        steps += 1
        log("=" * 80 + f"\nStep {steps - 1}\nAction: {action}\n\nObservation:\n{obs}\n\nScore: {score}\n"
            f"Done: {done}\nWon: {infos.get('won')}\nLost: {infos.get('lost')}")
        log("\nAdmissible commands:\n" + "\n".join(f"- {c}" for c in infos.get("admissible_commands") or []))
    env.close()
    return {"steps": steps, "score": score, "done": bool(done), "won": bool(infos.get("won")),
            "lost": bool(infos.get("lost")), "actions": actions}


def main(argv: Optional[List[str]] = None) -> Dict:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--game-file", default="data/tw_games/coin_l1_seed0.z8")
    ap.add_argument("--max-steps", type=int, default=20)
    ap.add_argument("--walkthrough", action="store_true",
                    help="request the game's walkthrough commands and follow them (debugging only)")
    a = ap.parse_args(argv)
    env = make_textworld_env(a.game_file, a.max_steps, policy_commands=a.walkthrough)
    result = play(env, a.max_steps)
    print(f"\nresult: {result}")
    return result


if __name__ == "__main__":
    main()
