"""Evaluation of a policy on TextWorld games with the native engine, without training or actors.

    python -m accerl_agent_b200.eval_textworld --model-path DIR --game-dir GAMES [--episodes 20]

Behaviour of the reference's ``textworld_local_infer.py`` (``:168-377, 509-577, 674-888, 891-990``):
the prompt is the chat re-rendered from the last ``--history-steps`` action/observation turns (0 keeps
a single-state prompt), ``--num-samples`` actions are sampled per step and the first one that parses
to an admissible command is executed; an invalid step feeds the illegal-action message back instead
of advancing the game. The summary reports win rate, average (normalised) score, steps and the
invalid-action rate. Requests go through the same interruptible runner as training rollouts.

``--env synthetic`` plays the seeded token-level game of the training benchmarks instead (every
action is valid; the score is the summed reward), so the script runs where TextWorld is not installed.
``--tensor-parallel-size`` is accepted for command-line compatibility; this script runs one engine on
one GPU.
"""

from __future__ import annotations

import argparse
import asyncio
import random
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .env import textworld as tw


@dataclass
class EpisodeResult:
    index: int
    game: str
    won: bool
    lost: bool
    score: float
    max_score: float
    steps: int
    env_steps: int
    invalid_actions: int
    actions: List[str] = field(default_factory=list)

    @property
    def normalized_score(self) -> float:
        return self.score / self.max_score if self.max_score > 0 else 0.0


def history_prompt(initial_obs: str, initial_infos: Dict, turns: List[Dict], tokenizer, history_steps: int) -> str:
    if history_steps <= 0:
        last = turns[-1] if turns else {"obs": initial_obs, "infos": initial_infos}
        return tw.format_initial_prompt(last["obs"], last["infos"], tokenizer=tokenizer)
    kept = turns[-history_steps:]
    if not kept or len(kept) == len(turns):
        first_obs, first_infos = initial_obs, initial_infos
    else:
        first_obs, first_infos = kept[0]["pre_obs"], kept[0]["pre_infos"]
    messages = [{"role": "system", "content": tw.TEXTWORLD_SYSTEM_PROMPT},
                {"role": "user", "content": tw.format_user_content(first_obs, first_infos)}]
    for t in kept:
        messages.append({"role": "assistant", "content": t["action"]})
        if t["kind"] == "illegal":
            messages.append({"role": "user", "content": tw.format_illegal_action_feedback(t["action"], t["obs"], t["infos"])})
        else:
            messages.append({"role": "user", "content": tw.format_user_content(t["obs"], t["infos"])})
    if tokenizer is not None and hasattr(tokenizer, "apply_chat_template"):
        return tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
    parts = [f"System: {tw.TEXTWORLD_SYSTEM_PROMPT}"]
    for m in messages[1:]:
        parts.append(("User:\n" if m["role"] == "user" else "Assistant:\n") + m["content"])
    parts.append("Assistant:")
    return "\n\n".join(parts)


async def run_textworld_episode(index: int, game: str, service, tokenizer, a) -> EpisodeResult:
    env = tw.make_textworld_env(game, a.max_episode_steps)
    obs, infos = env.reset()
    init_obs, init_infos = obs, dict(infos)
    turns: List[Dict] = []
    invalid = env_steps = step = 0
    done = False
    score = tw.textworld_score(0, infos)
    actions: List[str] = []
    while not done and step < a.max_episode_steps:
        prompt = history_prompt(init_obs, init_infos, turns, tokenizer, a.history_steps)
        ids = list(tokenizer.encode(prompt))
        results = await asyncio.gather(*[service.request_batch(ids, a.max_action_tokens) for _ in range(a.num_samples)])
        admissible = infos.get("admissible_commands", []) or []
        texts = [tokenizer.decode(r.output_tokens, skip_special_tokens=True) for r in results]
        parsed = [tw.parse_model_action(t, admissible) for t in texts]
        chosen = next((p for p in parsed if p.valid and p.action is not None), None)
        pre_obs, pre_infos = obs, dict(infos)
        if chosen is not None:
            action = chosen.action
            obs, step_score, done, infos = env.step(action)
            env_steps += 1
            score = tw.textworld_score(step_score, infos)
            turns.append({"kind": "env", "action": action, "pre_obs": pre_obs, "pre_infos": pre_infos, "obs": obs,
                          "infos": dict(infos)})
        else:
            invalid += 1
            action = parsed[0].normalized if parsed and parsed[0].normalized else (texts[0].strip() if texts else "")
            turns.append({"kind": "illegal", "action": action, "pre_obs": pre_obs, "pre_infos": pre_infos,
                          "obs": pre_obs, "infos": pre_infos})
        actions.append(action)
        if a.verbose:
            print(f"[step] episode={index} step={step} action={action!r} valid={chosen is not None} score={score:g}")
        step += 1
    env.close() if hasattr(env, "close") else None
    return EpisodeResult(index, game, bool(infos.get("won", False)), bool(infos.get("lost", False)), score,
                         tw.textworld_max_score(infos), step, env_steps, invalid, actions)


async def run_synthetic_episode(index: int, game: str, service, a) -> EpisodeResult:
    from .env.synthetic import SyntheticGameConfig, SyntheticTextGame

    cfg = SyntheticGameConfig(vocab_size=service.cfg.vocab_size, max_steps=a.max_episode_steps)
    env = SyntheticTextGame(hash((a.seed, game)) & 0x7FFFFFFF, cfg)
    obs, _ = env.reset()
    transcript = list(obs)
    score, step, done = 0.0, 0, False
    while not done and step < a.max_episode_steps:
        results = await asyncio.gather(*[service.request_batch(transcript, a.max_action_tokens)
                                         for _ in range(a.num_samples)])
        act = list(results[0].output_tokens)
        obs, reward, done, _ = env.step(act)
        transcript += act + (list(obs) if not done else [])
        score += float(reward)
        step += 1
    return EpisodeResult(index, game, False, False, score, 0.0, step, step, 0)


def print_summary(results: List[EpisodeResult], game_count: int) -> Dict[str, float]:
    n = len(results)
    if n == 0:
        print("[eval-summary] episodes=0")
        return {"episodes": 0}
    wins = sum(r.won for r in results)
    steps = sum(r.steps for r in results)
    summary = {
        "episodes": n,
        "wins": wins,
        "win_rate": wins / n,
        "avg_score": sum(r.score for r in results) / n,
        "avg_normalized_score": sum(r.normalized_score for r in results) / n,
        "avg_steps": steps / n,
        "avg_env_steps": sum(r.env_steps for r in results) / n,
        "invalid_action_rate": sum(r.invalid_actions for r in results) / steps if steps else 0.0,
        "game_count": game_count,
    }
    print("=" * 80)
    print("[eval-summary] " + " ".join(f"{k}={v:.4f}" if isinstance(v, float) else f"{k}={v}"
                                       for k, v in summary.items()))
    return summary


def parse_args(argv: Optional[List[str]] = None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Evaluate a policy on TextWorld games with the native engine.")
    a = p.add_argument
    a("--model-path", required=True, help="Local HF model directory, or a preset name (random init).")
    a("--game-dir", default=None, help="Directory containing TextWorld .z8 games (required with --env textworld).")
    a("--game-pattern", default="*.z8")
    a("--game-limit", type=int, default=None)
    a("--episodes", type=int, default=20)
    a("--max-episode-steps", type=int, default=20)
    a("--max-action-tokens", type=int, default=16)
    a("--temperature", type=float, default=0.7)
    a("--top-p", type=float, default=1.0)
    a("--num-samples", type=int, default=4)
    a("--collect-logprobs", action="store_true")
    a("--verbose", action="store_true")
    a("--history-steps", type=int, default=8)
    a("--fallback-action", default="auto", help="Accepted for compatibility; invalid actions are fed back.")
    a("--dtype", default="bfloat16", choices=("auto", "bfloat16", "float16", "float32"))
    a("--trust-remote-code", action="store_true", default=True)
    a("--tensor-parallel-size", type=int, default=1)
    a("--enable-expert-parallel", action="store_true")
    a("--gpu-memory-utilization", type=float, default=0.7)
    a("--max-model-len", type=int, default=32768)
    a("--disable-prefix-caching", action="store_true")
    a("--vllm-max-num-seqs", type=int, default=256)
    a("--vllm-max-num-batched-tokens", type=int, default=8192)
    a("--seed", type=int, default=42)
    a("--env", default="textworld", choices=("textworld", "synthetic"))
    a("--device", default="auto")
    return p.parse_args(argv)


async def _main(a) -> Dict[str, float]:
    from .core.config import make_args
    from .core.tokenizer import load_tokenizer
    from .models.config import resolve_model_config
    from .rollout.inference import InferenceService

    random.seed(a.seed)
    cfg = resolve_model_config(a.model_path)
    use_cuda = a.device != "cpu" and torch.cuda.is_available()
    dev = torch.device("cuda", 0) if use_cuda else torch.device("cpu")
    if a.env == "textworld":
        if not a.game_dir:
            raise ValueError("--game-dir is required with --env textworld")
        games = tw.load_game_files(a.game_dir, a.game_pattern, a.seed, a.game_limit)
        tokenizer = load_tokenizer(a.model_path, a.trust_remote_code, cfg.vocab_size, fallback=True)
    else:
        games = [f"synthetic-{i}" for i in range(a.game_limit or 64)]
        tokenizer = None
    args = make_args(model_path=a.model_path, env=a.env, infer_temperature=a.temperature, infer_top_p=a.top_p,
                     vllm_max_num_seqs=a.vllm_max_num_seqs, vllm_max_num_batched_tokens=a.vllm_max_num_batched_tokens,
                     vllm_max_model_len=min(a.max_model_len, cfg.max_position_embeddings),
                     disable_vllm_prefix_caching=a.disable_prefix_caching, seed=a.seed)
    if use_cuda:
        free, _ = torch.cuda.mem_get_info(dev)
        args.kv_cache_gb = max(1.0, a.gpu_memory_utilization * free / 1024**3)
    service = InferenceService(args, dev, tokenizer=tokenizer)
    import os

    if os.path.isdir(a.model_path) and any(f.endswith(".safetensors") for f in os.listdir(a.model_path)):
        from .models.hf_io import load_hf_checkpoint

        load_hf_checkpoint(service.engine.model, a.model_path)
    else:
        service.engine.model.init_weights(seed=a.seed)
    t0 = time.perf_counter()
    jobs = []
    for i in range(a.episodes):
        game = games[i % len(games)]
        if a.env == "textworld":
            jobs.append(run_textworld_episode(i, game, service, tokenizer, a))
        else:
            jobs.append(run_synthetic_episode(i, game, service, a))
    results = await asyncio.gather(*jobs)
    summary = print_summary(list(results), len(games))
    summary["seconds"] = time.perf_counter() - t0
    await service.shutdown()
    return summary


def main(argv: Optional[List[str]] = None) -> Dict[str, float]:
    return asyncio.run(_main(parse_args(argv)))


if __name__ == "__main__":
    main()
