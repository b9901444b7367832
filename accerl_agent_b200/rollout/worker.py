"""Rollout workers: play episodes against the inference service and feed replay shards.

Behaviour follows the reference's ``TextWorldRolloutWorkerActor`` (agent_textworld.py:2274-2791):

* GRPO: a group of ``grpo_group_size`` trajectories of one game is stepped together (all active
  trajectories request their next action concurrently); trajectory reward is the sum of step rewards
  minus ``invalid_penalty * #invalid``; group-normalised advantages are broadcast to response tokens;
  invalid actions get reward 0 at step level.
* PPO: ``rollout_batch_size`` independent episodes of one game; invalid, non-aborted outputs get
  ``-invalid_penalty`` on their last token; token advantages are Monte-Carlo returns.
* Every request's prompt is the whole growing transcript; a trajectory ends when the env says done,
  after ``tw_max_episode_steps`` steps, or when the transcript reaches the history window
  (``infer_max_tokens`` is capped by the remaining window).
* Games cycle as ``(worker_id + episode_index) % n_games``; samples go to ``replay_sink`` and one
  episode record per trajectory to ``stats_sink``.

Two environments are supported: TextWorld (text observations, the chat-template transcript, the action
parser) and the seeded synthetic token-level game used by the benchmarks.
"""

from __future__ import annotations

import asyncio
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

from ..algo.advantages import grpo_group_advantages
from ..env.synthetic import SyntheticGameConfig, SyntheticTextGame
from ..env import textworld as tw
from .episode import StepRecord, build_episode_rl_sample
from .generation import InferenceResult


@dataclass
class TrajectoryState:
    env: Any
    obs: Any
    infos: Dict
    latest_score: float
    step_records: List[StepRecord] = field(default_factory=list)
    transcript_ids: List[int] = field(default_factory=list)
    invalid_actions: int = 0
    done: bool = False
    won: bool = False
    lost: bool = False


@dataclass
class PendingRequest:
    state: TrajectoryState
    prompt_obs: Any
    prompt_infos: Dict
    input_ids: List[int]
    score_before: float


class RolloutWorker:
    def __init__(self, args, infer, worker_id: int, replay_sink: Callable[[list], Any],
                 stats_sink: Callable[..., Any], tokenizer=None, game_files: Optional[List[str]] = None):
        self.args = args
        self.infer = infer
        self.worker_id = int(worker_id)
        self.replay_sink = replay_sink
        self.stats_sink = stats_sink
        self.tokenizer = tokenizer
        self.env_kind = getattr(args, "env", "textworld")
        if self.env_kind == "textworld":
            if tokenizer is None:
                raise ValueError("TextWorld rollouts need the model's tokenizer")
            self.game_files = game_files or tw.load_game_files(args.tw_game_dir, args.tw_game_pattern, args.seed,
                                                               args.tw_game_limit)
        else:
            vocab = getattr(args, "synthetic_vocab_size", None)
            if vocab is None:
                from ..models.config import resolve_model_config

                vocab = resolve_model_config(args.model_path).vocab_size
            self.syn_cfg = SyntheticGameConfig(
                vocab_size=vocab, obs_min=args.synthetic_obs_min, obs_max=args.synthetic_obs_max,
                reward_prob=args.synthetic_reward_prob, end_prob=args.synthetic_end_prob,
                max_steps=args.tw_max_episode_steps,
            )
            self.game_files = [f"synthetic-{i}" for i in range(max(1, args.tw_game_limit or 1024))]
        self.stopped = False
        self.episodes = 0

    async def stop(self) -> None:
        self.stopped = True

    # ------------------------------------------------------------------ env plumbing
    def _make_env(self, game: str, member: int):
        if self.env_kind == "textworld":
            return tw.make_textworld_env(game, self.args.tw_max_episode_steps)
        seed = hash((self.args.seed, game, member)) & 0x7FFFFFFF
        return SyntheticTextGame(seed, self.syn_cfg)

    def _initial_transcript(self, obs, infos) -> List[int]:
        if self.env_kind == "textworld":
            prompt = tw.format_initial_prompt(obs, infos, tokenizer=self.tokenizer)
            return list(self.tokenizer.encode(prompt))
        return list(obs)

    def _reset(self, env) -> TrajectoryState:
        obs, infos = env.reset()
        infos = dict(infos)
        return TrajectoryState(env=env, obs=obs, infos=infos, latest_score=tw.textworld_score(0, infos),
                               transcript_ids=self._initial_transcript(obs, infos),
                               won=bool(infos.get("won", False)), lost=bool(infos.get("lost", False)))

    def _apply_result(self, pending: PendingRequest, result: InferenceResult, invalid_reward_mode: str) -> None:
        state = pending.state
        a = self.args
        state.transcript_ids.extend(result.output_tokens)
        if self.env_kind != "textworld":
            obs, reward, done, infos = state.env.step(list(result.output_tokens))
            state.obs, state.infos, state.done = obs, dict(infos), bool(done)
            state.latest_score = float(infos.get("score", state.latest_score))
            if not state.done:
                state.transcript_ids.extend(obs)
            state.step_records.append(StepRecord(result, list(pending.input_ids), float(reward)))
            return
        commands = state.infos.get("admissible_commands", []) or []
        raw = self.tokenizer.decode(result.output_tokens, skip_special_tokens=True)
        parsed = tw.parse_model_action(raw, commands)
        if parsed.action is not None:
            obs, step_score, done, infos = state.env.step(parsed.action)
            state.obs, state.infos = obs, dict(infos)
            state.latest_score = tw.textworld_score(step_score, infos)
            state.done = bool(done)
            state.won = bool(infos.get("won", False))
            state.lost = bool(infos.get("lost", False))
            if not state.done:
                state.transcript_ids.extend(
                    tw.encode_transcript_user_suffix(tw.format_user_content(state.obs, state.infos), self.tokenizer))
            reward = tw.step_reward(pending.score_before, state.latest_score, state.won, state.lost,
                                    a.tw_step_penalty, a.tw_win_bonus, a.tw_lost_penalty)
        else:
            state.invalid_actions += 1
            bad = parsed.normalized if parsed.normalized else raw.strip()
            state.transcript_ids.extend(tw.encode_transcript_user_suffix(
                tw.format_illegal_action_feedback(bad, pending.prompt_obs, pending.prompt_infos), self.tokenizer))
            if invalid_reward_mode == "zero":
                reward = 0.0
            elif result.output_tokens and result.stop_reason != "abort":
                reward = -a.tw_invalid_action_penalty
            else:
                reward = 0.0
        state.step_records.append(StepRecord(result, list(pending.input_ids), float(reward)))

    async def _step_batch(self, states: List[TrajectoryState], invalid_reward_mode: str) -> int:
        if self.stopped:
            return 0
        active = [s for s in states if not s.done and len(s.step_records) < self.args.tw_max_episode_steps]
        if not active:
            return 0
        pending: List[PendingRequest] = []
        coros = []
        window = self.args.tw_history_token_window
        for s in active:
            ids = list(s.transcript_ids)
            if len(ids) >= window:
                s.done = True
                continue
            max_tok = min(self.args.infer_max_tokens, window - len(ids))
            coros.append(self.infer.request_batch(ids, max_tok))
            pending.append(PendingRequest(s, s.obs, dict(s.infos), ids, s.latest_score))
        if not coros:
            return len(active)
        results = await asyncio.gather(*coros)
        for p, r in zip(pending, results):
            self._apply_result(p, r, invalid_reward_mode)
        return len(active)

    def _report(self, states: List[TrajectoryState]) -> None:
        max_score = tw.textworld_max_score(states[0].infos) if states else 0.0
        for s in states:
            self.stats_sink(self.worker_id, s.latest_score, max_score, bool(s.won), len(s.step_records),
                            s.invalid_actions)

    # ------------------------------------------------------------------ episode drivers
    async def run_grpo_group(self, game: str) -> List:
        a = self.args
        states = [self._reset(self._make_env(game, i)) for i in range(int(a.grpo_group_size))]
        try:
            for _ in range(a.tw_max_episode_steps):
                if await self._step_batch(states, "zero") == 0:
                    break
            rewards = [sum(r.reward for r in s.step_records) - a.tw_invalid_action_penalty * s.invalid_actions
                       for s in states]
            _, _, advs = grpo_group_advantages(rewards, a.grpo_adv_eps)
            samples = []
            for s, adv in zip(states, advs):
                smp = build_episode_rl_sample(s.step_records, "grpo", a.tw_history_token_window, a.tw_gamma, adv)
                if smp is not None:
                    samples.append(smp)
            if samples:
                self.replay_sink(samples)
            self._report(states)
            return samples
        finally:
            for s in states:
                s.env.close()

    async def run_ppo_batch(self, game: str) -> List:
        a = self.args
        states = [self._reset(self._make_env(game, i)) for i in range(int(a.rollout_batch_size))]
        try:
            for _ in range(a.tw_max_episode_steps):
                if await self._step_batch(states, "ppo_penalty") == 0:
                    break
            samples = []
            for s in states:
                smp = build_episode_rl_sample(s.step_records, "ppo", a.tw_history_token_window, a.tw_gamma)
                if smp is not None:
                    samples.append(smp)
            if samples:
                self.replay_sink(samples)
            self._report(states)
            return samples
        finally:
            for s in states:
                s.env.close()

    async def run(self) -> Dict[str, int]:
        index = 0
        while not self.stopped:
            game = self.game_files[(self.worker_id + index) % len(self.game_files)]
            if self.args.rl_algorithm == "ppo":
                await self.run_ppo_batch(game)
            else:
                await self.run_grpo_group(game)
            index += 1
            self.episodes = index
        print(f"[rollout] worker={self.worker_id} stopped; episodes={index}")
        return {"episodes": index}
