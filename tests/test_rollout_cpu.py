"""Rollout-side behaviour on the CPU: abort/resubmit/version handling of both generation front-ends
(the four behaviours of the reference's test_vllm_local_rollout_engine.py plus the runner), replay
buffer and statistics, TextWorld prompting/parser/reward, and episode -> RLSample construction."""

import asyncio
from types import SimpleNamespace

import pytest

from accerl_agent_b200.env.synthetic import SyntheticGameConfig, SyntheticTextGame
from accerl_agent_b200.env.textworld import (
    clean_action_text,
    format_user_content,
    parse_model_action,
    step_reward,
    transcript_user_suffix,
)
from accerl_agent_b200.replay import ReplayBuffer, RolloutStats
from accerl_agent_b200.rollout.episode import StepRecord, build_episode_rl_sample
from accerl_agent_b200.rollout.generation import (
    InferenceResult,
    InterruptibleGenerationRunner,
    OnlineGenerationState,
    normalize_stop_reason,
)
from accerl_agent_b200.rollout.local_engine import GenerationConfig, LocalRolloutEngine, RolloutRequest


class FakeSamplingParams:
    def __init__(self, **kwargs):
        self.kwargs = kwargs


def output(token_ids, finished, finish_reason=None, logprobs=None):
    return SimpleNamespace(finished=finished, outputs=[SimpleNamespace(token_ids=token_ids, finish_reason=finish_reason,
                                                                       logprobs=logprobs)])


class PlannedEngine:
    def __init__(self, plans):
        self.plans = list(plans)
        self.generate_calls = []
        self.pause_calls = []
        self.resume_calls = 0
        self.collective_rpc_calls = []

    async def generate(self, prompt, sampling_params, request_id):
        self.generate_calls.append((prompt, sampling_params, request_id))
        for item in self.plans.pop(0):
            if callable(item):
                item()
                await asyncio.sleep(0)
                continue
            yield item

    async def pause_generation(self, **kwargs):
        self.pause_calls.append(kwargs)

    async def collective_rpc(self, method, kwargs):
        self.collective_rpc_calls.append((method, kwargs))

    async def resume_generation(self):
        self.resume_calls += 1


class BlockingAbortEngine(PlannedEngine):
    def __init__(self):
        super().__init__([])
        self.partial_ready = asyncio.Event()
        self.pause_called = asyncio.Event()

    async def generate(self, prompt, sampling_params, request_id):
        self.generate_calls.append((prompt, sampling_params, request_id))
        if len(self.generate_calls) == 1:
            yield output([10, 11], finished=False)
            self.partial_ready.set()
            await self.pause_called.wait()
            yield output([10, 11], finished=True, finish_reason="abort")
        else:
            yield output([12, 13], finished=True, finish_reason="length")

    async def pause_generation(self, **kwargs):
        await super().pause_generation(**kwargs)
        self.pause_called.set()


def make_request(input_ids=None, max_new_tokens=4):
    input_ids = [1, 2] if input_ids is None else input_ids
    g = GenerationConfig(n_samples=1, max_new_tokens=max_new_tokens, max_tokens=len(input_ids) + max_new_tokens,
                         greedy=True)
    return RolloutRequest(rid="req", input_ids=input_ids, gconfig=g)


def run(coro):
    return asyncio.run(coro)


def test_normal_generation_finishes_once_with_version_zero():
    engine = PlannedEngine([[output([10, 11, 12], finished=True, finish_reason="stop")]])
    rollout = LocalRolloutEngine(engine, sampling_params_cls=FakeSamplingParams)
    resp = run(rollout.agenerate(make_request(max_new_tokens=3)))
    assert resp.input_tokens == [1, 2]
    assert resp.output_tokens == [10, 11, 12]
    assert resp.output_versions == [0, 0, 0]
    assert resp.stop_reason == "stop"
    assert len(engine.generate_calls) == 1
    assert engine.generate_calls[0][0] == {"prompt_token_ids": [1, 2]}


def test_pause_update_resume_resubmits_with_new_version():
    async def scenario():
        engine = BlockingAbortEngine()
        rollout = LocalRolloutEngine(engine, sampling_params_cls=FakeSamplingParams)
        task = asyncio.create_task(rollout.agenerate(make_request(max_new_tokens=4)))
        await engine.partial_ready.wait()
        await rollout.pause_generation()
        await rollout.update_weights("/tmp/checkpoint")
        await rollout.continue_generation()
        return engine, await task

    engine, resp = run(scenario())
    assert resp.output_tokens == [10, 11, 12, 13]
    assert resp.output_versions == [0, 0, 1, 1]
    assert resp.stop_reason == "length"
    assert engine.generate_calls[1][0] == {"prompt_token_ids": [1, 2, 10, 11]}


def test_generation_never_exceeds_max_new_tokens():
    engine = PlannedEngine([[output([10, 11, 12, 13, 14], finished=True, finish_reason="length")]])
    rollout = LocalRolloutEngine(engine, sampling_params_cls=FakeSamplingParams)
    resp = run(rollout.agenerate(make_request(max_new_tokens=3)))
    assert resp.output_tokens == [10, 11, 12]
    assert resp.output_versions == [0, 0, 0]
    assert resp.stop_reason == "length"
    assert engine.generate_calls[0][1].kwargs["max_tokens"] == 3


def test_lifecycle_methods_manage_pause_state():
    async def scenario():
        engine = PlannedEngine([])
        rollout = LocalRolloutEngine(engine, sampling_params_cls=FakeSamplingParams)
        await rollout.pause_generation()
        assert rollout.paused.is_set()
        assert engine.pause_calls == [{"mode": "abort", "clear_cache": True}]
        await rollout.update_weights("/tmp/weights")
        assert rollout.version == 1
        assert engine.collective_rpc_calls == [
            ("reload_weights", {"weights_path": "/tmp/weights", "is_checkpoint_format": True})
        ]
        await rollout.continue_generation()
        assert not rollout.paused.is_set()
        assert engine.resume_calls == 1

    run(scenario())


def test_interruptible_runner_keeps_partial_tokens_across_abort():
    async def scenario():
        engine = BlockingAbortEngine()
        runner = InterruptibleGenerationRunner(engine, temperature=1.0, top_p=1.0, stop_sequences=["\n"],
                                               collect_logprobs=False, sampling_params_cls=FakeSamplingParams)
        state = OnlineGenerationState(index=0, input_ids=[1, 2], requested_max_tokens=4)
        task = asyncio.create_task(runner.generate(state))
        await engine.partial_ready.wait()
        runner.pause()
        await engine.pause_generation(mode="abort", clear_cache=True)
        await runner.wait_for_idle()
        assert runner.active_attempts == 0
        runner.version += 1
        runner.resume()
        return engine, await task

    engine, state = run(scenario())
    assert state.output_tokens == [10, 11, 12, 13]
    assert state.output_versions == [0, 0, 1, 1]
    assert state.stop_reason == "length"
    assert engine.generate_calls[1][0] == {"prompt_token_ids": [1, 2, 10, 11]}
    assert engine.generate_calls[1][1].kwargs["max_tokens"] == 2


def test_runner_logprob_mismatch_counts_as_abort_and_retries():
    engine = PlannedEngine([
        [output([5, 6], finished=True, finish_reason="stop", logprobs=[{5: -0.1}])],
        [output([5], finished=True, finish_reason="stop", logprobs=[{5: SimpleNamespace(logprob=-0.3)}])],
    ])
    runner = InterruptibleGenerationRunner(engine, collect_logprobs=True, sampling_params_cls=FakeSamplingParams)
    state = run(runner.generate(OnlineGenerationState(index=1, input_ids=[1], requested_max_tokens=3)))
    assert state.output_tokens == [5] and state.output_logprobs == [-0.3] and state.stop_reason == "stop"
    assert engine.generate_calls[0][1].kwargs["logprobs"] == 1


def test_runner_gives_up_after_max_retries():
    engine = PlannedEngine([[] for _ in range(3)])
    runner = InterruptibleGenerationRunner(engine, max_resubmit_retries=3, sampling_params_cls=FakeSamplingParams)
    state = run(runner.generate(OnlineGenerationState(index=2, input_ids=[1], requested_max_tokens=3)))
    assert state.stop_reason == "abort" and state.output_tokens == []


def test_stop_reason_normalisation():
    assert normalize_stop_reason("eos") == "stop"
    assert normalize_stop_reason("stop_sequence") == "stop"
    assert normalize_stop_reason(None) == "abort"
    assert normalize_stop_reason("length") == "length"


def test_replay_fifo_eviction_and_counters():
    rb = ReplayBuffer(3, seed=0)
    stats = rb.add_samples([1, 2])
    assert stats["size"] == 2 and stats["total_samples_evicted"] == 0
    stats = rb.add_samples([3, 4, 5])
    assert stats["size"] == 3 and stats["total_samples_evicted"] == 2 and stats["total_samples_added"] == 5
    assert rb.snapshot() == [3, 4, 5]
    got = rb.sample(10)
    assert sorted(got) == [3, 4, 5] and len(rb) == 3  # sampling does not remove
    assert rb.get_stats()["total_samples_sampled"] == 3
    assert rb.sample(0) == []
    # one call larger than the ring keeps its newest samples in order
    stats = rb.add_samples([6, 7, 8, 9, 10])
    assert rb.snapshot() == [8, 9, 10] and stats["total_samples_evicted"] == 7
    rb.add_samples([11])
    assert rb.snapshot() == [9, 10, 11]


def test_rollout_stats_window_and_active_workers():
    now = [100.0]
    st = RolloutStats(window_size=2, active_timeout_seconds=10, clock=lambda: now[0])
    st.add_textworld_episode(0, 1.0, 4.0, False, 10, 2)
    st.add_textworld_episode(1, 4.0, 4.0, True, 5, 0)
    st.add_textworld_episode(1, 2.0, 4.0, False, 5, 5)
    s = st.get_stats()
    assert s["active_workers"] == 2
    assert s["tw_win_rate"] == 0.5
    assert s["tw_normalized_score"] == 6.0 / 8.0
    assert s["tw_invalid_action_rate"] == 5 / 10
    now[0] = 1000.0
    assert st.get_stats()["active_workers"] == 0


def test_action_parser():
    cmds = ["go north", "take red apple", "Open Door"]
    assert parse_model_action("> go north\nmore", cmds).action == "go north"
    assert parse_model_action("Action: Take  RED apple.", cmds).action == "take red apple"
    assert parse_model_action("`open door`", cmds).action == "Open Door"
    assert parse_model_action("command: answer: go north", cmds).action == "go north"
    p = parse_model_action("dance", cmds)
    assert p.action is None and p.normalized == "dance"
    assert clean_action_text("") == ""


def test_prompt_and_reward_helpers():
    text = format_user_content("You see a door.", {"objective": "Win", "inventory": "nothing",
                                                    "admissible_commands": ["open door"]})
    assert "Objective:\nWin" in text and "- open door" in text and text.endswith("Return one command only.")
    tok = SimpleNamespace(apply_chat_template=lambda *a, **k: "", chat_template="<|im_start|>x<|im_end|>")
    suffix = transcript_user_suffix("hi", tok)
    assert suffix == "<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    bad = SimpleNamespace(apply_chat_template=lambda *a, **k: "", chat_template="{{ message }}")
    with pytest.raises(ValueError):
        transcript_user_suffix("hi", bad)
    assert step_reward(1.0, 3.0, True, False, 0.1, 1.0, 0.5) == pytest.approx(2.9)
    assert step_reward(1.0, 1.0, False, True, 0.0, 1.0, 0.5) == -0.5


def _rec(prompt, tokens, stop="stop", reward=0.0, version=0):
    return StepRecord(InferenceResult(tokens, [-0.5] * len(tokens), [version] * len(tokens), stop), prompt, reward)


def test_episode_sample_grpo_keeps_aborted_context():
    recs = [
        _rec([1, 2, 3], [10, 11]),
        _rec([1, 2, 3, 10, 11, 4], [12], stop="abort"),
        _rec([1, 2, 3, 10, 11, 4, 12, 5], [13, 14], version=1),
    ]
    s = build_episode_rl_sample(recs, "grpo", history_window=100, sample_advantage=0.7)
    assert s.input_ids == [1, 2, 3, 10, 11, 4, 12, 5, 13, 14]
    assert s.labels == [-100, -100, -100, 10, 11, -100, -100, -100, 13, 14]
    assert s.response_indices == [-1, -1, -1, 0, 0, -1, -1, -1, 1, 1]
    assert s.output_versions == [0, 0, 1, 1]
    assert s.token_advantages[3] == 0.7 and s.token_advantages[0] == 0.0
    assert build_episode_rl_sample(recs, "grpo", history_window=5, sample_advantage=0.7) is None


def test_episode_sample_ppo_rewards_to_go_and_prefix_check():
    recs = [_rec([1, 2], [10, 11], reward=1.0), _rec([1, 2, 10, 11, 3], [12], reward=2.0)]
    s = build_episode_rl_sample(recs, "ppo", history_window=100, gamma=1.0)
    assert s.token_advantages == [0.0, 0.0, 3.0, 3.0, 0.0, 2.0]
    broken = [_rec([1, 2], [10]), _rec([9, 9, 9], [11])]
    assert build_episode_rl_sample(broken, "ppo", history_window=100) is None


def test_synthetic_game_is_seeded():
    cfg = SyntheticGameConfig(vocab_size=100, max_steps=5, end_prob=0.0, reward_prob=0.5)
    a, b = SyntheticTextGame(3, cfg), SyntheticTextGame(3, cfg)
    oa, _ = a.reset()
    ob, _ = b.reset()
    assert oa == ob and 64 <= len(oa) <= 256
    steps = 0
    done = False
    while not done:
        _, r, done, info = a.step([1])
        steps += 1
        assert r in (0.0, 1.0)
    assert steps == 5 and info["moves"] == 5


def test_eval_script_synthetic_cpu():
    """The TextWorld evaluation entry point end to end on the synthetic game (CPU engine)."""
    from accerl_agent_b200.eval_textworld import main

    summary = main(["--model-path", "tiny-qwen2", "--env", "synthetic", "--device", "cpu", "--episodes", "3",
                    "--max-episode-steps", "2", "--num-samples", "2", "--max-action-tokens", "4", "--game-limit", "2"])
    assert summary["episodes"] == 3 and summary["avg_steps"] == 2.0


def test_history_prompt_keeps_last_turns():
    from accerl_agent_b200.eval_textworld import history_prompt

    infos = {"objective": "win", "admissible_commands": ["go north", "look"], "inventory": "nothing"}
    turns = [{"kind": "env", "action": f"a{i}", "pre_obs": f"pre{i}", "pre_infos": infos, "obs": f"obs{i}",
              "infos": infos} for i in range(5)]
    turns.append({"kind": "illegal", "action": "dance", "pre_obs": "obs4", "pre_infos": infos, "obs": "obs4",
                  "infos": infos})
    p = history_prompt("start", infos, turns, None, history_steps=2)
    assert "pre4" in p and "a4" in p and "dance" in p and "a3" not in p and "start" not in p
    p0 = history_prompt("start", infos, [], None, history_steps=0)
    assert "start" in p0


def test_engine_socket_transport_round_trip(tmp_path):
    """Rollout worker processes reach the engine over a Unix socket: concurrent requests are answered
    in completion order with tokens, log-probs, versions and stop reason; an engine error fails only
    its own request; a closed server fails pending requests instead of hanging them."""
    from accerl_agent_b200.rollout.remote import EngineClient, EngineRequestServer

    class Service:
        async def request_batch(self, ids, max_tokens):
            if ids[0] == 666:
                raise ValueError("bad prompt")
            await asyncio.sleep(0.01 * (5 - len(ids)))  # shorter prompts finish later
            return InferenceResult([ids[-1] + 1] * max_tokens, [-0.5] * max_tokens, [3] * max_tokens, "length")

    async def scenario():
        server = EngineRequestServer(Service(), str(tmp_path / "e.sock"))
        await server.start()
        client = EngineClient(server.path)
        await client.connect()
        results = await asyncio.gather(*(client.request_batch(list(range(n)), n) for n in (1, 2, 3, 4)))
        with pytest.raises(RuntimeError, match="bad prompt"):
            await client.request_batch([666], 2)
        ok = await client.request_batch([7, 8], 1)
        await server.close()
        with pytest.raises(ConnectionError):
            await asyncio.wait_for(client.request_batch([1], 1), 5)
        await client.close()
        return results, ok

    results, ok = run(scenario())
    for n, r in zip((1, 2, 3, 4), results):
        assert r.output_tokens == [n] * n and r.output_versions == [3] * n and r.stop_reason == "length"
    assert ok.output_tokens == [9]


def test_rule_based_textworld_sanity_run():
    """The rule-based TextWorld sanity script on a fake game: walkthrough first, then coin, movement,
    look; stops when the game is done."""
    from accerl_agent_b200.textworld_gym import play, rule_action

    assert rule_action({"policy_commands": ["open box"], "admissible_commands": ["go north"]}) == "open box"
    assert rule_action({"admissible_commands": ["look", "go west", "take coin from table"]}) == "take coin from table"
    assert rule_action({"admissible_commands": ["inventory", "look", "go east"]}) == "go east"
    assert rule_action({"admissible_commands": ["inventory", "look"]}) == "look"
    assert rule_action({"admissible_commands": ["inventory"]}) == "inventory"
    assert rule_action({}) == "look"

    class Game:
        def __init__(self):
            self.t = 0
            self.closed = False

        def reset(self):
            return "room", {"objective": "find the coin", "admissible_commands": ["look", "go north"]}

        def step(self, action):
            self.t += 1
            won = action == "take coin"
            return f"obs{self.t}", int(won), won, {"won": won, "lost": False,
                                                  "admissible_commands": ["take coin"] if self.t == 2 else ["go north"]}

        def close(self):
            self.closed = True

    g = Game()
    res = play(g, 20, log=lambda s: None)
    assert res["actions"] == ["go north", "go north", "take coin"] and res["won"] and res["done"] and g.closed
    res = play(Game(), 2, log=lambda s: None)
    assert res["steps"] == 2 and not res["done"]
