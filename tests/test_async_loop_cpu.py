"""The whole asynchronous loop on CPU ranks (gloo): two trainer processes, one engine process with
rollout workers on the synthetic game, weight syncs with version bumps, and the HF checkpoint.
Also the actor runtime's failure detection (a dying actor fails its pending calls)."""

import json
import os

import pytest

from accerl_agent_b200.agent_textworld import main
from accerl_agent_b200.runtime.actors import ActorDied, ActorError, get, spawn_actor


def test_async_loop_end_to_end_cpu(tmp_path):
    log = tmp_path / "run"
    main([
        "--model-path", "tiny-qwen2", "--env", "synthetic", "--device", "cpu", "--fsdp-world-size", "2",
        "--infer-size", "1", "--num-rollout-workers", "2", "--rollout-batch-size", "2",
        "--tw-max-episode-steps", "4", "--tw-history-token-window", "256", "--max-length", "256",
        "--train-packing", "varlen", "--train-token-budget", "512", "--batch-size", "2", "--grad-accum-steps", "1",
        "--max-steps", "2", "--sync-every-optimizer-steps", "1", "--min-replay-size-per-rank", "2",
        "--replay-capacity", "16", "--synthetic-obs-min", "8", "--synthetic-obs-max", "16", "--infer-max-tokens", "4",
        "--log-dir", str(log), "--save-checkpoint", "--learning-rate", "1e-4", "--lr-warmup-steps", "0",
        "--dtype", "bfloat16", "--train-logprob-mode", "response_only_lm_head",
    ])
    assert (log / "args.json").exists() and (log / "command.txt").exists()
    recs = [json.loads(l) for l in open(log / "metrics.jsonl")]
    steps = [r for r in recs if "Train/Loss" in r]
    assert [r["step"] for r in steps] == [1, 2]
    for r in steps:
        assert r["Train/TokensPerSec"] > 0 and r["Infer/TokensPerSec"] > 0
        # engine sampling log-probs and trainer log-probs come from the same weights
        assert abs(r["KL/OldNewK3TokenMean"]) < 1e-2
    assert any("Sync/ElapsedSeconds" in r for r in recs)
    ck = log / "checkpoints" / "latest"
    state = json.load(open(ck / "trainer_state.json"))
    assert state["optimizer_step"] == 2 and state["fsdp_world_size"] == 2
    assert (ck / "model.safetensors").exists() and (ck / "config.json").exists()


class Flaky:
    def ping(self):
        return "pong"

    def boom(self):
        raise ValueError("bad input")

    def die(self):
        os._exit(3)


def test_actor_errors_and_death_are_reported():
    h = spawn_actor(Flaky, name="flaky")
    assert h.ping() == "pong"
    with pytest.raises(ActorError, match="bad input"):
        get(h.boom.remote())
    fut = h.die.remote()
    with pytest.raises(ActorDied):
        get(fut, timeout=30)
    with pytest.raises(ActorDied):
        h.ping()
    h.stop_process()
