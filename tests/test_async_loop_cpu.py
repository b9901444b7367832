"""The whole asynchronous loop on CPU ranks (gloo): two trainer processes, one engine process with
rollout workers on the synthetic game, weight syncs with version bumps, and the HF checkpoint.
Also the actor runtime's failure detection (a dying actor fails its pending calls)."""

import json
import os

import pytest

from accerl_agent_b200.agent_textworld import main
from accerl_agent_b200.runtime.actors import ActorDied, ActorError, get, spawn_actor


@pytest.mark.parametrize("shard_params", [False, True])
def test_async_loop_end_to_end_cpu(tmp_path, shard_params):
    """With ``--shard-params`` the engine pulls every weight from the trainer rank that stores it; the
    small old/new KL shows that it samples with the trainers' weights either way."""
    log = tmp_path / "run"
    main(["--shard-params"] * shard_params + [
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
    assert (ck / "config.json").exists()
    assert (ck / "model.safetensors.index.json").exists() if shard_params else (ck / "model.safetensors").exists()


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


class FakeTrainer:
    def __init__(self, rank, die=False):
        self.rank, self.die = rank, die

    def export_weights_handle(self):
        if self.die:
            os._exit(5)
        return {"kind": "test", "rank": self.rank}


class FakeEngine:
    def __init__(self):
        self.handle = None

    def attach_trainer_weights(self, handle):
        self.handle = handle

    def attached(self):
        return self.handle

    def die(self):
        os._exit(4)


def test_weight_handle_exchange_and_peer_drop():
    """Every engine rank gets trainer ``i % world``'s handle; a trainer that dies during the
    exchange, or an engine that died before it, fails the exchange with ``ActorDied``."""
    import time

    from accerl_agent_b200.agent_textworld import exchange_weight_handles

    trainers = [spawn_actor(FakeTrainer, r, name=f"t{r}") for r in range(2)]
    engines = [spawn_actor(FakeEngine, name=f"e{i}") for i in range(3)]
    follower = spawn_actor(FakeEngine, name="f0")
    try:
        exchange_weight_handles(trainers, engines, [[follower], [], []])
        assert [e.attached()["rank"] for e in engines] == [0, 1, 0]
        assert follower.attached()["rank"] == 0

        dead_trainer = spawn_actor(FakeTrainer, 0, True, name="tdead")
        t0 = time.monotonic()
        with pytest.raises(ActorDied):
            exchange_weight_handles([dead_trainer], engines[:1], [[]])
        assert time.monotonic() - t0 < 30
        dead_trainer.stop_process()

        with pytest.raises(ActorDied):
            get(engines[2].die.remote(), timeout=30)
        with pytest.raises(ActorDied):
            exchange_weight_handles(trainers, engines, [[], [], []])
    finally:
        for h in trainers + engines + [follower]:
            h.stop_process()
