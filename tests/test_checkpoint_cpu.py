"""Checkpoint and resume of the trainer on CPU: a run that saves after two optimizer steps (weights in
HF format, the optimizer shard and the counters) and resumes in a fresh worker takes the same third
step as the run that never stopped."""

import torch

from accerl_agent_b200.core.config import make_args
from accerl_agent_b200.core.sample import RLSample
from accerl_agent_b200.replay import ReplayBuffer
from accerl_agent_b200.models.hf_io import load_hf_checkpoint, save_hf_checkpoint
from accerl_agent_b200.trainer.worker import TrainWorker


def _args(**kw):
    return make_args(model_path="tiny-qwen2", train_packing="varlen", train_token_budget=64, max_length=64,
                     tw_history_token_window=64, batch_size=1, grad_accum_steps=1, device="cpu", dtype="float32",
                     min_replay_size_per_rank=1, replay_sample_timeout_seconds=5.0, replay_wait_sleep_seconds=0.01,
                     learning_rate=1e-3, max_steps=10, **kw)


def _buffer():
    rb = ReplayBuffer(8)
    rb.add_samples([RLSample("grpo", list(range(3, 19)), [1] * 16, [-100] * 8 + list(range(11, 19)), [-2.0] * 16,
                             0.8, [0.0] * 16, [-1] * 8 + [0] * 8, [0])])
    return rb


def test_resume_continues_the_same_optimisation(tmp_path):
    a = TrainWorker(_args(save_optimizer_state=True), replay_buffer=_buffer(), device=torch.device("cpu"))
    a.train_until_next_sync(2)
    a.save_checkpoint(str(tmp_path), "step2")
    files = sorted(p.name for p in (tmp_path / "step2").iterdir())
    assert "optimizer_rank00000.pt" in files and "trainer_state.json" in files
    assert any(f.endswith(".safetensors") for f in files)
    a.train_until_next_sync(1)

    b = TrainWorker(_args(resume_from=str(tmp_path / "step2")), replay_buffer=_buffer(), device=torch.device("cpu"))
    assert b.optimizer_step == 2 and b.optimizer.step_count == a.optimizer.step_count - 1
    b.train_until_next_sync(1)
    assert b.optimizer_step == a.optimizer_step == 3
    torch.testing.assert_close(b.model.params, a.model.params, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(b.optimizer.exp_avg_sq, a.optimizer.exp_avg_sq, rtol=1e-5, atol=1e-12)


def test_weights_only_checkpoint_restores_parameters(tmp_path):
    a = TrainWorker(_args(), replay_buffer=_buffer(), device=torch.device("cpu"))
    a.train_until_next_sync(1)
    a.save_checkpoint(str(tmp_path), "w")
    assert not (tmp_path / "w" / "optimizer_rank00000.pt").exists()
    b = TrainWorker(_args(), replay_buffer=_buffer(), device=torch.device("cpu"))
    b.load_checkpoint(str(tmp_path / "w"))
    assert b.optimizer_step == 1
    torch.testing.assert_close(b.model.params, a.model.params)


def test_expert_partitioned_checkpoint_round_trip(tmp_path):
    """Two ranks holding disjoint expert ranges write one HF checkpoint (replicated shards + one expert
    file per rank + an index naming every expert); it loads into the unpartitioned model and back into
    each partition."""
    from accerl_agent_b200.models.config import get_preset
    from accerl_agent_b200.models.transformer import build_model
    from accerl_agent_b200.parallel.expert_parallel import expert_partition

    cfg = get_preset("tiny-qwen2")
    cfg.vocab_size, cfg.model_type, cfg.num_experts, cfg.num_experts_per_tok = 512, "qwen2_moe", 5, 2
    cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size = 64, 96
    full = build_model(cfg, "full", torch.device("cpu"), torch.float32)
    full.init_weights(seed=7)
    parts = []
    for r in range(2):
        m = build_model(expert_partition(cfg, r, 2), "full", torch.device("cpu"), torch.float32, pad_to=2,
                        experts_last=True)
        m.init_weights(seed=7)
        parts.append(m)
    for r, m in enumerate(parts):
        written = save_hf_checkpoint(m, str(tmp_path), rank=r, world=2)
        assert f"model-experts-{r + 1:05d}-of-00002.safetensors" in written
    back = build_model(cfg, "full", torch.device("cpu"), torch.float32)
    load_hf_checkpoint(back, str(tmp_path))
    torch.testing.assert_close(back.params, full.params)
    for r in range(2):
        pcfg = expert_partition(cfg, r, 2)
        m = build_model(pcfg, "full", torch.device("cpu"), torch.float32, pad_to=2, experts_last=True)
        load_hf_checkpoint(m, str(tmp_path))
        for name in m.layout.order:
            want = full.w(name)
            if name.endswith("experts.gate_up_proj") or name.endswith("experts.down_proj"):
                want = want[pcfg.expert_offset : pcfg.expert_offset + pcfg.local_experts]
            torch.testing.assert_close(m.w(name), want)
