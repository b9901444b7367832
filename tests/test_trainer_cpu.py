"""Single-rank trainer on CPU: the padded-batch step (``--train-packing padded``) and the replay
polling (warm-up, candidate draws, a timeout with the rank's replay statistics in the message)."""

import pytest
import torch

from accerl_agent_b200.core.config import make_args
from accerl_agent_b200.core.sample import RLSample
from accerl_agent_b200.replay import ReplayBuffer
from accerl_agent_b200.trainer.worker import TrainWorker


def _samples(n, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        L = 20 + 3 * i
        ids = torch.randint(3, 4096, (L,), generator=g).tolist()
        out.append(RLSample("grpo", ids, [1] * L, [-100] * 10 + ids[10:], [-6.0] * L, 0.5 - 0.2 * i, [0.0] * L,
                            [-1] * 10 + [0] * (L - 10), [0]))
    return out


def _worker(packing, rb, **kw):
    args = make_args(model_path="tiny-qwen2", train_packing=packing, train_token_budget=128, max_length=64,
                     tw_history_token_window=64, batch_size=2, grad_accum_steps=2, device="cpu",
                     min_replay_size_per_rank=2, replay_sample_timeout_seconds=kw.pop("timeout", 5.0),
                     replay_wait_sleep_seconds=0.01, dtype="float32", learning_rate=1e-3, lr_warmup_steps=0, **kw)
    return TrainWorker(args, rank=0, fsdp_world_size=1, replay_buffer=rb, device=torch.device("cpu"))


@pytest.mark.parametrize("packing", ["padded", "varlen"])
def test_one_optimizer_step(packing):
    rb = ReplayBuffer(16, seed=0)
    rb.add_samples(_samples(6))
    w = _worker(packing, rb)
    before = {n: v.clone() for n, v in w.model.named_parameters()}
    out = w.train_until_next_sync(1)
    assert w.optimizer_step == 1
    assert torch.isfinite(torch.tensor(out["segment_loss_mean"]))
    assert any(not torch.equal(before[n], v) for n, v in w.model.named_parameters())


def test_replay_warmup_timeout_names_the_rank_and_sizes():
    rb = ReplayBuffer(16, seed=0)
    rb.add_samples(_samples(1))  # below min_replay_size_per_rank = 2
    w = _worker("varlen", rb, timeout=0.2)
    # the varlen window reports a preparation failure of any rank, with this rank's original error
    with pytest.raises(RuntimeError, match=r"replay warmup: rank=0 size=1 min_replay_size_per_rank=2"):
        w.train_until_next_sync(1)
