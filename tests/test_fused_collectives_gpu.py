"""Fused peer-memory optimizer step (reduce-scatter + norm, AdamW + all-gather push) against the NCCL
path, on 2 GPUs of one node."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, port, fused, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["ACCERL_FUSED_COLLECTIVES"] = "1" if fused else "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank))
    from accerl_agent_b200.models.config import ModelConfig
    from accerl_agent_b200.models.transformer import build_model
    from accerl_agent_b200.parallel.fsdp import ShardedAdamW

    cfg = ModelConfig(vocab_size=4096, hidden_size=256, num_hidden_layers=2, num_attention_heads=2,
                      num_key_value_heads=1, head_dim=128, intermediate_size=512)
    m = build_model(cfg, "full", torch.device("cuda", rank), torch.bfloat16, pad_to=2)
    m.init_weights(seed=0)
    opt = ShardedAdamW(m, lr=1e-3, weight_decay=0.01)
    assert opt.fused == fused
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    for step in range(3):
        m.grads.copy_(torch.randn(m.grads.shape, generator=g, device=m.grads.device) * (1 + rank))
        opt.step(1e-3)
    torch.cuda.synchronize()
    q.put((rank, fused, m.params.float().cpu(), opt.master.cpu(), float(m.grads.abs().max())))
    dist.barrier()
    dist.destroy_process_group()


def _run(fused):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, fused, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return {o[0]: o for o in out}


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_step_matches_nccl_step():
    ref = _run(False)
    fus = _run(True)
    for r in (0, 1):
        assert fus[r][4] == 0.0  # full gradient buffer zeroed for the next accumulation
        assert torch.allclose(fus[r][3], ref[r][3], atol=1e-6, rtol=1e-5)
        assert torch.allclose(fus[r][2], ref[r][2], atol=1e-2, rtol=1e-2)
    # every rank holds the same full parameter copy after the push all-gather
    assert torch.equal(fus[0][2], fus[1][2])
