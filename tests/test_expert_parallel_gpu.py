"""Expert parallelism over NVLink peer memory on 2 GPUs: P2P token dispatch, grouped expert GEMMs of
the local experts and the scatter-epilogue combine give the same log-probabilities as the local
grouped path and, summed over ranks, the same gradients."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _worker(rank, port, model_type, q):
    try:
        _work(rank, port, model_type, q)
    except BaseException as exc:  # report instead of leaving the parent waiting on the queue
        q.put((rank, repr(exc), None, None))
        raise


def _work(rank, port, model_type, q):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank))
    from test_model_gpu import batch_of, small_cfg

    from accerl_agent_b200.models.transformer import build_model
    from accerl_agent_b200.parallel.expert_parallel import ExpertParallel

    cfg = small_cfg(model_type, moe=True)
    dev = torch.device("cuda", rank)
    batch = {k: v.to(dev) for k, v in batch_of([300, 77 + 50 * rank, 513], cfg.vocab_size, seed=rank).items()}
    out = []
    for use_ep in (False, True):
        m = build_model(cfg, "full", dev, torch.bfloat16, pad_to=2)
        m.init_weights(seed=5, std=0.05)
        if use_ep:
            m.expert_parallel = ExpertParallel(cfg, max_tokens=1024, device=dev)
            assert m.expert_parallel.p2p
        lp, ctx = m.forward_logprobs(batch, 513)
        w = torch.linspace(-1, 1, lp.numel(), device=dev)
        m.backward_from_logprobs(w, ctx)
        g = m.grads.clone()
        dist.all_reduce(g)
        out.append((lp.float().cpu(), g.cpu()))
    # expert-partitioned storage: this rank's buffer holds only its experts
    from accerl_agent_b200.parallel.expert_parallel import expert_partition

    pcfg = expert_partition(cfg, rank, 2)
    m = build_model(pcfg, "full", dev, torch.bfloat16, pad_to=2, experts_last=True)
    m.init_weights(seed=5, std=0.05)
    m.expert_parallel = ExpertParallel(cfg, max_tokens=1024, device=dev)
    lp, ctx = m.forward_logprobs(batch, 513)
    m.backward_from_logprobs(torch.linspace(-1, 1, lp.numel(), device=dev), ctx)
    rep = m.layout.replicated_numel
    dist.all_reduce(m.grads[:rep])
    full = build_model(cfg, "full", dev, torch.bfloat16, pad_to=2)  # layout of the replicated run's grads
    full.grads.copy_(out[1][1].to(dev))
    lo, nloc = pcfg.expert_offset, pcfg.local_experts
    gerr, gmax = 0.0, 0.0
    for n in m.layout.order:
        if not m.layout.slots[n].trainable:
            continue
        want = full.g(n).float()
        if ".mlp.experts." in n:
            want = want[lo:lo + nloc]
        gerr = max(gerr, float((m.g(n).float() - want).abs().max()))
        gmax = max(gmax, float(want.abs().max()))
    torch.cuda.synchronize()
    q.put((rank, out[0][0], out[1][0], ((out[0][1], out[1][1]) if rank == 0 else None,
                                        float((lp.float().cpu() - out[1][0]).abs().max()), gerr, gmax)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("model_type", ["qwen2_moe", "qwen3_moe"])
def test_expert_parallel_p2p_matches_local(model_type):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    env_path = os.environ.get("PYTHONPATH", "")
    os.environ["PYTHONPATH"] = os.path.dirname(__file__) + (os.pathsep + env_path if env_path else "")
    ps = [ctx.Process(target=_worker, args=(r, port, model_type, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        r, lp_local, lp_ep, grads = q.get(timeout=300)
        assert not isinstance(lp_local, str), f"rank {r} failed: {lp_local}"
        res[r] = (lp_local, lp_ep, grads)
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    for r in (0, 1):
        # each expert row sees the same inputs and weights in both paths
        assert (res[r][0] - res[r][1]).abs().max() < 1e-3
        # partitioned storage: same log-probabilities, and its gradients (replicated part summed over
        # ranks, local experts as computed) equal the replicated-storage run's for the same tensors
        _, lp_diff, gerr, gmax = res[r][2]
        assert lp_diff < 1e-3, lp_diff
        assert gerr <= 2e-2 * gmax + 1e-4, (gerr, gmax)
    g_local, g_ep = res[0][2][0]
    err = (g_local - g_ep).abs().max()
    assert err <= 2e-2 * g_local.abs().max() + 1e-4, err
