"""Expert parallelism on CPU ranks (gloo): the dispatch/combine plan of ``ExpertParallel`` gives the
same log-probabilities and, summed over ranks, the same gradients as every rank running all experts
on its own tokens. The row exchange is the gloo emulation; the GPU path shares the plan."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from accerl_agent_b200.algo.packing import make_varlen_batch
from accerl_agent_b200.core.sample import RLSample
from accerl_agent_b200.models.config import get_preset
from accerl_agent_b200.models.transformer import build_model
from accerl_agent_b200.parallel.expert_parallel import ExpertParallel


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg(model_type, num_experts=6):
    cfg = get_preset("tiny-qwen2")
    cfg.vocab_size = 512
    cfg.model_type = model_type
    cfg.num_experts = num_experts
    cfg.num_experts_per_tok = 2
    cfg.moe_intermediate_size = 64
    cfg.norm_topk_prob = model_type == "qwen3_moe"
    if model_type == "qwen2_moe":
        cfg.shared_expert_intermediate_size = 96
    else:
        cfg.qkv_bias = False
        cfg.qk_norm = True
    return cfg


def _pack(seed, vocab):
    g = torch.Generator().manual_seed(seed)
    out = []
    for L in (23, 11 + seed % 5):
        ids = torch.randint(0, vocab, (L,), generator=g).tolist()
        labels = [-100] * (L // 2) + ids[L // 2:]
        out.append(RLSample("grpo", ids, [1] * L, labels, [-8.0] * L, 0.5, [0.0] * L,
                            [-1] * (L // 2) + [0] * (L - L // 2), [0]))
    return make_varlen_batch(out)


def _run(model, batch):
    lp, ctx = model.forward_logprobs(batch, 32)
    dlp = torch.linspace(-1.0, 1.0, lp.numel(), dtype=lp.dtype) * 0.01
    model.backward_from_logprobs(dlp, ctx)
    return lp.detach().clone()


def _worker(rank, port, model_type, num_experts, transport, out):
    try:
        _work(rank, port, model_type, num_experts, transport, out)
    except BaseException as exc:  # report instead of leaving the parent waiting on the queue
        out.put((rank, repr(exc), None))
        raise


def _work(rank, port, model_type, num_experts, transport, out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    cfg = _cfg(model_type, num_experts)
    model = build_model(cfg, "full", torch.device("cpu"), torch.float32, pad_to=2)
    model.init_weights(seed=3)
    model.expert_parallel = ExpertParallel(cfg, max_tokens=64, device=torch.device("cpu"), dtype=torch.float32,
                                           transport=transport)
    lp = _run(model, _pack(40 + rank, cfg.vocab_size))
    grads = model.grads.clone()
    dist.all_reduce(grads)
    out.put((rank, lp, grads if rank == 0 else None))
    dist.barrier()
    dist.destroy_process_group()


def _check(model_type, num_experts=6, transport="emulated"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, model_type, num_experts, transport, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, lp, g = q.get(timeout=180)
        assert not isinstance(lp, str), f"rank {rank} failed: {lp}"
        res[rank] = (lp, g)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    cfg = _cfg(model_type, num_experts)
    model = build_model(cfg, "full", torch.device("cpu"), torch.float32, pad_to=2)
    model.init_weights(seed=3)
    lps = [_run(model, _pack(40 + r, cfg.vocab_size)) for r in range(2)]
    for r in range(2):
        torch.testing.assert_close(res[r][0], lps[r], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(res[0][1], model.grads, rtol=1e-4, atol=1e-6)


def test_expert_parallel_matches_local_experts_qwen2_moe():
    _check("qwen2_moe")


def test_expert_parallel_matches_local_experts_qwen3_moe():
    _check("qwen3_moe")


def test_expert_parallel_uneven_expert_partition():
    # 5 experts on 2 ranks: rank 0 owns 3, rank 1 owns 2
    _check("qwen3_moe", num_experts=5)


def test_expert_parallel_all_to_all_transport():
    # the all_to_all_single transport (NCCL on GPUs) runs on gloo ranks too
    _check("qwen2_moe", num_experts=5, transport="all_to_all")


def _partition_worker(rank, port, out):
    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        from accerl_agent_b200.parallel.expert_parallel import expert_partition
        from accerl_agent_b200.parallel.fsdp import ShardedAdamW

        cfg = _cfg("qwen2_moe", 5)  # uneven: rank 0 owns 3 experts, rank 1 owns 2
        pcfg = expert_partition(cfg, rank, 2)
        model = build_model(pcfg, "full", torch.device("cpu"), torch.float32, pad_to=2, experts_last=True)
        model.init_weights(seed=3)
        model.expert_parallel = ExpertParallel(cfg, max_tokens=64, device=torch.device("cpu"), dtype=torch.float32,
                                               transport="emulated")
        opt = ShardedAdamW(model, lr=1e-3)
        lp = _run(model, _pack(40 + rank, cfg.vocab_size))
        names = [n for n in model.layout.order if n.endswith("experts.gate_up_proj")]
        local_grads = {n: model.g(n).clone() for n in names}
        opt.step(1e-3)
        after = {n: model.w(n).clone() for n in model.layout.order}
        # numpy copies travel by value (tensors would be shared with a process that is about to exit)
        out.put((rank, (lp.numpy(), {n: g.numpy() for n, g in local_grads.items()},
                        {n: w.numpy() for n, w in after.items()}, pcfg.expert_offset, pcfg.local_experts,
                        model.layout.replicated_numel, model.layout.trainable_numel), None))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        out.put((rank, repr(exc), None))
        raise


def test_expert_partitioned_storage_matches_full_model():
    """Each rank holding only its experts (weights, gradients, optimizer state) computes the same
    log-probabilities, expert gradients and post-step parameters as one rank holding every expert and
    training on both ranks' packs; the optimizer shards only the replicated prefix."""
    from accerl_agent_b200.parallel.fsdp import ShardedAdamW

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_partition_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, payload, _ = q.get(timeout=180)
        assert not isinstance(payload, str), payload
        res[r] = payload
    for p in procs:
        p.join(60)
    cfg = _cfg("qwen2_moe", 5)
    ref = build_model(cfg, "full", torch.device("cpu"), torch.float32)
    ref.init_weights(seed=3)
    opt = ShardedAdamW(ref, lr=1e-3)
    lps = [_run(ref, _pack(40 + r, cfg.vocab_size)) for r in range(2)]
    ref_grads = {n: ref.g(n).clone() for n in ref.layout.order if n.endswith("experts.gate_up_proj")}
    opt.step(1e-3)
    for r in range(2):
        lp, local_grads, after, lo, nloc, repl, trainable = res[r]
        assert repl < trainable  # a rank-local expert region exists
        assert torch.allclose(torch.from_numpy(lp), lps[r], atol=1e-5, rtol=1e-4)
        for n, g in local_grads.items():
            assert torch.allclose(torch.from_numpy(g), ref_grads[n][lo : lo + nloc], atol=1e-6, rtol=1e-4), n
        for n, w in after.items():
            want = ref.w(n)
            if n.endswith("experts.gate_up_proj") or n.endswith("experts.down_proj"):
                want = want[lo : lo + nloc]
            assert torch.allclose(torch.from_numpy(w), want, atol=1e-6, rtol=1e-5), n


def _plan_reference(C, nloc, lo_of, me, seg):
    """Loop form of the expert-parallel plan arithmetic (owner layout, source bases, owner blocks)."""
    W, E = len(C), len(C[0])
    seg_rows = [[sum(C[s][lo_of[d] + el] for s in range(W)) for el in range(nloc[d])] for d in range(W)]
    seg_pad = [[(r + seg - 1) // seg * seg for r in rows] for rows in seg_rows]
    seg_start = []
    for d in range(W):
        st, acc = [], 0
        for p in seg_pad[d]:
            st.append(acc)
            acc += p
        seg_start.append(st)
    owner = [d for d in range(W) for _ in range(nloc[d])]
    base = [seg_start[owner[e]][e - lo_of[owner[e]]] + sum(C[s][e] for s in range(me)) for e in range(E)]
    blocks = ([], [], [], [])
    for el in range(nloc[me]):
        e = lo_of[me] + el
        r = seg_start[me][el]
        for s in range(W):
            n = C[s][e]
            if n:
                for lst, v in zip(blocks, (r, n, s, sum(C[s][:e]))):
                    lst.append(v)
            r += n
    return base, blocks, seg_pad[me]


def test_vectorised_plan_matches_the_loop_form(monkeypatch):
    """The vectorised plan gives the loop form's destination rows, owner blocks and padded layout for
    uneven expert partitions and empty experts."""
    import random

    import torch.distributed as dist

    from accerl_agent_b200.parallel.expert_parallel import SEG, ExpertParallel, expert_ranges

    rnd = random.Random(1)
    for W, E in ((2, 6), (8, 60), (3, 10), (4, 128)):
        C = [[rnd.choice([0, 0, rnd.randint(1, 300)]) for _ in range(E)] for _ in range(W)]
        monkeypatch.setattr(dist, "all_gather",
                            lambda lst, t, group=None: [x.copy_(torch.tensor([C[i]])) for i, x in enumerate(lst)])
        for me in range(W):
            ep = ExpertParallel.__new__(ExpertParallel)
            ep.world, ep.rank, ep.E, ep.k, ep.group = W, me, E, 4, None
            ep.nloc, ep.lo_of = expert_ranges(E, W)
            ep.E_loc, ep.lo = ep.nloc[me], ep.lo_of[me]
            ep.device, ep.transport, ep.p2p = torch.device("cpu"), "emulated", False
            plan = ep.plan(torch.tensor(C[me]))
            base, blocks, pads = _plan_reference(C, ep.nloc, ep.lo_of, me, SEG)
            assert plan["base"] == base
            assert tuple(plan["blocks"]) == blocks
            assert plan["lay"]["rows"].tolist() == pads and plan["n_send"] == sum(C[me])
