"""Distributed behaviour on CPU ranks (gloo): the local SFT smoke run with world size 2, sharded
optimizer steps that equal the single-rank step on the union of the packs (global valid-token
normalisation), and the all-reduce(MIN) failure propagation of varlen window preparation."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from accerl_agent_b200.algo.objectives import ObjectiveConfig
from accerl_agent_b200.algo.packing import make_varlen_batch
from accerl_agent_b200.core.sample import RLSample
from accerl_agent_b200.models.config import get_preset
from accerl_agent_b200.models.transformer import build_model
from accerl_agent_b200.parallel.fsdp import ShardedAdamW
from accerl_agent_b200 import ops


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pack(seed):
    g = torch.Generator().manual_seed(seed)
    out = []
    for L in (20, 13):
        ids = torch.randint(0, 4096, (L,), generator=g).tolist()
        labels = [-100] * (L - 5) + ids[L - 5:]
        out.append(RLSample("grpo", ids, [1] * L, labels, [-8.0] * L, 0.7 if seed % 2 else -0.4, [0.0] * L,
                            [-1] * (L - 5) + [0] * 5, [0]))
    return make_varlen_batch(out)


def _step(model, opt, packs, global_tokens):
    cfg = ObjectiveConfig()
    for b in packs:
        lp, ctx = model.forward_logprobs(b, 20)
        tgt = b["target_indices"]
        adv = b["sample_advantages"][b["sequence_ids"][tgt]]
        dlp, _ = ops.policy_loss(lp, b["old_logprobs"][tgt], adv, cfg, loss_scale=1.0 / global_tokens)
        model.backward_from_logprobs(dlp, ctx)
    opt.step(1e-3)


def _sharded_worker(rank, port, out):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    cfg = get_preset("tiny-qwen2")
    model = build_model(cfg, "full", torch.device("cpu"), torch.float32, pad_to=2)
    model.init_weights(seed=1)
    opt = ShardedAdamW(model, lr=1e-3)
    packs = [_pack(10 + rank)]
    total = sum(int(p["target_indices"].numel()) for p in (_pack(10), _pack(11)))
    _step(model, opt, packs, total)
    if rank == 0:
        out.put(model.params.clone())
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_step_equals_single_rank_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    sharded = q.get(timeout=120)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    cfg = get_preset("tiny-qwen2")
    model = build_model(cfg, "full", torch.device("cpu"), torch.float32, pad_to=2)
    model.init_weights(seed=1)
    opt = ShardedAdamW(model, lr=1e-3)
    packs = [_pack(10), _pack(11)]
    total = sum(int(p["target_indices"].numel()) for p in packs)
    _step(model, opt, packs, total)
    assert torch.allclose(sharded, model.params, atol=1e-6, rtol=1e-5)


def test_local_trainer_fsdp_world2_cpu():
    from accerl_agent_b200.local_trainer import main

    res = main(["--model-path", "tiny-qwen2", "--device", "cpu", "--use-fsdp", "--fsdp-world-size", "2",
                "--batch-size", "1", "--max-length", "128", "--response-length", "32", "--learning-rate", "1e-5",
                "--max-steps", "5", "--grad-accum-steps", "1", "--train-mode", "full", "--dataset", "random",
                "--dtype", "float32"])
    assert sorted(res) == [0, 1]
    for r in res.values():
        assert r["steps"] == 5 and torch.isfinite(torch.tensor(r["last_loss"]))


def _fail_worker(rank, port, out):
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    args = make_args(model_path="tiny-qwen2", train_packing="varlen", train_token_budget=64, max_length=64,
                     tw_history_token_window=64, batch_size=1, grad_accum_steps=1, device="cpu",
                     min_replay_size_per_rank=1, replay_sample_timeout_seconds=0.5, replay_wait_sleep_seconds=0.05)
    rb = ReplayBuffer(8)
    if rank == 0:  # rank 1 never receives samples and times out preparing its window
        rb.add_samples([RLSample("grpo", list(range(10)), [1] * 10, [-100] * 5 + list(range(5, 10)), [-1.0] * 10,
                                 1.0, [0.0] * 10, [-1] * 5 + [0] * 5, [0])])
    w = TrainWorker(args, rank=rank, fsdp_world_size=2, replay_buffer=rb, device=torch.device("cpu"))
    try:
        w.train_until_next_sync(1)
        out.put((rank, "ok"))
    except Exception as exc:
        out.put((rank, type(exc).__name__ + ": " + str(exc)[:80]))
    dist.destroy_process_group()


def test_window_preparation_failure_fails_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_fail_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(60)
    assert all("At least one FSDP rank failed" in v for v in res.values()), res


def _drop_worker(rank, port, out):
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker

    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    os.environ["ACCERL_PG_TIMEOUT"] = "10"
    args = make_args(model_path="tiny-qwen2", train_packing="varlen", train_token_budget=64, max_length=64,
                     tw_history_token_window=64, batch_size=1, grad_accum_steps=1, device="cpu",
                     min_replay_size_per_rank=1, replay_sample_timeout_seconds=5.0, replay_wait_sleep_seconds=0.01)
    rb = ReplayBuffer(8)
    rb.add_samples([RLSample("grpo", list(range(10)), [1] * 10, [-100] * 5 + list(range(5, 10)), [-1.0] * 10,
                             1.0, [0.0] * 10, [-1] * 5 + [0] * 5, [0])])
    w = TrainWorker(args, rank=rank, fsdp_world_size=2, fsdp_master_addr="127.0.0.1", fsdp_master_port=port,
                    replay_buffer=rb, device=torch.device("cpu"))
    w.train_until_next_sync(1)
    if rank == 1:  # leaves between steps, with nothing in flight
        out.put((rank, "left"))
        out.close()
        out.join_thread()
        os._exit(0)
    import time

    t0 = time.monotonic()
    try:
        w.train_until_next_sync(1)
        out.put((rank, "no error"))
    except Exception as exc:
        out.put((rank, f"error after {time.monotonic() - t0:.1f}s: {type(exc).__name__}"))
    out.close()
    out.join_thread()
    os._exit(0)


def test_rank_that_leaves_fails_the_next_collective_of_the_others():
    """A trainer rank that exits between optimizer steps makes the next step of the remaining rank
    raise (the lost peer or the short process-group timeout ends its collective) instead of hanging."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_drop_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(60)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res
    assert float(res[0].split()[2].rstrip("s:")) < 60.0, res


def _ep_worker(rank, port, storage, out):
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker

    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        args = make_args(model_path="tiny-qwen2-moe", train_packing="varlen", train_token_budget=64, max_length=64,
                         tw_history_token_window=64, batch_size=1, grad_accum_steps=1, device="cpu",
                         expert_parallel=True, expert_storage=storage, min_replay_size_per_rank=1,
                         replay_sample_timeout_seconds=5.0, replay_wait_sleep_seconds=0.05, dtype="float32")
        rb = ReplayBuffer(8)
        g = torch.Generator().manual_seed(5 + rank)
        ids = torch.randint(3, 4096, (24,), generator=g).tolist()
        rb.add_samples([RLSample("grpo", ids, [1] * 24, [-100] * 12 + ids[12:], [-6.0] * 24, 0.5 - rank,
                                 [0.0] * 24, [-1] * 12 + [0] * 12, [0])])
        w = TrainWorker(args, rank=rank, fsdp_world_size=2, replay_buffer=rb, device=torch.device("cpu"))
        w.train_until_next_sync(1)
        names = [n for n in w.model.layout.order if n.endswith("experts.gate_up_proj")]
        out.put((rank, (w.expert_partitioned, w.model.cfg.local_experts, w.model.cfg.expert_offset,
                        int(w.model.params.numel()), w.optimizer_step,
                        {n: w.model.w(n).detach().numpy().copy() for n in names})))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        out.put((rank, repr(exc)))
        raise


def _run_ep(storage):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ep_worker, args=(r, port, storage, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, payload = q.get(timeout=240)
        assert not isinstance(payload, str), payload
        res[r] = payload
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return res


def test_trainer_expert_partitioned_storage_matches_replicated():
    """A trainer run with ``--expert-parallel`` stores only its 3 of 6 experts per rank by default
    (smaller parameter buffer) and, after one optimizer step, holds exactly the slice of the expert
    weights that the replicated-storage run holds for the same experts."""
    part, repl = _run_ep("partitioned"), _run_ep("replicated")
    for r in range(2):
        is_part, nloc, lo, numel, steps, experts = part[r]
        r_part, r_nloc, _, r_numel, r_steps, r_experts = repl[r]
        assert is_part and not r_part and nloc == 3 and lo == 3 * r and r_nloc is None
        assert numel < r_numel and steps == r_steps == 1
        for n, w in experts.items():
            assert w.shape[0] == 3
            assert torch.allclose(torch.from_numpy(w), torch.from_numpy(r_experts[n][lo:lo + nloc]),
                                  atol=1e-6, rtol=1e-5), n


def _ep_resume_worker(rank, port, ckpt, out):
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker

    def args(**kw):
        return make_args(model_path="tiny-qwen2-moe", train_packing="varlen", train_token_budget=64, max_length=64,
                         tw_history_token_window=64, batch_size=1, grad_accum_steps=1, device="cpu", dtype="float32",
                         expert_parallel=True, min_replay_size_per_rank=1, replay_sample_timeout_seconds=5.0,
                         replay_wait_sleep_seconds=0.01, learning_rate=1e-3, max_steps=10, **kw)

    def buffer():
        rb = ReplayBuffer(8)
        g = torch.Generator().manual_seed(11 + rank)
        ids = torch.randint(3, 4096, (20,), generator=g).tolist()
        rb.add_samples([RLSample("grpo", ids, [1] * 20, [-100] * 10 + ids[10:], [-6.0] * 20, 0.6 - rank,
                                 [0.0] * 20, [-1] * 10 + [0] * 10, [0])])
        return rb

    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        a = TrainWorker(args(save_optimizer_state=True), rank=rank, fsdp_world_size=2, replay_buffer=buffer(),
                        device=torch.device("cpu"))
        a.train_until_next_sync(2)
        a.save_checkpoint(ckpt, "step2")
        a.train_until_next_sync(1)
        b = TrainWorker(args(resume_from=os.path.join(ckpt, "step2")), rank=rank, fsdp_world_size=2,
                        replay_buffer=buffer(), device=torch.device("cpu"))
        resumed_step = b.optimizer_step
        b.train_until_next_sync(1)
        diff = float((a.model.params - b.model.params).abs().max())
        out.put((rank, (a.expert_partitioned, resumed_step, a.optimizer_step, b.optimizer_step, diff,
                        sorted(os.listdir(os.path.join(ckpt, "step2"))))))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        out.put((rank, repr(exc)))
        raise


def test_expert_partitioned_trainer_resumes_the_same_optimisation(tmp_path):
    """Checkpoint and resume with expert-partitioned storage on 2 gloo ranks: each rank writes its own
    experts file and optimizer shard (replicated-prefix shard plus its experts' full state); the
    resumed run's next step equals the uninterrupted run's on every rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ep_resume_worker, args=(r, port, str(tmp_path), q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, payload = q.get(timeout=300)
        assert not isinstance(payload, str), payload
        res[r] = payload
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for r in range(2):
        part, resumed, sa, sb, diff, files = res[r]
        assert part and resumed == 2 and sa == sb == 3
        assert diff < 1e-6, diff
        assert "model-experts-00002-of-00002.safetensors" in files and "optimizer_rank00001.pt" in files


def _balance_worker(rank, port, balance_packs, out):
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker

    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        args = make_args(model_path="tiny-qwen2", train_packing="varlen", train_token_budget=96, max_length=96,
                         tw_history_token_window=96, batch_size=1, grad_accum_steps=4, device="cpu", dtype="float32",
                         min_replay_size_per_rank=4, replay_sample_timeout_seconds=5.0, learning_rate=1e-3,
                         replay_wait_sleep_seconds=0.01, balance_packs=balance_packs, seed=3)
        rb = ReplayBuffer(4, seed=rank)
        g = torch.Generator().manual_seed(100 + rank)
        # rank 0 draws long episodes, rank 1 short ones: the unbalanced window is skewed
        for L in ((90, 80, 85, 70) if rank == 0 else (12, 16, 20, 10)):
            ids = torch.randint(3, 4096, (L,), generator=g).tolist()
            rb.add_samples([RLSample("grpo", ids, [1] * L, [-100] * (L - 6) + ids[L - 6:], [-6.0] * L,
                                     0.5 - rank, [0.0] * L, [-1] * (L - 6) + [0] * 6, [0])])
        w = TrainWorker(args, rank=rank, fsdp_world_size=2, replay_buffer=rb, device=torch.device("cpu"))
        w.model.init_weights(seed=7)
        w.optimizer.refresh_master_from_params()
        summary = w.train_until_next_sync(1)
        out.put((rank, (w.model.params.detach().clone(), dict(w.last_balance), summary["segment_valid_tokens"])))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        out.put((rank, repr(exc)))
        raise


def _run_balance(flag):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_balance_worker, args=(r, port, flag, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, payload = q.get(timeout=240)
        assert not isinstance(payload, str), payload
        res[r] = payload
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return res


def test_pack_balancing_moves_packs_and_keeps_the_step():
    """Spreading the window's packs over the ranks by estimated work moves packs from the rank with
    the long episodes and gives the same optimizer step (parameters, global token count) as computing
    every pack where it was drawn."""
    bal, plain = _run_balance(True), _run_balance(False)
    moved = bal[0][1].get("moved_in", 0) + bal[1][1].get("moved_in", 0)
    assert moved > 0
    assert abs(bal[0][1]["rank_cost"] - bal[1][1]["rank_cost"]) < abs(bal[0][1]["mean_cost"]) * 0.5
    assert plain[0][1] == {} and plain[1][1] == {}
    for r in range(2):
        assert bal[r][2] == plain[r][2]
        torch.testing.assert_close(bal[r][0], plain[r][0], atol=1e-6, rtol=1e-5)
