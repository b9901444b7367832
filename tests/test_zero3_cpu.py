"""Layer-sharded parameters (``--shard-params``, parallel/zero3.py) on CPU ranks (gloo): the trainer's
optimisation equals the replicated-parameter trainer's, the checkpoint it writes loads into either
kind of trainer, and the engine's copy plans assemble the same weights from the per-rank shards."""

import os
import random
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from accerl_agent_b200.core.sample import RLSample


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full_params(w):
    """name -> fp32 copy of every parameter, from either kind of trainer (a collective when sharded)."""
    out = {}
    if w.sharding is None:
        for n, v in w.model.named_parameters():
            out[n] = v.detach().float().clone()
        return out

    def take(u, views):
        for n in u.names:
            out[n] = views[n].detach().float().clone()

    w.sharding.for_each_unit_gathered(take)
    return out


def _worker(rank, port, model_path, sharded, ckpt, out, checkpointing=False, world=2, train_mode="full"):
    from accerl_agent_b200.core.config import make_args
    from accerl_agent_b200.replay import ReplayBuffer
    from accerl_agent_b200.trainer.worker import TrainWorker

    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        args = make_args(model_path=model_path, train_packing="varlen", train_token_budget=64, max_length=64,
                         tw_history_token_window=64, batch_size=1, grad_accum_steps=2, device="cpu",
                         shard_params=sharded, min_replay_size_per_rank=1, replay_sample_timeout_seconds=5.0,
                         replay_wait_sleep_seconds=0.05, dtype="float32", learning_rate=1e-3, lr_warmup_steps=0,
                         gradient_checkpointing=checkpointing, train_mode=train_mode)
        rb = ReplayBuffer(8, seed=rank)
        g = torch.Generator().manual_seed(5 + rank)
        for i in range(2):
            L = 24 + 8 * i
            ids = torch.randint(3, 4096, (L,), generator=g).tolist()
            rb.add_samples([RLSample("grpo", ids, [1] * L, [-100] * 12 + ids[12:], [-6.0] * L, 0.5 - rank + 0.3 * i,
                                     [0.0] * L, [-1] * 12 + [0] * (L - 12), [0])])
        w = TrainWorker(args, rank=rank, fsdp_world_size=world, replay_buffer=rb, device=torch.device("cpu"))
        n_local = int(w.flat_weights("all").numel())
        w.train_until_next_sync(2)
        params = _full_params(w)
        if ckpt:
            w.save_checkpoint(ckpt, "step2")
        # numpy arrays travel by value (tensors would be shared through files of the exiting process)
        out.put((rank, (n_local, w.optimizer_step, {n: v.numpy() for n, v in params.items()})))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        out.put((rank, repr(exc)))
        raise


def _run(model_path, sharded, ckpt=None, checkpointing=False, world=2, train_mode="full"):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, model_path, sharded, ckpt, q, checkpointing, world,
                                                 train_mode))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, payload = q.get(timeout=300)
        assert not isinstance(payload, str), payload
        n_local, steps, params = payload
        res[r] = (n_local, steps, {n: torch.from_numpy(v) for n, v in params.items()})
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("model_path", ["tiny-qwen2", "tiny-qwen2-moe"])
def test_layer_sharded_trainer_matches_replicated(model_path, tmp_path):
    """Two optimizer steps (two packs per window) with sharded parameters give the same weights as
    with replicated parameters, while each rank stores about half of them; the sharded run's
    checkpoint loads into a replicated model with the same values."""
    ck = str(tmp_path)
    sh = _run(model_path, True, ck)
    rep = _run(model_path, False)
    for r in range(2):
        n_sh, steps_sh, p_sh = sh[r]
        n_rep, steps_rep, p_rep = rep[r]
        assert steps_sh == steps_rep == 2
        assert n_sh < 0.6 * n_rep
        assert p_sh.keys() == p_rep.keys()
        for n in p_rep:
            assert torch.allclose(p_sh[n], p_rep[n], atol=2e-5, rtol=1e-4), n
        # every rank sees the same full weights
        assert all(torch.equal(sh[0][2][n], sh[1][2][n]) for n in p_sh)
    from accerl_agent_b200.models.config import resolve_model_config
    from accerl_agent_b200.models.hf_io import load_hf_checkpoint
    from accerl_agent_b200.models.transformer import build_model

    m = build_model(resolve_model_config(model_path), "full", torch.device("cpu"), torch.float32)
    load_hf_checkpoint(m, os.path.join(ck, "step2"))
    for n, v in m.named_parameters():
        assert torch.equal(v, sh[0][2][n]), n
    # and back into sharded storage (one rank here): the same values unit by unit
    from accerl_agent_b200.models.hf_io import load_hf_checkpoint_sharded
    from accerl_agent_b200.parallel.zero3 import LayerShardedParams

    sp = LayerShardedParams(resolve_model_config(model_path), torch.device("cpu"), torch.float32)
    load_hf_checkpoint_sharded(sp, os.path.join(ck, "step2"))
    back = {}
    sp.for_each_unit_gathered(lambda u, views: back.update({n: views[n].clone() for n in u.names}))
    for n, v in back.items():
        assert torch.equal(v, sh[0][2][n]), n


def test_layer_sharded_tied_embeddings_with_recomputation(tmp_path):
    """Tied embeddings (the head unit holds only the final norm; the embedding unit serves both ends)
    with gradient checkpointing (each layer's forward is recomputed inside its backward, while the
    layer is gathered): the same weights as replicated parameters."""
    from accerl_agent_b200.models.config import get_preset

    cfg = get_preset("tiny-qwen2")
    cfg.tie_word_embeddings = True
    path = str(tmp_path / "tied")
    cfg.save(path)
    sh = _run(path, True, checkpointing=True)
    rep = _run(path, False, checkpointing=True)
    assert "lm_head.weight" not in rep[0][2]
    for n, w in rep[0][2].items():
        assert torch.allclose(sh[0][2][n], w, atol=2e-5, rtol=1e-4), n


def test_layer_sharded_three_ranks():
    """An odd number of ranks (units padded to a multiple of 3 x 64 elements, a third per rank)."""
    sh = _run("tiny-qwen2", True, world=3)
    rep = _run("tiny-qwen2", False, world=3)
    assert sh[0][0] < 0.4 * rep[0][0]
    for n, w in rep[2][2].items():
        assert torch.allclose(sh[2][2][n], w, atol=2e-5, rtol=1e-4), n


@pytest.mark.parametrize("train_mode", ["last_layer", "lm_head"])
def test_layer_sharded_partial_train_modes(train_mode):
    """Frozen units are gathered but get no gradient or optimizer state: the trained parameters move
    exactly as with replicated parameters and the frozen ones keep their initial values."""
    sh = _run("tiny-qwen2", True, train_mode=train_mode)
    rep = _run("tiny-qwen2", False, train_mode=train_mode)
    for n, w in rep[0][2].items():
        assert torch.allclose(sh[0][2][n], w, atol=2e-5, rtol=1e-4), n
    from accerl_agent_b200.models.config import get_preset
    from accerl_agent_b200.models.transformer import build_model

    init = build_model(get_preset("tiny-qwen2"), "full", torch.device("cpu"), torch.float32)
    init.init_weights(seed=42)
    moved = [n for n, v in init.named_parameters() if not torch.equal(v, sh[0][2][n])]
    assert moved and all(("lm_head" in n) or (train_mode == "last_layer" and "layers.1." in n) for n in moved)


def test_shard_copy_plans_assemble_the_engine_weights():
    """The engine's plans against three trainers' shard buffers write exactly what the plan against
    one full buffer writes, for every tensor-parallel rank."""
    from accerl_agent_b200.models.config import get_preset
    from accerl_agent_b200.models.transformer import ParamLayout
    from accerl_agent_b200.parallel.zero3 import build_units, shard_pieces
    from accerl_agent_b200.rollout.weight_map import (apply_map_torch, build_weight_map, build_weight_map_sharded,
                                                      tp_shard_config)

    cfg = get_preset("tiny-qwen2-moe")
    world = 3
    full = ParamLayout.build(cfg, "full", pad_to=1)
    units = build_units(full, world)
    src = torch.randn(full.total_numel)
    local = [torch.full((sum(u.shard for u in units),), float("nan")) for _ in range(world)]
    for u in units:
        padded = torch.zeros(u.numel)
        padded[: u.span] = src[u.lo : u.lo + u.span]
        for r in range(world):
            local[r][u.base : u.base + u.shard] = padded[r * u.shard : (r + 1) * u.shard]
    pieces = shard_pieces(units, world)
    for tp in (1, 2):
        for tr in range(tp):
            dst_layout = ParamLayout.build(tp_shard_config(cfg, tp), "full")
            want = torch.zeros(dst_layout.total_numel)
            apply_map_torch(src, want, build_weight_map(cfg, full, dst_layout, tr, tp, "all"))
            got = torch.zeros(dst_layout.total_numel)
            for r, plan in enumerate(build_weight_map_sharded(cfg, full, pieces, world, dst_layout, tr, tp, "all")):
                apply_map_torch(local[r], got, plan)
            assert torch.equal(got, want), (tp, tr)


def test_split_by_pieces_random_copies():
    from accerl_agent_b200.rollout.weight_map import CopyDesc, apply_map_torch, split_by_pieces

    rnd = random.Random(0)
    for _ in range(200):
        N = rnd.randint(50, 400)
        src = torch.arange(N, dtype=torch.float32)
        bounds = [0] + sorted(rnd.sample(range(1, N), rnd.randint(0, 6))) + [N]
        bufs = [torch.full((N,), -1.0) for _ in range(3)]
        fill = [0, 0, 0]
        pieces = []
        for a, b in zip(bounds[:-1], bounds[1:]):
            r = rnd.randrange(3)
            bufs[r][fill[r] : fill[r] + b - a] = src[a:b]
            pieces.append((a, b, r, fill[r]))
            fill[r] += b - a
        C = rnd.randint(1, 20)
        ld = C + rnd.randint(0, 10)
        R = rnd.randint(1, 8)
        if (R - 1) * ld + C > N:
            continue
        d = CopyDesc(rnd.randint(0, N - ((R - 1) * ld + C)), ld, rnd.randint(0, 30), C + rnd.randint(0, 3), R, C)
        want = torch.full((N + 300,), -2.0)
        got = want.clone()
        apply_map_torch(src, want, [d])
        for r, pl in enumerate(split_by_pieces([d], pieces, 3)):
            apply_map_torch(bufs[r], got, pl)
        assert torch.equal(want, got)


@pytest.mark.parametrize("train_mode,tied", [("full", False), ("lm_head", False), ("last_layer", False),
                                             ("lm_head", True)])
def test_units_cover_the_layout_and_split_by_trainability(train_mode, tied):
    """Units tile the parameter layout without gaps, every unit is trained whole or frozen whole, a
    decoder layer is one unit, and the trainable units' shards come first in local storage."""
    from accerl_agent_b200.models.config import get_preset
    from accerl_agent_b200.parallel.zero3 import build_units, sharded_layout

    cfg = get_preset("tiny-qwen2")
    cfg.tie_word_embeddings = tied
    layout = sharded_layout(cfg, train_mode)
    flags = {n: s.trainable for n, s in layout.slots.items()}
    units = build_units(layout, 3, flags)
    ordered = sorted(units, key=lambda u: u.lo)
    assert ordered[0].lo == 0
    for a, b in zip(ordered, ordered[1:]):
        assert a.lo + a.span == b.lo
    assert [n for u in ordered for n in u.names] == list(layout.order)
    for u in units:
        assert {flags[n] for n in u.names} == {u.trainable}
        assert u.numel % (3 * 64) == 0 and u.shard * 3 == u.numel
    layers = [u.layer for u in units if u.layer >= 0]
    assert sorted(layers) == list(range(cfg.num_hidden_layers))
    n_train = sum(u.shard for u in units if u.trainable)
    assert all(u.base < n_train for u in units if u.trainable) and all(u.base >= n_train for u in units
                                                                       if not u.trainable)
    if train_mode == "lm_head":
        trained = {n for u in units if u.trainable for n in u.names}
        assert trained == ({"model.embed_tokens.weight"} if tied else {"lm_head.weight"})
