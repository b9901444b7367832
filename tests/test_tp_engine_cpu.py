"""Tensor-parallel generation engine on CPU ranks (gloo): weight shards pulled through copy plans
from a full flat buffer, the leader scheduling and broadcasting every step, the follower replaying
it, row-parallel all-reduces (and expert parallelism inside the TP group for MoE layers). Greedy
outputs equal those of a single-rank engine on the same weights. Also the copy plans themselves:
shards of every TP rank reassemble the full weights, and plans between different trainer layouts."""

import asyncio
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from accerl_agent_b200.models.config import get_preset
from accerl_agent_b200.models.transformer import ParamLayout, build_model
from accerl_agent_b200.rollout.engine import GenerationEngine
from accerl_agent_b200.rollout.generation import SamplingParams
from accerl_agent_b200.rollout.weight_map import apply_map_torch, build_weight_map, tp_shard_config


def _cfg(kind):
    cfg = get_preset("tiny-qwen2")
    cfg.vocab_size = 512
    if kind == "moe":
        cfg.model_type = "qwen2_moe"
        cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size = 6, 2, 64
        cfg.shared_expert_intermediate_size = 96
    return cfg


def _full_params(cfg):
    m = build_model(cfg, "full", torch.device("cpu"), torch.float32)
    m.init_weights(seed=11, std=0.08)
    return m.params, m.layout


PROMPTS = [[5, 9, 33, 7, 100, 2], [41, 42, 43], list(range(60, 97))]


async def _generate(engine):
    outs = []
    for i, ids in enumerate(PROMPTS):
        sp = SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True)
        last = None
        async for o in engine.generate({"prompt_token_ids": ids}, sp, request_id=f"r{i}"):
            last = o
        outs.append(list(last.outputs[0].token_ids))
    return outs


def _tp_worker(rank, port, kind, q):
    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        dist.init_process_group("gloo", rank=rank, world_size=2)
        cmd = dist.new_group(backend="gloo")
        cfg = _cfg(kind)
        full, layout = _full_params(cfg)
        eng = GenerationEngine(cfg, torch.device("cpu"), torch.float32, max_num_seqs=8, max_num_batched_tokens=64,
                               num_blocks=64, block_size=8, tp_group=dist.group.WORLD, cmd_group=cmd)
        eng.set_weight_source(layout, tensor=full)
        if rank == 0:
            eng.pull_weights("all")
            outs = asyncio.run(_generate(eng))
            asyncio.run(eng.shutdown())
            eng.stop_followers()
            q.put((rank, outs))
        else:
            import threading

            # the follower pulls its shard when the leader's pull command arrives
            eng.serve_follower()
            q.put((rank, None))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        q.put((rank, repr(exc)))
        raise


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_tp2_engine_matches_single_rank(kind):
    cfg = _cfg(kind)
    full, layout = _full_params(cfg)
    ref = GenerationEngine(cfg, torch.device("cpu"), torch.float32, max_num_seqs=8, max_num_batched_tokens=64,
                           num_blocks=64, block_size=8, params=full.clone())
    want = asyncio.run(_generate(ref))
    asyncio.run(ref.shutdown())
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_tp_worker, args=(r, port, kind, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(60)
    assert not isinstance(res[0], str), res[0]
    assert not isinstance(res[1], str), res[1]
    assert res[0] == want


@pytest.mark.parametrize("kind", ["dense", "moe"])
def test_tp_shards_reassemble_full_weights(kind):
    cfg = _cfg(kind)
    full, layout = _full_params(cfg)
    shards = []
    for r in range(2):
        scfg = tp_shard_config(cfg, 2)
        if scfg.local_experts:
            scfg.expert_offset = r * scfg.local_experts
        sl = ParamLayout.build(scfg, "full")
        dst = torch.zeros(sl.total_numel)
        apply_map_torch(full, dst, build_weight_map(cfg, layout, sl, r, 2))
        shards.append((sl, dst))
    H, D, Hq, Hkv = cfg.hidden_size, cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads

    def get(lay, buf, name):
        s = lay.slots[name]
        return buf[s.offset : s.offset + s.numel].view(s.shape)

    p = "model.layers.0."
    qkv = get(layout, full, p + "self_attn.qkv_proj.weight")
    q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D])
    parts = [get(sl, b, p + "self_attn.qkv_proj.weight") for sl, b in shards]
    ql, kl = Hq * D // 2, Hkv * D // 2
    assert torch.equal(torch.cat([x[:ql] for x in parts]), q)
    assert torch.equal(torch.cat([x[ql : ql + kl] for x in parts]), k)
    assert torch.equal(torch.cat([x[ql + kl :] for x in parts]), v)
    o = get(layout, full, p + "self_attn.o_proj.weight")
    assert torch.equal(torch.cat([get(sl, b, p + "self_attn.o_proj.weight") for sl, b in shards], 1), o)
    emb = get(layout, full, "model.embed_tokens.weight")
    assert all(torch.equal(get(sl, b, "model.embed_tokens.weight"), emb) for sl, b in shards)
    if kind == "moe":
        e = get(layout, full, p + "mlp.experts.down_proj")
        assert torch.equal(torch.cat([get(sl, b, p + "mlp.experts.down_proj") for sl, b in shards]), e)
    else:
        gu = get(layout, full, p + "mlp.gate_up_proj.weight")
        I = cfg.intermediate_size
        parts = [get(sl, b, p + "mlp.gate_up_proj.weight") for sl, b in shards]
        assert torch.equal(torch.cat([x[: I // 2] for x in parts]), gu[:I])
        assert torch.equal(torch.cat([x[I // 2 :] for x in parts]), gu[I:])


def test_plans_between_trainer_and_engine_layouts():
    cfg = _cfg("dense")
    m = build_model(cfg, "lm_head", torch.device("cpu"), torch.float32, pad_to=3)
    m.init_weights(seed=2)
    eng_layout = ParamLayout.build(cfg, "full")
    dst = torch.zeros(eng_layout.total_numel)
    apply_map_torch(m.params, dst, build_weight_map(cfg, m.layout, eng_layout))
    for name, s in eng_layout.slots.items():
        t = m.layout.slots[name]
        assert torch.equal(dst[s.offset : s.offset + s.numel], m.params[t.offset : t.offset + t.numel]), name
    # trainable scope: only the LM head (the embedding when tied) moves
    dst2 = torch.zeros(eng_layout.total_numel)
    apply_map_torch(m.params, dst2, build_weight_map(cfg, m.layout, eng_layout, scope="trainable"))
    s = eng_layout.slots["model.embed_tokens.weight" if cfg.tie_word_embeddings else "lm_head.weight"]
    assert torch.equal(dst2[s.offset : s.offset + s.numel], dst[s.offset : s.offset + s.numel])
    assert int((dst2 != 0).sum()) == s.numel


def test_async_loop_with_tp2_engine_cpu(tmp_path):
    """The driver with a 2-rank tensor-parallel engine (leader + follower processes) on CPU ranks."""
    import json

    from accerl_agent_b200.agent_textworld import main

    log = tmp_path / "run"
    main([
        "--model-path", "tiny-qwen2", "--env", "synthetic", "--device", "cpu", "--fsdp-world-size", "1",
        "--infer-size", "1", "--infer-tp-size", "2", "--num-rollout-workers", "2", "--rollout-batch-size", "2",
        "--tw-max-episode-steps", "3", "--tw-history-token-window", "256", "--max-length", "256",
        "--train-packing", "varlen", "--train-token-budget", "512", "--batch-size", "2", "--grad-accum-steps", "1",
        "--max-steps", "2", "--sync-every-optimizer-steps", "1", "--min-replay-size-per-rank", "2",
        "--replay-capacity", "16", "--synthetic-obs-min", "8", "--synthetic-obs-max", "16", "--infer-max-tokens", "4",
        "--log-dir", str(log), "--learning-rate", "1e-4", "--lr-warmup-steps", "0", "--train-mode", "last_layer",
        "--dtype", "bfloat16", "--train-logprob-mode", "response_only_lm_head",
    ])
    recs = [json.loads(l) for l in open(log / "metrics.jsonl")]
    steps = [r for r in recs if "Train/Loss" in r]
    assert [r["step"] for r in steps] == [1, 2]
    # the sharded engine samples from the same weights the trainer scores with
    assert all(abs(r["KL/OldNewK3TokenMean"]) < 1e-2 for r in steps)


def test_weight_map_from_expert_partitioned_trainers():
    """An engine rank (TP 1 or 2) filled from trainers that each hold only their experts gets the same
    weights as from one trainer holding the whole model."""
    import torch

    from accerl_agent_b200.models.config import get_preset
    from accerl_agent_b200.models.transformer import ParamLayout, build_model
    from accerl_agent_b200.parallel.expert_parallel import expert_partition
    from accerl_agent_b200.rollout.weight_map import (apply_map_torch, build_weight_map, build_weight_map_multi,
                                                      tp_shard_config)

    cfg = get_preset("tiny-qwen2")
    cfg.vocab_size, cfg.model_type, cfg.num_experts, cfg.num_experts_per_tok = 512, "qwen2_moe", 6, 2
    cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size = 64, 96
    full = build_model(cfg, "full", torch.device("cpu"), torch.float32, pad_to=3)
    full.init_weights(seed=5)
    trainers = []
    for t in range(3):
        pc = expert_partition(cfg, t, 3)
        m = build_model(pc, "full", torch.device("cpu"), torch.float32, pad_to=3, experts_last=True)
        m.init_weights(seed=5)
        trainers.append((m, pc))
    for tp in (1, 2):
        for r in range(tp):
            scfg = tp_shard_config(cfg, tp)
            if scfg.local_experts:
                scfg.expert_offset = r * scfg.local_experts
            dst_layout = ParamLayout.build(scfg, "full")
            want = torch.zeros(dst_layout.total_numel)
            apply_map_torch(full.params, want, build_weight_map(cfg, full.layout, dst_layout, r, tp, "all"))
            got = torch.zeros(dst_layout.total_numel)
            srcs = [(m.layout, pc.expert_offset, pc.local_experts) for m, pc in trainers]
            plans = build_weight_map_multi(cfg, srcs, dst_layout, r, tp, "all", primary=r % 3)
            for (m, _), plan in zip(trainers, plans):
                apply_map_torch(m.params, got, plan)
            assert torch.equal(got, want), (tp, r)
