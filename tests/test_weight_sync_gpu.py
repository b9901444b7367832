"""Trainer -> rollout weight sync over CUDA IPC into a tensor-parallel (TP=2) engine, validated the way
the reference validates its NCCL transfer (accerl_agent/vllm_nccl.py:484-578: after the sync, greedy
outputs must equal those of a fresh engine loaded with the same weights).

Three processes on 2 GPUs: a trainer that owns a flat bf16 parameter buffer on GPU 0 and exports it
once, and the two ranks of one TP=2 engine (GPUs 0 and 1) that map it and pull their shards with the
copy-plan kernel. Checked twice -- after the initial full sync and after the trainer changed its
weights and the engine (paused, requests suspended) pulled again:
  * every engine rank's parameter buffer equals its shard of the trainer's weights, bit for bit;
  * greedy tokens equal those of a fresh TP=2 engine loaded from a local copy of the same weights,
    and their log-probabilities agree.
"""

import asyncio
import os
import socket
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

PROMPTS = [[5, 9, 33, 7, 100, 2], [41, 42, 43], list(range(60, 160))]


def _cfg():
    from accerl_agent_b200.models.config import ModelConfig

    return ModelConfig(vocab_size=2048, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                       num_key_value_heads=2, head_dim=128, intermediate_size=512, tie_word_embeddings=False)


def _update(params: torch.Tensor) -> None:
    """The trainer's 'optimizer step': a seeded change of every weight (same bits on every process)."""
    g = torch.Generator().manual_seed(11)
    delta = torch.randn(params.numel(), generator=g) * 0.01
    params.add_(delta.to(params.device, params.dtype))


async def _generate(engine, n=12):
    from accerl_agent_b200.rollout.generation import SamplingParams

    outs = []
    for i, ids in enumerate(PROMPTS):
        sp = SamplingParams(temperature=0.0, max_tokens=n, ignore_eos=True, logprobs=1)
        last = None
        async for o in engine.generate({"prompt_token_ids": ids}, sp, request_id=f"q{i}"):
            last = o
        outs.append((list(last.outputs[0].token_ids), [list(d.values())[0] for d in last.outputs[0].logprobs]))
    return outs


def _trainer(q_handle, q_cmd, q_ack):
    from accerl_agent_b200.models.transformer import build_model
    from accerl_agent_b200.ops._ext import native

    torch.cuda.set_device(0)
    m = build_model(_cfg(), "full", torch.device("cuda", 0), torch.bfloat16)
    m.init_weights(seed=7, std=0.05)
    torch.cuda.synchronize()
    rc, handle, offset = native().ipc_export(m.params)
    assert rc == 0
    probe = bytes(m.params[:8].view(torch.uint8).cpu().numpy().tobytes())
    h = {"kind": "cuda-ipc", "handle": bytes(handle), "offset": int(offset), "numel": m.params.numel(),
         "device": 0, "probe": probe}
    q_handle.put(h)
    q_handle.put(h)
    while True:
        cmd = q_cmd.get(timeout=600)
        if cmd == "update":
            _update(m.params)
            torch.cuda.synchronize()
            q_ack.put("updated")
        else:
            break


def _engine_rank(rank, port, q_handle, q_cmd, q_ack, q_out):
    try:
        from accerl_agent_b200.models.transformer import build_model
        from accerl_agent_b200.rollout.engine import GenerationEngine
        from accerl_agent_b200.rollout.inference import attach_weight_source
        from accerl_agent_b200.rollout.weight_map import apply_map_torch, build_weight_map

        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
        cmd = dist.new_group(backend="gloo")
        cfg = _cfg()
        local = build_model(cfg, "full", dev, torch.bfloat16)  # this rank's own copy of the trainer's weights
        local.init_weights(seed=7, std=0.05)

        def engine():
            return GenerationEngine(cfg, dev, torch.bfloat16, max_num_seqs=8, max_num_batched_tokens=256,
                                    num_blocks=128, tp_group=dist.group.WORLD, cmd_group=cmd)

        def expected_shard(eng):
            descs = build_weight_map(cfg, local.layout, eng.layout, rank, 2, "all")
            want = torch.zeros_like(eng.model.params)
            apply_map_torch(local.params, want, descs)
            return want

        handle = q_handle.get(timeout=300)
        eng = engine()
        attach_weight_source(eng, SimpleNamespace(train_mode="full", fsdp_world_size=1), dev, handle, [])
        synced = {}
        if rank == 0:
            eng.pull_weights("all")  # every rank pulls its shard over the IPC mapping
            synced["ipc0"] = asyncio.run(_generate(eng))
            q_cmd.put("update")
            assert q_ack.get(timeout=120) == "updated"
            asyncio.run(eng.pause_generation(mode="suspend", clear_cache=True))
            eng.pull_weights("all")
            asyncio.run(eng.resume_generation(version=1))
            synced["ipc1"] = asyncio.run(_generate(eng))
            asyncio.run(eng.shutdown())
            eng.stop_followers()
        else:
            eng.serve_follower()
        torch.cuda.synchronize()
        _update(local.params)  # this rank's copy now holds the trainer's updated weights
        params_equal = bool(torch.equal(eng.model.params, expected_shard(eng)))
        # a fresh TP=2 engine loaded from the local copy of the updated weights
        ref = engine()
        ref.set_weight_source(local.layout, addr=local.params.data_ptr())
        if rank == 0:
            ref.pull_weights("all")
            fresh = asyncio.run(_generate(ref))
            asyncio.run(ref.shutdown())
            ref.stop_followers()
            q_out.put((rank, (params_equal, synced, fresh)))
        else:
            ref.serve_follower()
            q_out.put((rank, (params_equal, None, None)))
        dist.barrier()
        dist.destroy_process_group()
        if rank == 0:
            q_cmd.put("stop")
    except BaseException as exc:
        q_out.put((rank, repr(exc)))
        raise


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ipc_sync_into_tp2_engine_matches_fresh_engine():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q_handle, q_cmd, q_ack, q_out = ctx.Queue(), ctx.Queue(), ctx.Queue(), ctx.Queue()
    trainer = ctx.Process(target=_trainer, args=(q_handle, q_cmd, q_ack))
    trainer.start()
    ranks = [ctx.Process(target=_engine_rank, args=(r, port, q_handle, q_cmd, q_ack, q_out)) for r in range(2)]
    for p in ranks:
        p.start()
    try:
        res = dict(q_out.get(timeout=600) for _ in range(2))
    finally:
        q_cmd.put("stop")
        for p in ranks + [trainer]:
            p.join(60)
            if p.is_alive():
                p.kill()
    assert not isinstance(res[0], str), res[0]
    assert not isinstance(res[1], str), res[1]
    assert res[0][0] and res[1][0], "engine parameters differ from the trainer's updated weights"
    _, synced, fresh = res[0]
    for (tok, lp), (tok_w, lp_w) in zip(synced["ipc1"], fresh):
        assert tok == tok_w
        assert max(abs(a - b) for a, b in zip(lp, lp_w)) < 1e-3
    # the update changed the engine's log-probabilities, so the second sync was not a no-op
    lp0 = [v for _, lps in synced["ipc0"] for v in lps]
    lp1 = [v for _, lps in synced["ipc1"] for v in lps]
    assert max(abs(a - b) for a, b in zip(lp0, lp1)) > 1e-3
