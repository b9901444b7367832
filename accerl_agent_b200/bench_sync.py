"""Trainer -> rollout weight-sync benchmark on one node.

    python -m accerl_agent_b200.bench_sync [--model qwen3-8b] [--trainers 1] [--tp 1] [--iters 5]

``--trainers T`` processes play trainer ranks on GPUs 0..T-1, each holding the full bf16 compute copy
in the trainer's flat layout (the resident-parameter design); ``--tp P`` processes on GPUs T..T+P-1
play one tensor-parallel rollout engine. Two transfer paths are timed with CUDA events, max over the
receiving ranks:

* ``kernel_pull``: every engine rank maps trainer ``r % T``'s buffer once (CUDA IPC, opened on the
  engine's GPU) and runs its copy plan: one kernel that reads exactly its TP shard of every parameter
  over NVLink and writes it into the engine's fused layout in place (no gather, no rank-0 funnel);
* ``nccl_broadcast``: the reference's transfer (trainer rank 0 broadcasts the whole model packed into
  1 GiB buffers, double-buffered; every engine rank receives all of it and would slice afterwards).

The weight-sync configuration of Qwen3-8B is ``--trainers 6 --tp 2`` on 8 GPUs.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _time(fn, warmup: int, iters: int, sync_group=None):
    ts = []
    for i in range(warmup + iters):
        torch.cuda.synchronize()
        if sync_group is not None:
            dist.barrier(group=sync_group)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        if i >= warmup:
            ts.append(s.elapsed_time(e))
    return sorted(ts)[len(ts) // 2]


def _proc(rank: int, world: int, a, port: int, q):
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    from .models.config import get_preset
    from .models.transformer import ParamLayout
    from .ops._ext import native
    from .rollout.weight_map import build_weight_map, descs_tensor, map_bytes, tp_shard_config
    from . import ops

    T, P = a.trainers, a.tp
    cfg = get_preset(a.model)
    src_layout = ParamLayout.build(cfg, "full", pad_to=T)
    is_trainer = rank < T
    results = {}
    if is_trainer:
        buf = torch.empty(src_layout.total_numel, dtype=torch.bfloat16, device=dev)
        gen = torch.Generator(device=dev).manual_seed(0)
        buf.normal_(generator=gen)
        rc, handle, off = native().ipc_export(buf)
        assert rc == 0
        info = (rank, handle, off)
    else:
        info = None
    infos = [None] * world
    dist.all_gather_object(infos, info)
    engine_ranks = list(range(T, T + P))
    engine_group = dist.new_group(engine_ranks)
    bcast_group = dist.new_group([0] + engine_ranks)
    # ---- kernel pull of this rank's shard
    if not is_trainer:
        r = rank - T
        scfg = tp_shard_config(cfg, P)
        if scfg.local_experts:
            scfg.expert_offset = r * scfg.local_experts
        dst_layout = ParamLayout.build(scfg, "full")
        dst = torch.empty(dst_layout.total_numel, dtype=torch.bfloat16, device=dev)
        tr, handle, off = infos[r % T]
        native().enable_peer_access(tr)
        rc, base = native().ipc_open(handle)
        assert rc == 0
        descs = build_weight_map(cfg, src_layout, dst_layout, r, P, "all")
        plan = descs_tensor(descs, dev)
        ms = _time(lambda: ops.weight_pull(plan, base + off, dst), a.warmup, a.iters, engine_group)
        results["kernel_pull_ms"] = ms
        results["kernel_pull_bytes"] = map_bytes(descs)
        # spot check against a host copy of one parameter slice
        name = "model.layers.0.self_attn.o_proj.weight"
        s_slot, d_slot = src_layout.slots[name], dst_layout.slots[name]
        ql = cfg.q_dim // P
        got = dst[d_slot.offset : d_slot.offset + d_slot.numel].view(cfg.hidden_size, ql)
        rc, raw = native().peer_read(base + off + 2 * s_slot.offset, 2 * s_slot.numel)
        assert rc == 0
        full = torch.frombuffer(bytearray(raw), dtype=torch.bfloat16).view(cfg.hidden_size, cfg.q_dim)
        assert torch.equal(got.cpu(), full[:, r * ql : (r + 1) * ql]), "pulled shard differs from the trainer's"
    dist.barrier()
    # ---- NCCL broadcast of the packed full model from trainer 0 to every engine rank
    if rank == 0 or not is_trainer:
        n = src_layout.total_numel
        payload = buf if rank == 0 else torch.empty(n, dtype=torch.bfloat16, device=dev)
        bucket = (1 << 30) // 2

        def bcast():
            for o in range(0, n, bucket):
                dist.broadcast(payload[o : o + bucket], src=0, group=bcast_group)

        results["nccl_broadcast_ms"] = _time(bcast, a.warmup, a.iters, bcast_group)
    dist.barrier()
    gathered = [None] * world
    dist.all_gather_object(gathered, results)
    if rank == T:
        pulls = [g["kernel_pull_ms"] for g in gathered if "kernel_pull_ms" in g]
        bytes_max = max(g["kernel_pull_bytes"] for g in gathered if "kernel_pull_bytes" in g)
        bc = max(g["nccl_broadcast_ms"] for g in gathered if "nccl_broadcast_ms" in g)
        full_bytes = src_layout.total_numel * 2
        q.put({
            "metric": "weight-sync ms",
            "model": a.model,
            "trainers": T,
            "engine_tp": P,
            "model_bytes": full_bytes,
            "kernel_pull_ms": round(max(pulls), 3),
            "kernel_pull_bytes_per_engine_rank": bytes_max,
            "kernel_pull_gbs_per_rank": round(bytes_max / 1e9 / (max(pulls) / 1e3), 1),
            "nccl_broadcast_ms": round(bc, 3),
            "speedup_vs_broadcast": round(bc / max(pulls), 2),
            "link_roofline_ms_at_770GBs": round(bytes_max / 770e9 * 1e3, 3),
            "frac_of_link_roofline": round(bytes_max / 770e9 * 1e3 / max(pulls), 3),
        })
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--trainers", type=int, default=1)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    import socket

    world = a.trainers + a.tp
    if torch.cuda.device_count() < world:
        raise SystemExit(f"needs {world} GPUs, found {torch.cuda.device_count()}")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_proc, args=(r, world, a, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join()
    out = q.get(timeout=5)
    print(json.dumps(out))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
