"""Trainer -> rollout weight-sync benchmark on one node.

    python -m accerl_agent_b200.bench_sync [--model qwen3-8b] [--trainers 1] [--tp 1] [--iters 5]

``--trainers T`` processes play trainer ranks on GPUs 0..T-1, each holding the full bf16 compute copy
in the trainer's flat layout (the resident-parameter design); ``--tp P`` processes on GPUs T..T+P-1
play one tensor-parallel rollout engine. Two transfer paths are timed with CUDA events, max over the
receiving ranks:

* ``kernel_pull``: every engine rank maps trainer ``r % T``'s buffer once (CUDA IPC, opened on the
  engine's GPU) and runs its copy plan: one kernel that reads exactly its TP shard of every parameter
  over NVLink and writes it into the engine's fused layout in place (no gather, no rank-0 funnel);
* ``nccl_broadcast``: the reference's transfer pattern (trainer rank 0 broadcasts the whole model packed
  into 1 GiB buffers; every engine rank receives all of it and would slice afterwards);
* ``vllm_packed_broadcast`` (``--vllm-arm``): the library call the reference's sync makes
  (``agent_textworld.py:1447-1500``): vLLM's ``NCCLWeightTransferEngine.trainer_send_weights(packed=True)``
  on trainer rank 0 over a ``PyNcclCommunicator`` built as ``trainer_init`` builds it, fed the
  HF-named tensors of every parameter, and vLLM's ``packed_nccl_broadcast_consumer`` on every engine
  rank (what ``receive_weights`` runs) with a ``load_weights`` that copies each tensor's TP shard into
  the rank's weight buffer (the narrow + copy of vLLM's weight loaders). The FSDP all-gather that
  precedes the reference's send is not included, so this is a lower bound on the reference's sync.

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
    if a.vllm_arm:
        results.update(_vllm_arm(rank, T, P, cfg, src_layout, buf if rank == 0 else None, dev, a, bcast_group))
    dist.barrier()
    gathered = [None] * world
    dist.all_gather_object(gathered, results)
    if rank == T:
        pulls = [g["kernel_pull_ms"] for g in gathered if "kernel_pull_ms" in g]
        bytes_max = max(g["kernel_pull_bytes"] for g in gathered if "kernel_pull_bytes" in g)
        bc = max(g["nccl_broadcast_ms"] for g in gathered if "nccl_broadcast_ms" in g)
        full_bytes = src_layout.total_numel * 2
        out = {
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
        }
        vl = [g["vllm_packed_broadcast_ms"] for g in gathered if "vllm_packed_broadcast_ms" in g]
        if vl:
            out["vllm_packed_broadcast_ms"] = round(max(vl), 3)
            out["speedup_vs_vllm_packed_broadcast"] = round(max(vl) / max(pulls), 2)
        q.put(out)
    dist.barrier()
    dist.destroy_process_group()


# tensor-parallel split of an HF checkpoint tensor as vLLM's loaders take it: output rows for the
# column-parallel projections and the vocabulary-parallel embedding / head, input columns for the
# row-parallel projections, whole for norms and biases of row-parallel layers
_ROW_SPLIT = ("q_proj.weight", "k_proj.weight", "v_proj.weight", "q_proj.bias", "k_proj.bias", "v_proj.bias",
              "gate_proj.weight", "up_proj.weight", "embed_tokens.weight", "lm_head.weight")
_COL_SPLIT = ("o_proj.weight", "down_proj.weight")


def _tp_shard(name: str, t: torch.Tensor, r: int, P: int) -> torch.Tensor:
    if name.endswith(_ROW_SPLIT):
        n = t.shape[0] // P
        return t.narrow(0, r * n, n)
    if name.endswith(_COL_SPLIT):
        n = t.shape[1] // P
        return t.narrow(1, r * n, n)
    return t


def _vllm_arm(rank, T, P, cfg, src_layout, buf, dev, a, bcast_group):
    """Time vLLM's packed NCCL weight transfer from trainer 0 to the engine ranks (see the module
    docstring). Returns ``{"vllm_packed_broadcast_ms": ms}`` on engine ranks."""
    if rank != 0 and rank < T:
        return {}
    from vllm.distributed.weight_transfer.nccl_engine import NCCLTrainerSendWeightsArgs, NCCLWeightTransferEngine
    from vllm.distributed.weight_transfer.packed_tensor import packed_nccl_broadcast_consumer

    from .models.hf_io import hf_items

    port = [None]
    if rank == 0:
        import socket

        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port[0] = s.getsockname()[1]
    dist.broadcast_object_list(port, src=0, group=bcast_group)
    xfer_rank = 0 if rank == 0 else rank - T + 1
    if rank == 0:
        group = NCCLWeightTransferEngine.trainer_init(dict(master_address="127.0.0.1", master_port=port[0],
                                                           world_size=P + 1))
    else:  # what the vLLM worker's init_transfer_engine does
        group = NCCLWeightTransferEngine._stateless_init_process_group("127.0.0.1", port[0], xfer_rank, P + 1,
                                                                       dev.index)

    def named_views(src):
        for name, slot in src_layout.slots.items():
            view = src[slot.offset : slot.offset + slot.numel].view(slot.shape)
            yield from hf_items(cfg, name, view)

    meta = [(n, (list(t.shape), t.dtype)) for n, t in named_views(torch.empty(src_layout.total_numel,
                                                                               dtype=torch.bfloat16, device="meta"))]
    if rank == 0:
        def run():
            NCCLWeightTransferEngine.trainer_send_weights(named_views(buf),
                                                          NCCLTrainerSendWeightsArgs(group=group, packed=True))
    else:
        r = rank - T
        dst = torch.empty(src_layout.total_numel // P + (1 << 24), dtype=torch.bfloat16, device=dev)

        def load_weights(items):
            off = 0 if not hasattr(load_weights, "off") else load_weights.off
            for name, t in items:
                sh = _tp_shard(name, t, r, P)
                dst[off : off + sh.numel()].view(sh.shape).copy_(sh)
                off += sh.numel()
            load_weights.off = off

        def run():
            load_weights.off = 0
            packed_nccl_broadcast_consumer(iterator=iter(meta), group=group, src=0, post_unpack_func=load_weights)
    ms = _time(run, a.warmup, a.iters, bcast_group)
    del group
    return {} if rank == 0 else {"vllm_packed_broadcast_ms": ms}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--trainers", type=int, default=1)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--json", default=None)
    ap.add_argument("--vllm-arm", action="store_true",
                    help="also time vLLM's packed NCCL weight transfer (the reference's sync call)")
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
