"""Two-GPU bandwidth of moving one large contiguous bf16 "model" (default 4 GiB).

    python -m accerl_agent_b200.bench_nccl [--op broadcast|all_reduce|p2p_pull] [--size-gib 4] [--shards 1]

``broadcast`` and ``all_reduce`` are the NCCL collectives the reference measures
(``minimal_model_nccl_bandwidth.py``: warm-up 5, 20 timed iterations, GB/s = payload / time);
``p2p_pull`` is this framework's path for weights: GPU 1 maps GPU 0's buffers once by CUDA IPC and
its copy kernel reads them over NVLink. Device time with CUDA events, max over the two ranks.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank: int, a, port: int, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
    from . import ops
    from .ops._ext import native
    from .rollout.weight_map import CopyDesc, descs_tensor

    total = int(a.size_gib * 1024**3) // 2
    base, extra = divmod(total, a.shards)
    shards = [torch.empty(base + (1 if i < extra else 0), dtype=torch.bfloat16, device=dev) for i in range(a.shards)]
    if rank == 0:
        for t in shards:
            t.normal_()
    payload = sum(t.numel() for t in shards) * 2
    if a.op == "p2p_pull":
        handles = [native().ipc_export(t) for t in shards] if rank == 0 else None
        obj = [handles]
        dist.broadcast_object_list(obj, src=0)
        if rank == 1:
            native().enable_peer_access(0)
            plans = []
            for (rc, h, off), t in zip(obj[0], shards):
                rc2, b = native().ipc_open(h)
                assert rc == 0 and rc2 == 0
                plans.append((descs_tensor([CopyDesc(0, t.numel(), 0, t.numel(), 1, t.numel())], dev), b + off, t))

            def step():
                for plan, src, dst in plans:
                    ops.weight_pull(plan, src, dst)
        else:
            def step():
                pass
    elif a.op == "broadcast":
        def step():
            for t in shards:
                dist.broadcast(t, src=0)
    else:
        def step():
            for t in shards:
                dist.all_reduce(t)
    ts = []
    for i in range(a.warmup + a.iters):
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step()
        e.record()
        torch.cuda.synchronize()
        if i >= a.warmup:
            ts.append(s.elapsed_time(e))
    ms = torch.tensor([sum(ts) / len(ts)], dtype=torch.float64, device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    if rank == 0:
        t = float(ms.item())
        q.put({"metric": "bandwidth GB/s", "op": a.op, "payload_gb": round(payload / 1e9, 3), "shards": a.shards,
               "ms": round(t, 3), "value": round(payload / 1e9 / (t / 1e3), 1)})
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="broadcast", choices=("broadcast", "all_reduce", "p2p_pull"))
    ap.add_argument("--size-gib", type=float, default=4.0)
    ap.add_argument("--shards", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, a, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join()
    out = q.get(timeout=5)
    print(json.dumps(out))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
