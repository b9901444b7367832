"""Trainer -> rollout weight-sync benchmark on two GPUs of one node.

    python -m accerl_agent_b200.bench_sync [--model qwen3-8b] [--iters 5]

GPU 0 plays a trainer rank holding the full bf16 compute copy of the model in the fused layout;
GPU 1 plays a rollout engine. Two transfer paths are timed with CUDA events (device time of the
receiving GPU, max over the two processes where both take part):

* ``ipc_pull``: the engine maps the trainer buffer once (CUDA IPC) and copies it into its own weights
  in place (one peer-to-peer copy over NVLink, no staging, no rank-0 funnel);
* ``nccl_broadcast``: the baseline transfer of the reference (NCCL broadcast of the weights packed into
  1 GiB buffers, double-buffered), between the same two GPUs.
"""

from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _proc(rank: int, a, port: int, q):
    torch.cuda.set_device(rank)
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=torch.device("cuda", rank))
    from .models.config import get_preset
    from .models.transformer import ParamLayout

    cfg = get_preset(a.model)
    n = ParamLayout.build(cfg, "full").total_numel
    buf = torch.empty(n, dtype=torch.bfloat16, device="cuda")
    if rank == 0:
        buf.normal_()
    results = {}
    # ---- IPC pull
    if rank == 0:
        from torch.multiprocessing.reductions import reduce_tensor

        obj = [reduce_tensor(buf)]
    else:
        obj = [None]
    dist.broadcast_object_list(obj, src=0)
    if rank == 1:
        fn, fargs = obj[0]
        src = fn(*fargs)
        ts = []
        for i in range(a.warmup + a.iters):
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            buf.copy_(src, non_blocking=True)
            e.record()
            torch.cuda.synchronize()
            if i >= a.warmup:
                ts.append(s.elapsed_time(e))
        assert torch.equal(buf[:1024].cpu(), src[:1024].cpu())
        results["ipc_pull_ms"] = sorted(ts)[len(ts) // 2]
    dist.barrier()
    # ---- NCCL broadcast in packed 1 GiB buffers
    bucket = (1 << 30) // 2
    ts = []
    for i in range(a.warmup + a.iters):
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for off in range(0, n, bucket):
            dist.broadcast(buf[off : off + bucket], src=0)
        e.record()
        torch.cuda.synchronize()
        if i >= a.warmup:
            ts.append(s.elapsed_time(e))
    t = torch.tensor([sorted(ts)[len(ts) // 2]], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    results["nccl_broadcast_ms"] = float(t.item())
    if rank == 1:
        gb = n * 2 / 1e9
        q.put({
            "metric": "weight-sync ms",
            "model": a.model,
            "bytes": n * 2,
            "ipc_pull_ms": round(results["ipc_pull_ms"], 3),
            "ipc_pull_gbs": round(gb / (results["ipc_pull_ms"] / 1e3), 1),
            "nccl_broadcast_ms": round(results["nccl_broadcast_ms"], 3),
            "nccl_broadcast_gbs": round(gb / (results["nccl_broadcast_ms"] / 1e3), 1),
            "link_roofline_ms_at_770GBs": round(gb / 770 * 1e3, 3),
        })
    dist.barrier()
    dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-8b")
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--json", default=None)
    a = ap.parse_args()
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_proc, args=(r, a, port, q)) for r in range(2)]
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
