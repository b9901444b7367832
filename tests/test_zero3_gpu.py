"""Layer-sharded parameters on 2 GPUs (NCCL, gathers and reduce-scatters on the communication stream
overlapping the layers) against replicated parameters: the same weights after three optimizer steps
of two packs each, and the shard of each rank is half the model."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _cfg():
    from accerl_agent_b200.models.config import ModelConfig

    return ModelConfig(vocab_size=4096, hidden_size=256, num_hidden_layers=3, num_attention_heads=2,
                       num_key_value_heads=1, head_dim=128, intermediate_size=512)


def _batch(seed, dev):
    from accerl_agent_b200.algo.packing import make_varlen_batch
    from accerl_agent_b200.core.sample import RLSample

    g = torch.Generator().manual_seed(seed)
    out = []
    for L in (300, 170):
        ids = torch.randint(0, 4096, (L,), generator=g).tolist()
        labels = [-100] * (L - 40) + ids[L - 40 :]
        out.append(RLSample("grpo", ids, [1] * L, labels, [-8.0] * L, 0.7 if seed % 2 else -0.4, [0.0] * L,
                            [-1] * (L - 40) + [0] * 40, [0]))
    return {k: v.to(dev) for k, v in make_varlen_batch(out).items()}


def _worker(rank, port, sharded, q):
    try:
        os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
        from accerl_agent_b200 import ops
        from accerl_agent_b200.algo.objectives import ObjectiveConfig
        from accerl_agent_b200.models.transformer import build_model
        from accerl_agent_b200.parallel.fsdp import ShardedAdamW
        from accerl_agent_b200.parallel.zero3 import LayerShardedParams, ShardedParamAdamW

        cfg = _cfg()
        if sharded:
            sp = LayerShardedParams(cfg, dev, torch.bfloat16)
            m = sp.model
            m.init_weights(seed=0)
            opt = ShardedParamAdamW(sp, lr=1e-3, weight_decay=0.01)
            stored = sp.local.numel()
        else:
            m = build_model(cfg, "full", dev, torch.bfloat16, pad_to=2)
            m.init_weights(seed=0)
            opt = ShardedAdamW(m, lr=1e-3, weight_decay=0.01)
            stored = m.params.numel()
        grads = {}
        for step in range(3):
            packs = [_batch(100 * step + 10 * rank + i, dev) for i in range(2)]
            total = 4 * 80
            for b in packs:
                lp, ctx = m.forward_logprobs(b, 300)
                tgt = b["target_indices"]
                adv = b["sample_advantages"][b["sequence_ids"][tgt]]
                dlp, _ = ops.policy_loss(lp, b["old_logprobs"][tgt], adv, ObjectiveConfig(), loss_scale=1.0 / total)
                m.backward_from_logprobs(dlp, ctx)
            if step == 0:  # the gradient summed over ranks and packs, before the optimizer consumes it
                if sharded:
                    for u in sp.units:
                        full = torch.empty(u.numel, dtype=torch.float32, device=dev)
                        dist.all_gather_into_tensor(full, sp.local_grads[u.base : u.base + u.shard].contiguous())
                        for n in u.names:
                            sl = sp.layout.slots[n]
                            grads[n] = full[sl.offset - u.lo : sl.offset - u.lo + sl.numel].cpu()
                else:
                    g = m.grads.clone()
                    dist.all_reduce(g)
                    for n, sl in m.layout.slots.items():
                        grads[n] = g[sl.grad_offset : sl.grad_offset + sl.numel].cpu()
            opt.step(1e-3)
        torch.cuda.synchronize()
        full = {}
        if sharded:
            sp.for_each_unit_gathered(lambda u, views: full.update({n: views[n].float().cpu() for n in u.names}))
        else:
            full = {n: v.float().cpu() for n, v in m.named_parameters()}
        ops.check_status(dev)
        q.put((rank, (stored, {n: v.numpy() for n, v in full.items()}, {n: v.numpy() for n, v in grads.items()})))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        q.put((rank, repr(exc)))
        raise


def _run(sharded):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, port, sharded, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(2):
        r, payload = q.get(timeout=300)
        assert not isinstance(payload, str), payload
        out[r] = payload
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return out


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_layer_sharded_training_matches_replicated_on_two_gpus():
    rep = _run(False)
    sh = _run(True)
    for r in (0, 1):
        assert sh[r][0] < 0.6 * rep[r][0]
        # the reduced gradient of the first window: the same sums in another order (fp32)
        for n, g in rep[r][2].items():
            a, b = torch.from_numpy(sh[r][2][n]), torch.from_numpy(g)
            assert (a - b).norm().item() <= 1e-4 * b.norm().item() + 1e-9, n
        # weights after three AdamW steps (lr 1e-3): Adam normalises each element's update, so an
        # element whose gradient is rounding noise steps in a direction set by that noise. The key
        # bias is such a parameter: adding a constant to every key of a head leaves the softmax
        # unchanged, so its gradient is zero up to rounding; it is left out. Everything else agrees
        # to bf16 rounding, with at most a few elements a step or two apart.
        cfg = _cfg()
        for n, w in rep[r][1].items():
            a, b = torch.from_numpy(sh[r][1][n]), torch.from_numpy(w)
            if n.endswith("qkv_proj.bias"):
                keep = torch.ones_like(b, dtype=torch.bool)
                keep[cfg.q_dim : cfg.q_dim + cfg.kv_dim] = False
                a, b = a[keep], b[keep]
            d = (a - b).abs()
            assert d.max().item() <= 7e-3, n
            assert (d > 2e-3 + 2e-2 * b.abs()).float().mean().item() <= 0.01, n
    for n in sh[0][1]:
        assert (sh[0][1][n] == sh[1][1][n]).all(), n
