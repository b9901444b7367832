"""Local supervised smoke trainer (response-only SFT), single process or sharded over ranks.

    python -m accerl_agent_b200.local_trainer --model-path tiny-qwen2 --device cpu --use-fsdp --fsdp-world-size 2

Same flags as the reference's ``local_trainer.py`` (LT:575-616). The data is either the reference's
eight dummy chat examples (needs a tokenizer with a chat template; prompt tokens are masked with -100,
LT:21-54,142-177) or, with ``--dataset random`` (used automatically when the model has no tokenizer),
uniform-random token sequences of ``--max-length`` tokens whose last ``--response-length`` tokens are
the labels. The loss is the mean token cross-entropy over labelled tokens (the HF ``outputs.loss``),
divided by ``--grad-accum-steps``; every ``grad-accum-steps`` micro-steps the gradient is clipped at
1.0 and the sharded AdamW steps (LT:349-398). ``--use-fsdp`` starts ``--fsdp-world-size`` ranks with
NCCL on GPUs or gloo on ``--device cpu``; each rank trains on its own slice of the data.
"""

from __future__ import annotations

import argparse
import os
import random
import socket
from typing import List

import torch
import torch.distributed as dist

DUMMY_CHAT_EXAMPLES = [
    {"user": "什么是 MoE 模型？", "assistant": "MoE 模型会把 token 路由到不同专家网络中处理，从而在控制计算量的同时扩大参数规模。"},
    {"user": "用一句话解释强化学习。", "assistant": "强化学习是让智能体通过奖励信号学习如何在环境中做决策的方法。"},
    {"user": "给我一个 Python 列表推导式例子。", "assistant": "例如 squares = [x * x for x in range(5)]，它会得到 0 到 4 的平方。"},
    {"user": "What is the capital of France?", "assistant": "The capital of France is Paris."},
    {"user": "Summarize local model training in one sentence.",
     "assistant": "Local model training loads weights, prepares batches, runs forward and backward passes, updates "
                  "parameters, and saves a checkpoint."},
    {"user": "解释一下 attention mask 的作用。", "assistant": "attention mask 用来告诉模型哪些 token 是有效输入，哪些 token 是 padding，应当被忽略。"},
    {"user": "什么是 checkpoint?", "assistant": "checkpoint 是训练过程中保存下来的模型权重和 tokenizer 文件，可用于恢复训练或推理。"},
    {"user": "Give a tiny JSON example.", "assistant": '{"name": "local-trainer", "status": "ok"}'},
]


def parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Local response-only SFT smoke test, optionally sharded over ranks.")
    p.add_argument("--model-path", required=True)
    p.add_argument("--device", default="cuda:0", help="auto, cpu, cuda, cuda:0, ...")
    p.add_argument("--dtype", default="auto", choices=("auto", "bfloat16", "float16", "float32"))
    p.add_argument("--train-mode", default="lm_head", choices=("lm_head", "last_layer", "full"))
    p.add_argument("--max-length", type=int, default=128)
    p.add_argument("--batch-size", type=int, default=2)
    p.add_argument("--max-steps", type=int, default=1000)
    p.add_argument("--learning-rate", type=float, default=1e-5)
    p.add_argument("--weight-decay", type=float, default=0.0)
    p.add_argument("--grad-accum-steps", type=int, default=2)
    p.add_argument("--dataset-repeat", type=int, default=4)
    p.add_argument("--log-every", type=int, default=1)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--trust-remote-code", action="store_true")
    p.add_argument("--gradient-checkpointing", action="store_true")
    p.add_argument("--use-fsdp", action="store_true")
    p.add_argument("--fsdp-world-size", type=int, default=4)
    p.add_argument("--fsdp-master-addr", default=None)
    p.add_argument("--fsdp-master-port", type=int, default=None)
    p.add_argument("--ray-address", default=None, help="Accepted for command-line compatibility (unused).")
    p.add_argument("--dataset", default="auto", choices=("auto", "dummy-chat", "random"))
    p.add_argument("--response-length", type=int, default=32)
    args = p.parse_args(argv)
    for name in ("grad_accum_steps", "max_steps", "batch_size", "fsdp_world_size"):
        if getattr(args, name) < 1:
            raise ValueError(f"--{name.replace('_', '-')} must be >= 1")
    return args


def _tokenizer(args):
    if not os.path.isdir(args.model_path):
        return None
    try:
        from transformers import AutoTokenizer

        tok = AutoTokenizer.from_pretrained(args.model_path, local_files_only=True,
                                            trust_remote_code=args.trust_remote_code)
        if tok.pad_token is None:
            tok.pad_token = tok.eos_token
        return tok
    except Exception:
        return None


def encode_chat(tokenizer, user: str, assistant: str, max_length: int):
    """(input_ids, labels) with the prompt masked (LT:142-177)."""
    if getattr(tokenizer, "chat_template", None):
        prompt = tokenizer.apply_chat_template([{"role": "user", "content": user}], tokenize=False,
                                               add_generation_prompt=True)
        full = tokenizer.apply_chat_template([{"role": "user", "content": user},
                                              {"role": "assistant", "content": assistant}], tokenize=False,
                                             add_generation_prompt=False)
    else:
        prompt = f"User: {user}\nAssistant: "
        full = f"User: {user}\nAssistant: {assistant}"
    p_ids = tokenizer(prompt, add_special_tokens=False, truncation=True, max_length=max_length)["input_ids"]
    ids = tokenizer(full, add_special_tokens=False, truncation=True, max_length=max_length)["input_ids"]
    labels = list(ids)
    n = min(len(p_ids), len(labels))
    labels[:n] = [-100] * n
    if labels and all(x == -100 for x in labels):
        labels[-1] = ids[-1]
    return ids, labels


def build_dataset(args, tokenizer, vocab_size: int) -> List:
    rng = random.Random(args.seed)
    data = []
    use_chat = args.dataset == "dummy-chat" or (args.dataset == "auto" and tokenizer is not None)
    for _ in range(args.dataset_repeat):
        if use_chat:
            if tokenizer is None:
                raise ValueError("--dataset dummy-chat needs a tokenizer in --model-path")
            for ex in DUMMY_CHAT_EXAMPLES:
                data.append(encode_chat(tokenizer, ex["user"], ex["assistant"], args.max_length))
        else:
            for _ in range(len(DUMMY_CHAT_EXAMPLES)):
                ids = [rng.randrange(vocab_size) for _ in range(args.max_length)]
                resp = min(args.response_length, args.max_length - 1)
                labels = [-100] * (args.max_length - resp) + ids[args.max_length - resp:]
                data.append((ids, labels))
    return data


def run_training(rank: int, world: int, args) -> dict:
    from .algo.packing import make_varlen_batch
    from .core.sample import RLSample
    from .models.config import resolve_model_config
    from .models.hf_io import load_hf_checkpoint
    from .models.transformer import build_model
    from .parallel.fsdp import ShardedAdamW
    from .trainer.worker import pick_dtype, set_seed

    if args.device in ("auto", "cuda") or args.device.startswith("cuda"):
        if torch.cuda.is_available():
            dev = torch.device("cuda", rank if world > 1 else (torch.device(args.device).index or 0)
                               if args.device.startswith("cuda:") else rank)
        else:
            dev = torch.device("cpu")
    else:
        dev = torch.device(args.device)
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    set_seed(args.seed + rank)
    cfg = resolve_model_config(args.model_path)
    dtype = pick_dtype(args.dtype, dev)
    model = build_model(cfg, args.train_mode, dev, dtype, pad_to=world)
    model.gradient_checkpointing = args.gradient_checkpointing
    if os.path.isdir(args.model_path) and any(f.endswith(".safetensors") for f in os.listdir(args.model_path)):
        load_hf_checkpoint(model, args.model_path)
    else:
        model.init_weights(seed=args.seed)
    opt = ShardedAdamW(model, lr=args.learning_rate, weight_decay=args.weight_decay)
    tokenizer = _tokenizer(args)
    data = build_dataset(args, tokenizer, cfg.vocab_size)
    data = data[rank::world]  # each rank trains on its own slice (the DistributedSampler split)
    if rank == 0:
        total = sum(s.numel for s in model.layout.slots.values())
        trainable = sum(s.numel for s in model.layout.slots.values() if s.trainable)
        print(f"[train] Parameter count: trainable={trainable:,} / total={total:,} ({trainable / total:.4%})")
        print(f"[train] Starting training: max_steps={args.max_steps}, batch_size={args.batch_size}, "
              f"grad_accum_steps={args.grad_accum_steps}")
    step = 0
    last_loss = 0.0
    idx = 0
    while step < args.max_steps:
        batch_items = [data[(idx + i) % len(data)] for i in range(args.batch_size)]
        idx += args.batch_size
        samples = [RLSample("grpo", ids, [1] * len(ids), [-100] + labels[1:], [0.0] * len(ids), 0.0, [0.0] * len(ids),
                            [-1] + [0 if l != -100 else -1 for l in labels[1:]], [0]) for ids, labels in batch_items]
        batch = {k: v.to(dev) for k, v in make_varlen_batch(samples).items()}
        lp, ctx = model.forward_logprobs(batch, max(len(s.input_ids) for s in samples))
        n = lp.numel()
        loss = -lp.float().mean()
        dlp = torch.full_like(lp, -1.0 / (n * args.grad_accum_steps * world))
        model.backward_from_logprobs(dlp, ctx)
        step += 1
        if step % args.grad_accum_steps == 0:
            opt.step(args.learning_rate)
        last_loss = float(loss.item())
        if world > 1:
            t = torch.tensor([last_loss], dtype=torch.float64, device=dev if dev.type == "cuda" else "cpu")
            dist.all_reduce(t)
            last_loss = float(t.item()) / world
        if rank == 0 and step % args.log_every == 0:
            print(f"[train] step={step} loss={last_loss:.6f}")
    return {"rank": rank, "steps": step, "last_loss": last_loss}


def _fsdp_entry(rank: int, args, port: int, results):
    os.environ["MASTER_ADDR"] = args.fsdp_master_addr or "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    world = args.fsdp_world_size
    use_cuda = args.device != "cpu" and torch.cuda.is_available()
    if use_cuda:
        torch.cuda.set_device(rank)
    dist.init_process_group("nccl" if use_cuda else "gloo", rank=rank, world_size=world)
    try:
        results[rank] = run_training(rank, world, args)
    finally:
        dist.destroy_process_group()


def main(argv=None) -> dict:
    args = parse_args(argv)
    if not args.use_fsdp:
        res = run_training(0, 1, args)
        print(f"[train] done: {res}")
        return res
    port = args.fsdp_master_port
    if not port:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
    import torch.multiprocessing as mp

    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.spawn(_fsdp_entry, args=(args, port, results), nprocs=args.fsdp_world_size, join=True)
    res = dict(results)
    print(f"[train] FSDP training finished: {[res[r] for r in sorted(res)]}")
    return res


if __name__ == "__main__":
    main()
