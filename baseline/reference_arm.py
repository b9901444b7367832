"""Reference arm of ``bench.py``: the reference's own trainer code, unmodified, from ``baseline/_ref``.

The reference is a set of scripts whose trainer class (``FSDPTrainWorker``,
accerl_agent/agent_textworld.py:419-1570) normally runs as a Ray actor. Ray and TextWorld are not
installed here, so this module provides an in-process stand-in for the small Ray surface that the
trainer path touches (``ray.remote`` on classes, ``.remote()`` method calls, ``ray.get``) and an empty
``textworld`` module for the module-level import. Everything that runs on the GPU is the reference's
own stack: HF ``AutoModelForCausalLM`` with ``flash_attention_2``, FSDP2 ``fully_shard`` per layer,
bf16 AdamW, its varlen packing and loss code. As under Ray, each rank sees exactly one GPU
(``CUDA_VISIBLE_DEVICES`` = local rank), which the reference assumes (it selects device index 0).

The model is a random-init HF checkpoint of the benchmark shape written to a local directory, with a
minimal word-level tokenizer (the trainer only needs its pad / eos ids). Samples are the same seeded
synthetic text-game episodes the native arm trains on.
"""

from __future__ import annotations

import json
import os
import sys
import time
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _install_ray_stand_in():
    ray = types.ModuleType("ray")

    class _Method:
        def __init__(self, fn):
            self._fn = fn

        def remote(self, *a, **k):
            return self._fn(*a, **k)

        def __call__(self, *a, **k):
            return self._fn(*a, **k)

    class _Handle:
        def __init__(self, obj):
            self._obj = obj

        def __getattr__(self, name):
            return _Method(getattr(self._obj, name))

    class _ActorClass:
        def __init__(self, cls):
            self._cls = cls

        def remote(self, *a, **k):
            return _Handle(self._cls(*a, **k))

        def options(self, **_):
            return self

    def remote(*args, **kwargs):
        if args and isinstance(args[0], type) and not kwargs:
            return _ActorClass(args[0])
        return lambda cls: _ActorClass(cls)

    def get(x, timeout=None):
        return list(x) if isinstance(x, (list, tuple)) else x

    ray.remote = remote
    ray.get = get
    ray.wait = lambda refs, num_returns=1, timeout=None: (list(refs)[:num_returns], list(refs)[num_returns:])
    ray.init = lambda *a, **k: None
    ray.shutdown = lambda *a, **k: None
    ray.cancel = lambda *a, **k: None
    sys.modules["ray"] = ray
    tw = types.ModuleType("textworld")
    tw_gym = types.ModuleType("textworld.gym")
    tw.gym = tw_gym
    tw.EnvInfos = lambda **k: k
    sys.modules["textworld"] = tw
    sys.modules["textworld.gym"] = tw_gym


def _write_model_dir(path: str, model: str, weights: bool = True):
    """Random-init HF checkpoint + word-level tokenizer of the benchmark shape (rank 0 writes).
    ``weights=False`` writes only the config and tokenizer (enough for vLLM's dummy weights)."""
    import torch
    import transformers
    from tokenizers import Tokenizer, models, pre_tokenizers

    from accerl_agent_b200.models.config import get_preset

    cfg = get_preset(model)
    hf_cfg = transformers.AutoConfig.for_model(**cfg.to_hf_dict())
    if weights:
        torch.manual_seed(42)
        m = transformers.AutoModelForCausalLM.from_config(hf_cfg, dtype=torch.bfloat16)
        m.save_pretrained(path, safe_serialization=True)
    else:
        hf_cfg.save_pretrained(path)
    # word-level vocabulary over every model id (no newline token), so any sampled id decodes
    vocab = {"<|endoftext|>": 0, "<|im_start|>": 1, "<|im_end|>": 2}
    for i in range(3, cfg.vocab_size):
        vocab[f"w{i}"] = i
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<|endoftext|>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    fast = transformers.PreTrainedTokenizerFast(tokenizer_object=tok, eos_token="<|endoftext|>",
                                                pad_token="<|endoftext|>")
    fast.save_pretrained(path)
    with open(os.path.join(path, "READY"), "w") as f:
        f.write("ok\n")


def _unavailable(reason: str):
    print(json.dumps({"impl": "reference", "unavailable": reason[:300]}), flush=True)


def run_reference(a):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    os.environ["CUDA_VISIBLE_DEVICES"] = str(local)
    if not os.path.isfile(os.path.join(REF_DIR, "accerl_agent", "agent_textworld.py")):
        _unavailable("reference not installed in baseline/_ref")
        return
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    sys.path.insert(0, REF_DIR)
    _install_ray_stand_in()
    import torch

    if not torch.cuda.is_available():
        _unavailable("no CUDA device")
        return
    try:
        import accerl_agent.agent_textworld as at
    except Exception as exc:  # pragma: no cover - depends on the image
        _unavailable(f"reference import failed: {type(exc).__name__}: {exc}")
        return
    from dataclasses import asdict

    model_dir = os.environ.get("ACCERL_REF_MODEL_DIR", f"/tmp/accerl_ref_{a.model}")
    if rank == 0 and not os.path.exists(os.path.join(model_dir, "READY")):
        os.makedirs(model_dir, exist_ok=True)
        _write_model_dir(model_dir, a.model)
    deadline = time.time() + 900
    while not os.path.exists(os.path.join(model_dir, "READY")):
        if time.time() > deadline:
            _unavailable("timed out waiting for the reference model directory")
            return
        time.sleep(1)
    game_dir = os.path.join(model_dir, "games")
    os.makedirs(game_dir, exist_ok=True)
    argv = [
        "agent_textworld.py", "--model-path", model_dir, "--tw-game-dir", game_dir,
        "--train-packing", "varlen", "--train-token-budget", str(a.token_budget), "--max-length", str(a.max_length),
        "--tw-history-token-window", str(a.max_length), "--batch-size", str(a.batch_size),
        "--grad-accum-steps", str(a.grad_accum_steps), "--train-logprob-mode", "response_only_lm_head",
        "--dtype", "bfloat16", "--fsdp-world-size", str(world), "--rl-algorithm", "grpo", "--clip-mode", "ppo",
        "--clip-eps", "0.2", "--learning-rate", "1e-6", "--lr-warmup-steps", "0", "--max-steps", "1000000",
        "--train-mode", "full", "--seed", "42", "--sync-every-optimizer-steps", "1",
    ]
    saved = sys.argv
    sys.argv = argv
    try:
        args = at.parse_args()
    finally:
        sys.argv = saved
    addr = os.environ.get("MASTER_ADDR", "127.0.0.1")
    port = int(os.environ.get("MASTER_PORT", "29517"))
    replay = at.ReplayBufferActor.remote(capacity=args.replay_capacity)
    from accerl_agent_b200.env.synthetic_samples import benchmark_pool

    pool = benchmark_pool(rank, 256, a.max_length)
    replay.add_samples.remote([at.RLSample(**asdict(s)) for s in pool[: args.replay_capacity]])
    try:
        worker = at.FSDPTrainWorker(args, rank, world, addr, port, replay)
    except Exception as exc:
        _unavailable(f"reference trainer init failed: {type(exc).__name__}: {exc}")
        return
    import torch.distributed as dist

    for _ in range(a.warmup):
        worker.train_until_next_sync(1)
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    from accerl_agent_b200.utils.clocks import ClockSampler

    tokens = 0.0
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        start.record()
        for _ in range(a.steps):
            summary = worker.train_until_next_sync(1)
            tokens += float(summary["segment_valid_tokens"])
        end.record()
        torch.cuda.synchronize()
        dist.barrier()
    ms = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    value = tokens / (ms / 1e3)
    cs = clocks.summary()
    if rank == 0:
        print(json.dumps({
            "impl": "reference",
            "metric": "trainer tok/s",
            "value": round(value, 1),
            "unit": "target tokens/s (global valid response tokens per second, Train/TokensPerSec)",
            "n_gpus": world,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": round(ms / a.steps, 3),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded synthetic text-game episodes, random-init weights)",
            "config": {
                "model": "Qwen2.5-1.5B-shape dense (HF Qwen2ForCausalLM, flash_attention_2, FSDP2)",
                "global_batch": a.batch_size * a.grad_accum_steps * world,
                "seq_len": a.max_length,
                "token_budget_per_pack": a.token_budget,
                "grad_accum_steps": a.grad_accum_steps,
                "parallelism": f"fsdp{world}",
                "code_path": "accerl_agent.agent_textworld.FSDPTrainWorker.train_until_next_sync (unmodified)",
            },
            "e2e": {"value": round(value, 1), "unit": "target tokens/s through the reference's own API",
                    "note": "the reference's call includes replay sampling, CPU packing, H2D and the stats read"},
            "clocks": {"sm_mhz": cs.get("sm_mhz"), "sm_max_mhz": cs.get("sm_max_mhz"),
                       "reasons": cs.get("reasons", []), "samples": cs.get("samples", 0)},
        }), flush=True)
    worker.close()
