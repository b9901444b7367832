"""Reference arm of ``bench_rollout.py``: the reference's own inference actor, unmodified, from
``baseline/_ref``.

The generation path timed here is the reference's ``VLLMInferenceActor``
(accerl_agent/agent_textworld.py:1916-2062) exactly as it builds itself: vLLM ``AsyncLLMEngine`` with
``load_format="dummy"`` (random weights), ``enforce_eager=True``, prefix caching, ``max_num_seqs`` /
``max_num_batched_tokens`` from the reference's flags, and its ``InterruptibleGenerationRunner``
(temperature 1.0, stop at ``"\\n"``, log-probs collected). The class is used directly (the Ray stand-in
of ``reference_arm.py`` serves the module-level Ray imports; nothing of Ray runs).

The client is the same synthetic text-game GRPO rollout loop the native arm uses (this repository's
``RolloutWorker`` on ``--env synthetic``): 8 trajectories per group, every request carries the whole
growing transcript as token ids, 16-token actions. It only calls ``request_batch(input_ids,
max_tokens)`` and reads the returned tokens; the reference's own TextWorld worker cannot run without
TextWorld. The tokenizer in the model directory is a word-level one covering the full vocabulary with
no newline token, so the ``"\\n"`` stop never fires and every action is 16 tokens, as in the native
arm.

The actor always enables vLLM expert parallelism, which vLLM 0.22 refuses for a dense model, so this
arm runs MoE shapes only (the reference's validated layout is the Qwen1.5-MoE-A2.7B shape); for a
dense shape it prints its ``unavailable`` line.
"""

from __future__ import annotations

import asyncio
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def _unavailable(reason: str):
    print(json.dumps({"impl": "reference", "metric": "rollout tok/s", "unavailable": reason[:300]}), flush=True)


async def _drive(actor, args, groups: int, seconds: float, warmup: float):
    from accerl_agent_b200.rollout.worker import RolloutWorker

    sink = []
    workers = [RolloutWorker(args, actor, i, sink.extend, lambda *a: None) for i in range(groups)]
    tasks = [asyncio.create_task(w.run()) for w in workers]
    await asyncio.sleep(warmup)
    tok0 = actor.total_tokens
    t0 = time.perf_counter()
    await asyncio.sleep(seconds)
    tok1 = actor.total_tokens
    el = time.perf_counter() - t0
    for w in workers:
        await w.stop()
    await asyncio.wait(tasks, timeout=120)
    return (tok1 - tok0) / el, el, len(sink)


def _vllm_version() -> str:
    try:
        import vllm

        return vllm.__version__
    except Exception:
        return "?"


def run_reference_rollout(a) -> None:
    os.environ.setdefault("CUDA_VISIBLE_DEVICES", "0")
    # this process touches CUDA before vLLM starts its workers, so they must be spawned, not forked
    os.environ.setdefault("VLLM_WORKER_MULTIPROC_METHOD", "spawn")
    if not os.path.isfile(os.path.join(REF_DIR, "accerl_agent", "agent_textworld.py")):
        _unavailable("reference not installed in baseline/_ref")
        return
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    sys.path.insert(0, REF_DIR)
    from baseline.reference_arm import _install_ray_stand_in, _write_model_dir

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
    from accerl_agent_b200.models.config import get_preset

    if get_preset(a.model).num_experts == 0:
        # VLLMInferenceActor always passes enable_expert_parallel=True
        # (accerl_agent/agent_textworld.py:1926); vLLM 0.22 rejects that for a dense model.
        _unavailable("the reference's inference actor hard-codes enable_expert_parallel=True, which vLLM "
                     f"{_vllm_version()} rejects for a dense model ({a.model}); run an MoE shape")
        return
    model_dir = os.environ.get("ACCERL_REF_MODEL_DIR", f"/tmp/accerl_ref_rollout_{a.model}")
    if not os.path.exists(os.path.join(model_dir, "READY")):
        os.makedirs(model_dir, exist_ok=True)
        _write_model_dir(model_dir, a.model, weights=False)
    game_dir = os.path.join(model_dir, "games")
    os.makedirs(game_dir, exist_ok=True)
    argv = ["agent_textworld.py", "--model-path", model_dir, "--tw-game-dir", game_dir,
            "--vllm-max-num-seqs", str(a.max_num_seqs), "--vllm-max-num-batched-tokens", str(a.max_num_batched_tokens),
            "--vllm-max-model-len", str(a.window + 64), "--infer-temperature", "1.0", "--infer-max-tokens", "16",
            "--tw-history-token-window", str(a.window), "--max-length", str(a.window), "--seed", "42",
            "--infer-size", "1", "--infer-tp-size", "1"]
    saved = sys.argv
    sys.argv = argv
    try:
        ref_args = at.parse_args()
    finally:
        sys.argv = saved
    try:
        actor = at.VLLMInferenceActor(ref_args)
    except Exception as exc:
        _unavailable(f"reference vLLM engine init failed: {type(exc).__name__}: {exc}")
        return
    from accerl_agent_b200.core.config import make_args

    args = make_args(model_path=a.model, env="synthetic", rl_algorithm="grpo", rollout_batch_size=8,
                     tw_max_episode_steps=50, tw_history_token_window=a.window, max_length=a.window,
                     infer_max_tokens=16, infer_temperature=1.0)
    async def _run():
        res = await _drive(actor, args, a.groups, a.seconds, a.warmup_seconds)
        try:
            await actor.shutdown()
        except Exception as exc:  # shutdown errors are swallowed, as the reference does
            print(f"[reference] shutdown: {type(exc).__name__}: {exc}", flush=True)
        return res

    rate, el, samples = asyncio.run(_run())
    out = {
        "impl": "reference",
        "metric": "rollout tok/s",
        "value": round(rate, 1),
        "unit": "generated tokens/s (Infer/TokensPerSec), one vLLM engine on 1 GPU",
        "tp": 1,
        "model": a.model,
        "concurrent_trajectories": a.groups * 8,
        "max_num_seqs": a.max_num_seqs,
        "seconds": round(el, 2),
        "samples_produced": samples,
        "code_path": "accerl_agent.agent_textworld.VLLMInferenceActor.request_batch (unmodified; vLLM "
                     "AsyncLLMEngine, enforce_eager, prefix caching, dummy weights)",
    }
    print(json.dumps(out), flush=True)
    if a.json:
        with open(a.json, "w") as f:
            json.dump(out, f, indent=1)
