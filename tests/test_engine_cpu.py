"""Generation engine on the CPU path (tiny fp32 model): greedy decoding equals recomputation of
full-sequence logits, chunked prefill and prefix caching give identical outputs, pause aborts
in-flight requests, and the interruptible runner resubmits prompt + partial output after resume."""

import asyncio

import pytest
import torch

from accerl_agent_b200.models.config import get_preset
from accerl_agent_b200.models.transformer import build_model
from accerl_agent_b200.rollout.engine import GenerationEngine
from accerl_agent_b200.rollout.generation import InterruptibleGenerationRunner, OnlineGenerationState, SamplingParams


def make_engine(**kw):
    cfg = get_preset("tiny-qwen2")
    m = build_model(cfg, "full", torch.device("cpu"), torch.float32, with_grads=False)
    m.init_weights(seed=7, std=0.08)
    eng = GenerationEngine(cfg, torch.device("cpu"), torch.float32, params=m.params, num_blocks=256, block_size=4,
                           **kw)
    return cfg, m, eng


def greedy_reference(m, prompt, n):
    ids = list(prompt)
    for _ in range(n):
        t = torch.tensor(ids)
        logits = m.forward_logits_full(t, torch.arange(len(ids)), torch.tensor([0, len(ids)], dtype=torch.int32),
                                       len(ids))
        ids.append(int(logits[-1].argmax()))
    return ids[len(prompt):]


async def collect(eng, prompt, params, rid):
    last = None
    async for out in eng.generate({"prompt_token_ids": prompt}, params, request_id=rid):
        last = out
    return last


def test_greedy_matches_full_recompute_with_chunking_and_prefix_cache():
    cfg, m, eng = make_engine(max_num_batched_tokens=7)
    prompts = [[5, 6, 7, 8, 9, 10, 11, 12, 13], [1, 2, 3], [5, 6, 7, 8, 9, 10, 11, 12, 40, 41]]
    params = SamplingParams(temperature=0.0, max_tokens=6, logprobs=1, ignore_eos=True)

    async def run():
        outs = await asyncio.gather(*[collect(eng, p, params, f"r{i}") for i, p in enumerate(prompts)])
        again = await collect(eng, prompts[2] + [1], params, "r-again")  # prefix-cache hit path
        await eng.shutdown()
        return outs, again

    outs, again = asyncio.run(run())
    for p, o in zip(prompts, outs):
        assert o.finished and o.outputs[0].finish_reason == "length"
        assert o.outputs[0].token_ids == greedy_reference(m, p, 6)
        assert len(o.outputs[0].logprobs) == 6
    assert again.outputs[0].token_ids == greedy_reference(m, prompts[2] + [1], 6)
    assert eng.allocator.hits > 0


def test_pause_aborts_and_runner_resumes_with_new_version():
    cfg, m, eng = make_engine(max_num_batched_tokens=64)
    N = 400
    _, _, eng_ref = make_engine(max_num_batched_tokens=64)

    async def reference():
        o = await collect(eng_ref, [3, 4, 5, 6], SamplingParams(temperature=0.0, max_tokens=N, ignore_eos=True), "ref")
        await eng_ref.shutdown()
        return o.outputs[0].token_ids

    uninterrupted = asyncio.run(reference())

    async def run():
        runner = InterruptibleGenerationRunner(eng, temperature=0.0, top_p=1.0, stop_sequences=None,
                                               collect_logprobs=True)
        runner.stop_sequences = None
        state = OnlineGenerationState(index=0, input_ids=[3, 4, 5, 6], requested_max_tokens=N)
        task = asyncio.create_task(runner.generate(state))
        while eng.stats["generated_tokens"] < 5:
            await asyncio.sleep(0.0005)
        runner.pause()
        await eng.pause_generation(mode="abort", clear_cache=True)
        await runner.wait_for_idle()
        partial = list(state.output_tokens)
        runner.version += 1
        await eng.resume_generation(version=runner.version)
        runner.resume()
        await task
        await eng.shutdown()
        return state, partial

    state, partial = asyncio.run(run())
    assert len(state.output_tokens) == N and state.stop_reason == "length"
    assert 0 < len(partial) < N and eng.stats["aborted"] == 1
    assert state.output_versions[: len(partial)] == [0] * len(partial)
    assert set(state.output_versions[len(partial):]) <= {1}
    # greedy continuation after the abort equals an uninterrupted greedy run
    assert state.output_tokens == uninterrupted


def test_suspend_keeps_one_submission_and_tags_versions():
    """Weight-sync pause in suspend mode: the request is parked (no abort, no resubmission), then
    continues under the new version; greedy output equals an uninterrupted run."""
    cfg, m, eng = make_engine(max_num_batched_tokens=64)
    N = 900  # long enough that the pause lands mid-generation even on a loaded host
    _, _, eng_ref = make_engine(max_num_batched_tokens=64)

    async def reference():
        o = await collect(eng_ref, [3, 4, 5, 6], SamplingParams(temperature=0.0, max_tokens=N, ignore_eos=True), "ref")
        await eng_ref.shutdown()
        return o.outputs[0].token_ids

    uninterrupted = asyncio.run(reference())

    async def run():
        runner = InterruptibleGenerationRunner(eng, temperature=0.0, top_p=1.0, stop_sequences=None,
                                               collect_logprobs=True)
        runner.stop_sequences = None
        state = OnlineGenerationState(index=0, input_ids=[3, 4, 5, 6], requested_max_tokens=N)
        task = asyncio.create_task(runner.generate(state))
        while eng.stats["generated_tokens"] < 5:
            await asyncio.sleep(0.0005)
        runner.pause()
        await eng.pause_generation(mode="suspend", clear_cache=True)
        before = eng.stats["generated_tokens"]
        await asyncio.sleep(0.05)
        assert eng.stats["generated_tokens"] == before  # nothing runs while paused
        runner.version += 1
        await eng.resume_generation(version=runner.version)
        runner.resume()
        await task
        await eng.shutdown()
        return state, before

    state, before = asyncio.run(run())
    assert before < N, "the request finished before the pause"
    assert state.stop_reason == "length" and len(state.output_tokens) == N
    assert eng.stats["aborted"] == 0 and eng.stats["suspended"] == 1
    assert state.output_versions == [0] * before + [1] * (N - before)
    assert len(state.output_logprobs) == N
    assert state.output_tokens == uninterrupted


def test_unsupported_sampling_parameter_is_refused():
    """A frequency penalty is not applied by the engine's sampler, so a request asking for one fails
    instead of silently sampling without it."""
    _, _, eng = make_engine()

    async def run():
        with pytest.raises(ValueError, match="frequency_penalty"):
            async for _ in eng.generate({"prompt_token_ids": [3, 4]},
                                        SamplingParams(max_tokens=2, frequency_penalty=0.5), "fp"):
                pass
        await eng.shutdown()

    asyncio.run(run())
