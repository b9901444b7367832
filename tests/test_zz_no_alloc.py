"""The allocation-free sampler entry point ``accerl_sample_logits_noalloc`` (exported C symbol,
called through ctypes; prototype in csrc/accerl_noalloc.h) against the workspace-taking sampler on
the same inputs, on two calls in a row (its static scratch keeps its contents between calls), on
logits with -inf entries, plus its row-limit rejection."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    import accerl_agent_b200._C as ext

    lib = ctypes.CDLL(ext.__file__)
    fn = lib.accerl_sample_logits_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _call(fn, logits, rows, temperature, seeds, offsets, tokens, lps):
    return fn(logits.data_ptr(), logits.stride(0), rows, logits.shape[1], temperature.data_ptr(), seeds.data_ptr(),
              offsets.data_ptr(), tokens.data_ptr(), lps.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_sampler_matches_workspace_sampler():
    from accerl_agent_b200 import ops

    fn = _symbol()
    torch.manual_seed(0)
    rows, V = 300, 151936
    logits = (torch.randn(rows, V, device="cuda") * 3).to(torch.bfloat16)
    temperature = torch.rand(rows, device="cuda") + 0.5
    temperature[::7] = 0.0  # greedy rows
    seeds = torch.randint(0, 2**62, (rows,), device="cuda", dtype=torch.int64)
    offsets = torch.arange(rows, device="cuda", dtype=torch.int64) * 3
    tok_ref, lp_ref = ops.sample(logits, temperature, seeds, offsets)
    torch.cuda.synchronize()
    for _ in range(2):
        tokens = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
        lps = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        assert _call(fn, logits, rows, temperature, seeds, offsets, tokens, lps) == 0
        torch.cuda.synchronize()
        assert torch.equal(tokens, tok_ref)
        torch.testing.assert_close(lps, lp_ref, rtol=1e-5, atol=1e-5)


def test_noalloc_sampler_minus_inf_logits():
    """-inf logits (leading chunks masked, a row with one finite logit): finite log-probabilities
    equal to log_softmax at the sampled token, and the same tokens as the workspace sampler."""
    from accerl_agent_b200 import ops

    fn = _symbol()
    rows, V = 6, 151936
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(rows, V, generator=g) * 2
    x[0, : V // 2] = float("-inf")
    x[1, torch.rand(V, generator=g) < 0.95] = float("-inf")
    x[2, :] = float("-inf")
    x[2, 17] = 0.25
    logits = x.bfloat16().cuda()
    temperature = torch.tensor([1.0, 0.8, 1.0, 0.0, 1.3, 1.0], device="cuda")
    seeds = torch.arange(rows, device="cuda", dtype=torch.int64) * 7 + 1
    offsets = torch.zeros(rows, device="cuda", dtype=torch.int64)
    tok_ref, lp_ref = ops.sample(logits, temperature, seeds, offsets)
    want_all = torch.log_softmax(logits.float(), -1)
    for _ in range(2):
        tokens = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
        lps = torch.full((rows,), float("nan"), dtype=torch.float32, device="cuda")
        assert _call(fn, logits, rows, temperature, seeds, offsets, tokens, lps) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(lps).all()
        assert torch.equal(tokens, tok_ref)
        want = want_all.gather(1, tokens.view(-1, 1)).squeeze(1)
        torch.testing.assert_close(lps, want, atol=2e-3, rtol=1e-4)
        torch.testing.assert_close(lps, lp_ref, rtol=1e-5, atol=1e-5)
        assert int(tokens[2]) == 17


def test_noalloc_sampler_rejects_more_rows_than_its_scratch():
    fn = _symbol()
    rows, V = 1025, 64
    logits = torch.zeros(rows, V, dtype=torch.bfloat16, device="cuda")
    temperature = torch.ones(rows, device="cuda")
    seeds = torch.zeros(rows, dtype=torch.int64, device="cuda")
    offsets = torch.zeros(rows, dtype=torch.int64, device="cuda")
    tokens = torch.full((rows,), -1, dtype=torch.int64, device="cuda")
    lps = torch.zeros(rows, dtype=torch.float32, device="cuda")
    assert _call(fn, logits, rows, temperature, seeds, offsets, tokens, lps) == -30
    torch.cuda.synchronize()
    assert bool((tokens == -1).all())  # nothing was launched
