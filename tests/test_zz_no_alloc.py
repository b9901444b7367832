"""The allocation-free sampler entry point ``accerl_sample_logits_noalloc`` (exported C symbol,
called through ctypes) against the workspace-taking sampler on the same inputs, on two calls in a
row (its static scratch keeps its contents between calls), plus its row-limit rejection."""

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
