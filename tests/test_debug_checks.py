"""Debug-checks build (``ACCERL_DEBUG_CHECKS=1 python setup.py build_ext --inplace``): data-dependent
indices (token ids, KV-cache slots, page ids, MoE row positions) are range-checked in the kernels; a
failing check is recorded (first failure wins) and the access is skipped, so nothing traps.

On CPU the kernel files are compiled with the flag (the debug build must keep building). On a GPU,
a release build reports no records; a debug build records an out-of-range token id and KV-cache
slot that the release kernels would have used as addresses (that case runs only when the loaded
extension was built with the checks, since only then is the access skipped)."""

import os
import shutil
import subprocess

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("nvcc") is None, reason="nvcc not found")
def test_debug_checks_build_compiles(tmp_path):
    from torch.utils.cpp_extension import include_paths

    incs = [f"-I{p}" for p in include_paths()] + [f"-I{os.path.join(ROOT, 'csrc')}"]
    procs = []
    for unit in ("elementwise", "moe", "rollout", "attention"):
        cmd = ["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17", "--expt-relaxed-constexpr",
               "-DACCERL_DEBUG_CHECKS", "-c", os.path.join(ROOT, "csrc", f"{unit}.cu"),
               "-o", str(tmp_path / f"{unit}.o")] + incs
        procs.append((unit, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    for unit, p in procs:
        out, _ = p.communicate(timeout=600)
        assert p.returncode == 0, (unit, out.decode()[-2000:])
        assert (tmp_path / f"{unit}.o").stat().st_size > 0


@pytest.mark.gpu
def test_debug_status_release_build_reports_nothing():
    from accerl_agent_b200 import ops

    if ops.debug_checks_enabled():
        pytest.skip("debug-checks build loaded")
    assert ops.debug_status() == {}


@pytest.mark.gpu
def test_debug_build_records_out_of_range_indices():
    from accerl_agent_b200 import ops

    if not ops.debug_checks_enabled():
        pytest.skip("release build: out-of-range indices are not checked (and must not be used)")
    ops.debug_status(reset=True)
    table = torch.randn(64, 128, device="cuda").bfloat16()
    ids = torch.tensor([3, 64, 5], device="cuda")  # 64 is one past the last row
    out = torch.zeros(3, 128, device="cuda", dtype=torch.bfloat16)
    ops.native().embedding_fwd(ids, table, out)
    torch.cuda.synchronize()
    assert ops.debug_status(reset=True) == {"elementwise": ("embedding token id", 64)}
    assert torch.equal(out[0], table[3]) and torch.equal(out[2], table[5]) and not out[1].any()
    kc = torch.zeros(4, 16, 2, 128, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    kv = torch.randn(2, 256, device="cuda").bfloat16()
    slots = torch.tensor([7, 64], device="cuda", dtype=torch.int32)  # 64 slots exist
    ops.kv_cache_write(kv, kv, kc, vc, slots, 2)
    torch.cuda.synchronize()
    assert ops.debug_status(reset=True) == {"rollout": ("KV-cache slot", 64)}
    assert torch.equal(kc.view(64, 256)[7], kv[0])


def test_debug_status_decoding_with_a_fake_extension(monkeypatch):
    """``ops.debug_status`` names the failed check per kernel file and drops files without a failure;
    ``debug_checks_enabled`` is true only when the extension returns records (a debug build)."""
    from accerl_agent_b200.ops import _ext

    class Fake:
        def __init__(self, recs):
            self.recs, self.resets = recs, 0

        def debug_status(self, reset):
            self.resets += int(reset)
            return self.recs

    fake = Fake([("attention", 3, 977), ("elementwise", 0, 0), ("moe", 4, -1), ("rollout", 0, 0)])
    monkeypatch.setattr(_ext, "native", lambda: fake)
    assert _ext.debug_checks_enabled()
    assert _ext.debug_status(reset=True) == {"attention": ("KV-cache page id", 977), "moe": ("MoE row position", -1)}
    assert fake.resets == 1
    monkeypatch.setattr(_ext, "native", lambda: Fake([]))
    assert not _ext.debug_checks_enabled() and _ext.debug_status() == {}
