"""Roofline arithmetic and NVTX ranges (host-only utilities)."""

import json

import pytest
import torch

from accerl_agent_b200.utils import nvtx, roofline


def test_roofline_against_given_peaks(tmp_path):
    f = tmp_path / "peaks.json"
    f.write_text(json.dumps({"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0}))
    p = roofline.load_peaks(str(f))
    assert p.source == "measured" and p.hbm_gbs == 6500.0
    g = roofline.gemm(8192, 8192, 8192, 1.0, peaks=p)
    assert g["tflops"] == pytest.approx(2 * 8192**3 / 1e-3 / 1e12)
    assert g["frac"] == pytest.approx(g["tflops"] / 1600.0)
    assert roofline.gemm(8192, 8192, 8192, 1.0, sustained=True, peaks=p)["peak_tflops"] == 1400.0
    m = roofline.memory(6.5e9, 1.0, peaks=p)
    assert m["frac"] == pytest.approx(1.0)
    # 1 GB over NVLink at 770 GB/s dominates 1 TFLOP of math at 1600 TF/s
    fu = roofline.fused(1e12, 1e9, 2.0, peaks=p)
    assert fu["bound"] == "link" and fu["target_ms"] == pytest.approx(1e9 / 770e9 * 1e3)
    assert fu["frac"] == pytest.approx(fu["target_ms"] / 2.0)
    assert roofline.ridge_point(p) == pytest.approx(1600e12 / 6500e9)
    assert roofline.arithmetic_intensity_gemm(4096, 4096, 4096) == pytest.approx(4096 / 3 * 2 / 2)


def test_roofline_fallback_and_cli(tmp_path, capsys):
    p = roofline.load_peaks(str(tmp_path / "missing.json"))
    assert p.source == "fallback" and p.bf16_tflops == roofline.FALLBACK_BF16_TFLOPS
    out = roofline.main(["bytes", "1e9", "0.5"])
    assert out["gbs"] == pytest.approx(2000.0)
    assert json.loads(capsys.readouterr().out)["gbs"] == pytest.approx(2000.0)


def test_nvtx_ranges_nest_and_default_off():
    assert isinstance(nvtx.range("x"), type(nvtx._NULL)) or nvtx.enabled()
    nvtx.enable(True)
    try:
        with nvtx.range("outer"):
            with nvtx.range("inner"):
                nvtx.mark("point")
                t = torch.ones(4).sum()
        assert float(t) == 4.0
    finally:
        nvtx.enable(False)
    assert not nvtx.enabled()
