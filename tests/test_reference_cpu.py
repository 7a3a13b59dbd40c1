"""The restated reference CPU path that bench.py times (``--impl reference`` and the
``cpu_baseline`` leg): same ops, inputs and timing rules as the reference's torch
backend (hbm.py:29-39, mfu.py:230-252, utils.py:14-29)."""
import math

import pytest
import torch

from oracle import reference_cpu


def test_run_mode_is_the_reference_ops():
    g = torch.Generator().manual_seed(3)
    src, aux = torch.rand(1000, generator=g), torch.rand(1000, generator=g)
    dst = torch.empty_like(src)
    reference_cpu.run_mode(torch, "copy", src, dst, None, 3.0)
    assert torch.equal(dst, src)
    reference_cpu.run_mode(torch, "scale", src, dst, None, 3.0)
    assert torch.equal(dst, torch.mul(src, 3.0))
    reference_cpu.run_mode(torch, "triad", src, dst, aux, 3.0)
    assert torch.equal(dst, torch.add(src, aux, alpha=3.0))
    with pytest.raises(KeyError, match="Unknown HBM mode: bogus"):
        reference_cpu.run_mode(torch, "bogus", src, dst, aux, 3.0)


def test_hbm_inputs_are_seeded_uniform_b_then_c():
    b, c = reference_cpu.hbm_inputs(torch, 4096, "bfloat16")
    b2, c2 = reference_cpu.hbm_inputs(torch, 4096, "bfloat16")
    assert b.dtype == torch.bfloat16 and torch.equal(b, b2) and torch.equal(c, c2)
    assert not torch.equal(b, c)
    assert float(b.float().min()) >= -1.0 and float(b.float().max()) <= 1.0


def test_time_hbm_reports_the_reference_bytes():
    r = reference_cpu.time_hbm(torch, "triad", 1 << 16, "float32", 3.0, 1, 2)
    assert r["moved_bytes"] == 3 * (1 << 16) * 4  # MODE_BYTE_FACTORS (hbm.py:18-22)
    assert r["elapsed_s"] > 0 and r["gbps"] > 0
    assert reference_cpu.time_hbm(torch, "copy", 1 << 16, "bfloat16", 3.0, 0, 1)["moved_bytes"] == 2 * (1 << 16) * 2


def test_gemm_inputs_are_seeded_and_scaled():
    a, b = reference_cpu.gemm_inputs(torch, 64, 48, 256, "bfloat16")
    a2, b2 = reference_cpu.gemm_inputs(torch, 64, 48, 256, "bfloat16")
    assert a.shape == (64, 256) and b.shape == (256, 48) and a.dtype == torch.bfloat16
    assert torch.equal(a, a2) and torch.equal(b, b2)
    assert abs(float(a.float().std()) - 1 / math.sqrt(256)) < 0.01


def test_time_gemm_runs_torch_mm_and_counts_2mnk():
    r = reference_cpu.time_gemm(torch, "bfloat16", 64, 48, 32, 1, 2)
    assert r["achieved_ops"] == 2 * 64 * 48 * 32  # mfu.py:252
    assert r["elapsed_s"] > 0 and r["tflops"] > 0 and r["iterations"] == 2
