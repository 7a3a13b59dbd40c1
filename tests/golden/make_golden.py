"""Generate the golden input/output fixtures that pin the CPU oracle.

Run in the build container (where the reference checkout is importable):

    python tests/golden/make_golden.py --reference-src <reference>/src

HBM fixtures call the reference's own torch implementation,
``HbmBandwidthBenchmark._run_mode`` (src/teamredbench/benchmarks/hbm.py:29-39),
on CPU tensors with a single torch thread.  GEMM fixtures restate the reference
torch path's one line ``torch.mm(a, b, out=out)`` with the output in the input
dtype (src/teamredbench/benchmarks/mfu.py:229-234); dtypes the reference torch
path does not cover (int8 with int32 accumulate, e4m3 with per-tensor scales,
tf32) use torch's CPU ``_int_mm`` / ``_scaled_mm`` / fp32 ``mm`` on tf32-rounded
inputs.  Inputs follow BASELINE.json's distributions (uniform[-1,1) for the
stream arrays, N(0,1)/sqrt(K) for GEMM operands, A drawn before B, seed 0).

The files are small (n=515 stream arrays, 64x96x128 GEMMs) and are read at
test time without the reference tree.
"""
from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
HBM_N = 515                      # 16 * 32 + 3: a ragged length with a scalar remainder
HBM_SCALES = (3.0, 0.1, -1.7)
HBM_DTYPES = ("float32", "float64", "bfloat16", "float16")
GEMM_SHAPES = {"square": (64, 96, 128), "ragged": (48, 80, 40)}


def _raw(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy().copy()
    return t.contiguous().numpy().copy()


def _reference_hbm_bench(reference_src: Path):
    sys.path.insert(0, str(reference_src))
    from teamredbench.benchmarks.base import BenchmarkContext
    from teamredbench.benchmarks.hbm import HbmBandwidthBenchmark
    from teamredbench.config import HardwareProfile, RuntimeProfile

    context = BenchmarkContext(
        hardware_profile=HardwareProfile(name="golden", family="cpu"),
        runtime_profile=RuntimeProfile(name="golden"),
        device_info=None,
        torch_module=torch,
        dtype_specs={},
    )
    return HbmBandwidthBenchmark(context=context, params={}, record_sink=None)


def make_hbm(reference_src: Path) -> dict[str, np.ndarray]:
    bench = _reference_hbm_bench(reference_src)
    out: dict[str, np.ndarray] = {"n": np.array(HBM_N), "scales": np.array(HBM_SCALES),
                                  "cpu_capability": np.array(torch.backends.cpu.get_cpu_capability())}
    for dtype_name in HBM_DTYPES:
        dt = getattr(torch, dtype_name)
        g = torch.Generator().manual_seed(0)
        if dt == torch.float64:
            b = torch.rand(HBM_N, generator=g, dtype=torch.float64) * 2 - 1
            c = torch.rand(HBM_N, generator=g, dtype=torch.float64) * 2 - 1
        else:
            b = (torch.rand(HBM_N, generator=g) * 2 - 1).to(dt)
            c = (torch.rand(HBM_N, generator=g) * 2 - 1).to(dt)
        out[f"{dtype_name}/b"] = _raw(b)
        out[f"{dtype_name}/c"] = _raw(c)
        dst = torch.empty_like(b)
        bench._run_mode("copy", b, dst, None, 1.0)
        out[f"{dtype_name}/copy"] = _raw(dst)
        for s in HBM_SCALES:
            dst = torch.empty_like(c)
            bench._run_mode("scale", c, dst, None, s)
            out[f"{dtype_name}/scale/{s}"] = _raw(dst)
            dst = torch.empty_like(b)
            bench._run_mode("triad", b, dst, c, s)
            out[f"{dtype_name}/triad/{s}"] = _raw(dst)
    g = torch.Generator().manual_seed(0)
    i8 = torch.randint(-128, 128, (HBM_N,), generator=g, dtype=torch.int8)
    dst = torch.empty_like(i8)
    bench._run_mode("copy", i8, dst, None, 1.0)
    out["int8/b"] = _raw(i8)
    out["int8/copy"] = _raw(dst)
    return out


def _round_tf32(x: torch.Tensor) -> torch.Tensor:
    bits = x.contiguous().view(torch.int32).numpy().astype(np.int64)
    bits = ((bits + 0x1000) & 0xFFFFE000) & 0xFFFFFFFF
    return torch.from_numpy(bits.astype(np.uint32).view(np.int32)).view(torch.float32)


def make_gemm() -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    for tag, (m, n, k) in GEMM_SHAPES.items():
        dtypes = (("bfloat16", "float16", "tfloat32", "float8_e4m3fn", "int8", "float32", "float64")
                  if tag == "square" else ("bfloat16",))
        for dtype_name in dtypes:
            g = torch.Generator().manual_seed(0)
            key = f"{tag}/{dtype_name}"
            out[f"{key}/shape"] = np.array([m, n, k])
            if dtype_name == "int8":
                a = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int8)
                b = torch.randint(-127, 128, (k, n), generator=g, dtype=torch.int8)
                c = torch._int_mm(a, b)
                out.update({f"{key}/a": _raw(a), f"{key}/b": _raw(b), f"{key}/c": _raw(c)})
                continue
            a32 = torch.randn(m, k, generator=g) / math.sqrt(k)
            b32 = torch.randn(k, n, generator=g) / math.sqrt(k)
            if dtype_name == "float64":
                a = torch.randn(m, k, generator=g, dtype=torch.float64) / math.sqrt(k)
                b = torch.randn(k, n, generator=g, dtype=torch.float64) / math.sqrt(k)
                c = torch.empty((m, n), dtype=torch.float64)
                torch.mm(a, b, out=c)
                out.update({f"{key}/a": _raw(a), f"{key}/b": _raw(b), f"{key}/c": _raw(c)})
            elif dtype_name in ("bfloat16", "float16", "float32"):
                dt = getattr(torch, dtype_name)
                a, b = a32.to(dt), b32.to(dt)
                c = torch.empty((m, n), dtype=dt)
                torch.mm(a, b, out=c)
                out.update({f"{key}/a": _raw(a), f"{key}/b": _raw(b), f"{key}/c": _raw(c)})
            elif dtype_name == "tfloat32":
                a, b = _round_tf32(a32), _round_tf32(b32)
                c = torch.empty((m, n), dtype=torch.float32)
                torch.mm(a, b, out=c)
                out.update({f"{key}/a": _raw(a), f"{key}/b": _raw(b), f"{key}/c": _raw(c)})
            else:  # e4m3 with per-tensor scales mapping absmax to 448
                sa = float(a32.abs().max()) / 448.0
                sb = float(b32.abs().max()) / 448.0
                qa = (a32 / sa).to(torch.float8_e4m3fn)
                qb = (b32 / sb).to(torch.float8_e4m3fn)
                c = torch._scaled_mm(qa, qb.t().contiguous().t(), scale_a=torch.tensor(sa), scale_b=torch.tensor(sb),
                                     out_dtype=torch.bfloat16)
                out.update({f"{key}/a": _raw(qa), f"{key}/b": _raw(qb), f"{key}/c": _raw(c),
                            f"{key}/scales": np.array([sa, sb], dtype=np.float64)})
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference-src", type=Path, required=True)
    args = parser.parse_args()
    torch.set_num_threads(1)
    np.savez_compressed(HERE / "hbm_golden.npz", **make_hbm(args.reference_src))
    np.savez_compressed(HERE / "gemm_golden.npz", **make_gemm())
    for name in ("hbm_golden.npz", "gemm_golden.npz"):
        print(name, (HERE / name).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
