"""The reference's own CPU implementation of the hot path, restated for timing.

TEST / BASELINE INFRASTRUCTURE ONLY (used by ``bench.py --impl reference`` and
the ``cpu_baseline`` leg; never by the product package).

The reference's torch backend runs the STREAM ops as
    copy : dst.copy_(src)
    scale: torch.mul(src, s, out=dst)
    triad: torch.add(src, aux, alpha=s, out=dst)
(src/teamredbench/benchmarks/hbm.py:29-39) and GEMM as torch.mm(a, b, out=out)
(src/teamredbench/benchmarks/mfu.py:229-234), timed by `timed_iterations`
(src/teamredbench/utils.py:14-29: warm up, synchronize, perf_counter around N
calls, mean seconds per call).  The reference tree cannot travel to the GPU
host, so these few lines restate those calls; with the same torch they are the
same computation.  On a CUDA-less run the reference itself reports "No ROCm
device visible to PyTorch" (hbm.py:179-184), so this restatement is the only
way to time the reference's arithmetic on host cores.
"""
from __future__ import annotations

import math
import time
from typing import Callable


def run_mode(torch, mode: str, src, dst, aux, scale: float) -> None:
    if mode == "copy":
        dst.copy_(src)
    elif mode == "scale":
        torch.mul(src, scale, out=dst)
    elif mode == "triad":
        torch.add(src, aux, alpha=scale, out=dst)
    else:
        raise KeyError(f"Unknown HBM mode: {mode}")


def timed_iterations(fn: Callable[[], None], warmup: int, iterations: int) -> float:
    for _ in range(warmup):
        fn()
    start = time.perf_counter()
    for _ in range(iterations):
        fn()
    return (time.perf_counter() - start) / max(iterations, 1)


def hbm_inputs(torch, n: int, dtype_name: str, seed: int = 0):
    """BASELINE inputs: b then c ~ uniform[-1, 1) from `seed` (CPU generator)."""
    g = torch.Generator().manual_seed(seed)
    dt = getattr(torch, dtype_name)
    b = torch.empty(n, dtype=torch.float32)
    c = torch.empty(n, dtype=torch.float32)
    b.uniform_(-1.0, 1.0, generator=g)
    c.uniform_(-1.0, 1.0, generator=g)
    return b.to(dt), c.to(dt)


def time_hbm(torch, mode: str, n: int, dtype_name: str, scale: float, warmup: int, iterations: int) -> dict:
    b, c = hbm_inputs(torch, n, dtype_name)
    dst = torch.empty_like(b)
    src = c if mode == "scale" else b
    aux = c if mode == "triad" else None
    elapsed = timed_iterations(lambda: run_mode(torch, mode, src, dst, aux, scale), warmup, iterations)
    factor = 3 if mode == "triad" else 2
    moved = factor * n * b.element_size()
    return {"elapsed_s": elapsed, "moved_bytes": moved, "gbps": moved / elapsed / 1e9,
            "threads": torch.get_num_threads()}


def gemm_inputs(torch, m: int, n: int, k: int, dtype_name: str, seed: int = 0):
    """BASELINE GEMM inputs: A (m x k) then B (k x n) ~ N(0, 1)/sqrt(k) from `seed`
    (CPU generator), cast to the dtype.  The reference draws unseeded randn
    (utils.py:32-48); the scale keeps bf16 products in range at every K."""
    g = torch.Generator().manual_seed(seed)
    dt = getattr(torch, dtype_name)
    a = torch.randn((m, k), generator=g) / math.sqrt(k)
    b = torch.randn((k, n), generator=g) / math.sqrt(k)
    return a.to(dt), b.to(dt)


def time_gemm(torch, dtype_name: str, m: int, n: int, k: int, warmup: int, iterations: int) -> dict:
    """The reference's torch GEMM case (mfu.py:230-240): torch.mm(a, b, out=out)
    with out in the input dtype, timed by timed_iterations; achieved_ops = 2mnk
    (mfu.py:252)."""
    a, b = gemm_inputs(torch, m, n, k, dtype_name)
    out = torch.empty((m, n), dtype=a.dtype)
    elapsed = timed_iterations(lambda: torch.mm(a, b, out=out), warmup, iterations)
    ops = 2 * m * n * k
    return {"elapsed_s": elapsed, "achieved_ops": ops, "tflops": ops / elapsed / 1e12,
            "threads": torch.get_num_threads(), "warmup": warmup, "iterations": iterations}
