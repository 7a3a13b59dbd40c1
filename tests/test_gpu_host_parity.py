"""Parity of the stream kernels with the reference's own torch-CPU arithmetic,
computed on the GPU host's CPU at the full BASELINE size.

The reference's torch backend runs scale as ``torch.mul(src, s, out=dst)`` and
triad as ``torch.add(src, aux, alpha=s, out=dst)``
(src/teamredbench/benchmarks/hbm.py:29-39).  Whether torch's CPU kernel fuses
the triad's multiply-add depends on the CPU capability torch dispatches to, so
the expected bits are decided here, on the machine that runs the kernels, with
torch using every core this process may run on.  Inputs are the BASELINE ones:
2^30 elements, b then c ~ uniform[-1, 1) from seed 0, s = 3.0.  Every element
is compared; the mismatch count and torch's CPU capability are printed.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from tests.helpers import to_raw, uniform_pm1

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200.kernels import stream_op  # noqa: E402

N = 1 << 30
SCALE = 3.0


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover - non-Linux
        return os.cpu_count() or 1


@pytest.mark.parametrize("mode", ["scale", "triad"])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_full_size_matches_host_torch_cpu(dtype, mode):
    b, c = uniform_pm1(N, dtype, seed=0)
    src, aux = (c, None) if mode == "scale" else (b, c)
    dst = torch.empty_like(b)
    stream_op(mode, dst, src, aux, SCALE)
    torch.cuda.synchronize()
    got = to_raw(dst)
    host_src = src.cpu()
    host_aux = aux.cpu() if aux is not None else None
    del dst, b, c, src, aux
    torch.cuda.empty_cache()

    threads_before = torch.get_num_threads()
    threads = _host_threads()
    torch.set_num_threads(threads)
    try:
        want_t = torch.empty_like(host_src)
        if mode == "scale":
            torch.mul(host_src, SCALE, out=want_t)
        else:
            torch.add(host_src, host_aux, alpha=SCALE, out=want_t)
    finally:
        torch.set_num_threads(threads_before)
    want = to_raw(want_t)
    bits = np.uint32 if dtype == "float32" else np.uint16  # compare bit patterns, not values
    mismatches = int(np.count_nonzero(got.view(bits) != want.view(bits)))
    print(f"{dtype} {mode}: torch CPU capability {torch.backends.cpu.get_cpu_capability()}, "
          f"{threads} threads, {mismatches} of {N} elements differ")
    assert mismatches == 0
