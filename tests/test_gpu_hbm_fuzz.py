"""Randomised HBM stream parity through the C ABI: seeded element counts
(ragged, from one element to millions), every dtype and mode, every launch
variant, misaligned pointers (element offsets into a larger buffer, which
take the scalar path), grid caps (the reference's --blocks-per-cu) and
scales, each compared bit for bit with the CPU oracle of the reference's
torch arithmetic (src/teamredbench/benchmarks/hbm.py:29-39).  Combinations
the reference also refuses (int8 scale / triad, memcpy for a non-copy mode)
must come back as skipped, never computed."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.helpers import to_raw, uniform_pm1

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200 import _native  # noqa: E402
from teamredbench_b200.kernels import stream_op  # noqa: E402

DTYPES = ["float32", "bfloat16", "float16", "float64", "int8"]
MODES = ["copy", "scale", "triad"]
VARIANTS = ["auto", "vec", "bulk", "memcpy"]


def _case(seed: int):
    rng = np.random.default_rng(1000 + seed)
    dtype = DTYPES[seed % len(DTYPES)]
    mode = MODES[int(rng.integers(3))]
    variant = VARIANTS[int(rng.integers(4))]
    count = int(rng.choice([int(rng.integers(1, 64)), int(rng.integers(64, 70000)), int(rng.integers(70000, 3_000_000))]))
    offsets = [int(x) for x in rng.integers(0, 8, size=3)] if rng.integers(3) == 0 else [0, 0, 0]
    bps = int(rng.choice([0, 0, 1, 4, 32]))
    scale = float(rng.choice([3.0, 0.1, -1.7, float(rng.uniform(-4, 4))]))
    return dtype, mode, variant, count, offsets, bps, scale


def _buffer(dtype, count, offset, seed):
    full = uniform_pm1(count + 8, dtype, seed=seed, device="cuda")[0]
    return full[offset:offset + count]  # element offset: misaligned for offset % (16 / elem) != 0


@pytest.mark.parametrize("seed", range(120))
def test_random_stream_op_matches_oracle(seed):
    dtype, mode, variant, count, (od, os_, oa), bps, scale = _case(seed)
    src = _buffer(dtype, count, os_, seed)
    aux = _buffer(dtype, count, oa, seed + 7) if mode == "triad" else None
    dst = torch.empty(count + 8, device="cuda", dtype=src.dtype)[od:od + count]
    try:
        stream_op(mode, dst, src, aux, scale, variant=variant, blocks_per_sm=bps)
    except _native.NativeSkipped:
        assert (dtype == "int8" and mode != "copy") or (variant == "memcpy" and mode != "copy"), \
            (dtype, mode, variant)
        return
    torch.cuda.synchronize()
    want = oracle.hbm(dtype, mode, to_raw(src), to_raw(aux) if aux is not None else None, scale)
    got = to_raw(dst)
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (dtype, mode, variant, count, od, os_, oa, bps, scale)
