"""Randomised GEMM parity through the C ABI: seeded ragged shapes, every input
type, both B layouts and the kernel options (automatic choice, single CTA or
CTA pair, tile widths, workspace or cluster split-K, the swapped-operand
kernel), each checked against the fp64 CPU oracle with the reference
harness's rel-to-max metric (tests/native/gemm_parity.hip.cpp:163-178).
Option combinations a kernel does not take must be refused with an error,
never computed wrongly."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests.helpers import GEMM_OUT, GEMM_TOLERANCE, gemm_operands, gemm_result_f64, to_raw, torch_dtype

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200 import _native  # noqa: E402
from teamredbench_b200.kernels import gemm  # noqa: E402

DTYPES = ["bfloat16", "float16", "tfloat32", "float8_e4m3fn", "int8", "float32", "float64"]
ELEM = {"bfloat16": 2, "float16": 2, "tfloat32": 4, "float8_e4m3fn": 1, "int8": 1, "float32": 4, "float64": 8}


def _case(seed: int):
    rng = np.random.default_rng(seed)
    name = DTYPES[seed % len(DTYPES)]
    es = ELEM[name]
    align = 1 if name == "float64" else 16 // es  # TMA: rows of 16-byte multiples
    m = int(rng.choice([int(rng.integers(1, 65)), int(rng.integers(65, 300)), int(rng.integers(300, 700))]))
    n = int(rng.integers(1, 1200 // align + 1)) * align
    k = int(rng.integers(1, 3000 // align + 1)) * align
    options = [{}, {"cta_pair": 0}, {"cta_pair": 1}, {"cta_pair": 0, "tile_n": 128}, {"splits": 3},
               {"splits": -2}, {"splits": -4}, {"tile_n": -1}, {"tile_n": -1, "splits": -2}]
    opt = options[int(rng.integers(len(options)))]
    return name, m, n, k, bool(rng.integers(2)), opt


@pytest.mark.parametrize("seed", range(160))
def test_random_gemm_matches_oracle(seed):
    name, m, n, k, b_transposed, opt = _case(seed)
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=seed)
    bb = b.t().contiguous() if b_transposed else b
    c = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
    try:
        gemm(a, bb, c, dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed, **opt)
    except _native.NativeError as e:
        # only combinations a kernel does not take may be refused
        refusable = ("cluster split-K" in str(e) or "swapped-operand kernel takes m <= 64" in str(e)
                     or "8-bit row-major B" in str(e))
        assert refusable, (name, m, n, k, b_transposed, opt, str(e))
        return
    torch.cuda.synchronize()
    assert _native.device_error(0, clear=True) == 0
    rows = np.arange(m) if m <= 160 else np.sort(np.random.default_rng(seed).choice(m, 160, replace=False))
    ref = oracle.gemm_rows(name, to_raw(a), to_raw(b), rows, sa, sb)
    got = gemm_result_f64(name, c)[rows]
    if name == "int8":
        assert np.array_equal(got.astype(np.int64), ref.astype(np.int64)), (m, n, k, b_transposed, opt)
        return
    tol = 1e-12 if name == "float64" else GEMM_TOLERANCE[name]
    err = oracle.rel_to_max_error(got, ref)
    assert err <= tol, (name, m, n, k, b_transposed, opt, err)
