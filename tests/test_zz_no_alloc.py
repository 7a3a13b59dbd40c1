"""The no-allocation GEMM entry point, through the C ABI.

trb_gemm_launch_noalloc is for callers that cannot let a library allocate
device memory: a framework whose caching allocator already holds nearly all of
HBM (a library cudaMalloc would fail there, or fragment memory the framework
manages), or a latency-critical path that cannot absorb the synchronisation
cudaMalloc / cudaFree may imply.  Its split-K scratch lives in one fixed array
inside the library, shared by every call, so these checks:
  * call it twice in a row on DIFFERENT operands: the first call leaves its
    partials and counters in the array, and the second must not read them.
    Each result must be bit-identical to the ordinary entry point
    (trb_gemm_launch_ex, single-CTA 128 x 256 kernel, same split count: the
    same kernel and the same summation order) and within the GEMM tolerance
    of the fp64 CPU oracle (int8 exact);
  * with splits = 0, pick a split count that fits the array instead of
    refusing the call;
  * refuse an explicit split count larger than the array with a clear error.
This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process."""
from __future__ import annotations

import numpy as np
import pytest

from tests.helpers import GEMM_OUT, GEMM_TOLERANCE, gemm_operands, gemm_result_f64, to_raw, torch_dtype

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

import oracle  # noqa: E402
from teamredbench_b200 import _native  # noqa: E402


def _stream() -> int:
    return int(torch.cuda.current_stream().cuda_stream)


def _existing(name, a, b, sa, sb, splits):
    m, n = a.shape[0], b.shape[1]
    c = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
    _native.gemm_launch_ex(name, m, n, a.shape[1], a.data_ptr(), b.data_ptr(), c.data_ptr(), sa, sb, splits=splits,
                           cta_pair=0, stream=_stream())
    torch.cuda.synchronize()
    return c


def _noalloc(name, a, b, sa, sb, splits):
    m, n = a.shape[0], b.shape[1]
    c = torch.full((m, n), 7, device="cuda", dtype=torch_dtype(GEMM_OUT[name]))  # not zero: must be overwritten
    _native.gemm_launch_noalloc(name, m, n, a.shape[1], a.data_ptr(), b.data_ptr(), c.data_ptr(), sa, sb, splits,
                                _stream())
    torch.cuda.synchronize()
    return c


def _check_oracle(name, a, b, sa, sb, c):
    m = a.shape[0]
    rows = np.arange(m) if m <= 128 else np.sort(np.random.default_rng(0).choice(m, 64, replace=False))
    ref = oracle.gemm_rows(name, to_raw(a), to_raw(b), rows, sa, sb)
    got = gemm_result_f64(name, c)[rows]
    if name == "int8":
        assert np.array_equal(got.astype(np.int64), ref.astype(np.int64))
    else:
        err = oracle.rel_to_max_error(got, ref)
        assert err <= GEMM_TOLERANCE[name], (name, err)


@pytest.mark.parametrize("name,shape,splits", [
    ("bfloat16", (16, 8192, 8192), 0),      # BASELINE skinny shape, automatic splits (4, as trb_gemm_launch_ex)
    ("bfloat16", (128, 4096, 4096), 4),
    ("float16", (96, 2048, 2048), 2),
    ("float8_e4m3fn", (100, 2048, 3072), 3),
    ("int8", (64, 1024, 2048), 5),
    ("tfloat32", (128, 512, 1024), 2),
])
def test_noalloc_two_calls_match_existing_entry_point_and_oracle(name, shape, splits):
    m, n, k = shape
    for seed in (m + n + k, m + n + k + 1):  # the second call runs on different operands
        a, b, sa, sb = gemm_operands(name, m, n, k, seed=seed)
        got = _noalloc(name, a, b, sa, sb, splits)
        want = _existing(name, a, b, sa, sb, splits)
        assert torch.equal(got, want), (name, seed)
        _check_oracle(name, a, b, sa, sb, got)
    assert _native.device_error(0, clear=True) == 0


def test_noalloc_automatic_splits_fit_the_scratch():
    """36 tiles of 128 x 256: trb_gemm_launch_ex's automatic count (4) would
    need 144 tile-splits; splits = 0 must lower it to what the array holds
    (128) and run, not refuse."""
    name, (m, n, k) = "bfloat16", (128, 9216, 8192)
    for seed in (3, 4):
        a, b, sa, sb = gemm_operands(name, m, n, k, seed=seed)
        c = _noalloc(name, a, b, sa, sb, 0)
        _check_oracle(name, a, b, sa, sb, c)
    assert _native.device_error(0, clear=True) == 0


def test_noalloc_rejects_explicit_splits_beyond_the_fixed_scratch():
    a = torch.zeros((512, 4096), device="cuda", dtype=torch.bfloat16)
    b = torch.zeros((4096, 8192), device="cuda", dtype=torch.bfloat16)
    c = torch.empty((512, 8192), device="cuda", dtype=torch.bfloat16)
    # 4 x 32 tiles x 8 splits = 1024 tile-splits > 128
    with pytest.raises(_native.NativeError) as info:
        _native.gemm_launch_noalloc("bfloat16", 512, 8192, 4096, a.data_ptr(), b.data_ptr(), c.data_ptr(), 1.0, 1.0,
                                    8, _stream())
    assert "fixed scratch" in str(info.value)
