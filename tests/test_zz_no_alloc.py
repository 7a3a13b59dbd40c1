"""The no-allocation GEMM entry point, through the C ABI.

trb_gemm_launch_noalloc is for callers that cannot let a library allocate
device memory (a framework whose allocator already owns most of HBM, or a
latency-critical path that cannot absorb cudaMalloc's synchronisation).  Its
split-K scratch lives in a fixed array inside the library, so these checks:
  * compare it with the ordinary entry point (trb_gemm_launch_ex, same
    kernel, same split count) within the GEMM tolerances of the other tests,
    on two calls in a row -- the array keeps the previous call's contents,
    and the second call must not see stale counters or partials;
  * check that a request larger than the fixed scratch is refused with a
    clear error.
This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process."""
from __future__ import annotations

import numpy as np
import pytest

from tests.helpers import GEMM_OUT, GEMM_TOLERANCE, gemm_operands, gemm_result_f64, torch_dtype

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


@pytest.mark.parametrize("name,shape,splits", [
    ("bfloat16", (16, 8192, 8192), 0),      # BASELINE skinny shape, automatic splits
    ("bfloat16", (128, 4096, 4096), 4),
    ("float8_e4m3fn", (100, 2048, 3072), 3),
    ("int8", (64, 1024, 2048), 5),
    ("tfloat32", (128, 512, 1024), 2),
])
def test_noalloc_matches_existing_entry_point_twice(name, shape, splits):
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=m + n + k)
    want = gemm_result_f64(name, _existing(name, a, b, sa, sb, splits))
    for _ in range(2):  # second call reuses the array as the first call left it
        got = gemm_result_f64(name, _noalloc(name, a, b, sa, sb, splits))
        if name == "int8":
            assert np.array_equal(got, want)
        else:
            assert oracle.rel_to_max_error(got, want) <= GEMM_TOLERANCE[name]
    assert _native.device_error(0, clear=True) == 0


def test_noalloc_rejects_requests_beyond_the_fixed_scratch():
    a = torch.zeros((512, 4096), device="cuda", dtype=torch.bfloat16)
    b = torch.zeros((4096, 8192), device="cuda", dtype=torch.bfloat16)
    c = torch.empty((512, 8192), device="cuda", dtype=torch.bfloat16)
    # 4 x 32 tiles x 8 splits = 1024 tile-splits > 128
    with pytest.raises(_native.NativeError) as info:
        _native.gemm_launch_noalloc("bfloat16", 512, 8192, 4096, a.data_ptr(), b.data_ptr(), c.data_ptr(), 1.0, 1.0,
                                    8, _stream())
    assert "fixed scratch" in str(info.value)
