"""Host-side checks of the torch-tensor front end (teamredbench_b200/kernels.py)
that need no GPU: dtype mapping and the argument checks that run before any
launch."""
from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from teamredbench_b200 import _native  # noqa: E402
from teamredbench_b200.kernels import gemm, stream_op, trb_dtype  # noqa: E402


@pytest.mark.parametrize("tdt, name", [(torch.float32, "float32"), (torch.bfloat16, "bfloat16"),
                                       (torch.float16, "float16"), (torch.float64, "float64"),
                                       (torch.int8, "int8"), (torch.float8_e4m3fn, "float8_e4m3fn")])
def test_trb_dtype_maps_torch_dtypes(tdt, name):
    t = torch.empty(1, dtype=tdt)
    assert trb_dtype(t) == name
    assert trb_dtype(t) == name  # second lookup goes through the per-dtype cache


def test_trb_dtype_rejects_unsupported_as_skipped():
    with pytest.raises(_native.NativeSkipped):
        trb_dtype(torch.empty(1, dtype=torch.complex64))


def test_gemm_rejects_host_tensors_before_launching():
    a = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA device"):
        gemm(a, a.t().contiguous(), torch.zeros(4, 4, dtype=torch.bfloat16))


def test_stream_op_rejects_host_tensors_before_launching():
    x = torch.zeros(16)
    with pytest.raises(ValueError, match="CUDA device"):
        stream_op("copy", x, x)
