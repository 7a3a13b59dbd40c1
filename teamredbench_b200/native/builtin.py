"""Built-in native kernels: the B200 launchers over libtrb_b200.so.

`hbm_b200` / `mfu_b200` are the defaults of the hbm / mfu benchmarks.  The
reference's built-in names `hbm_hip` / `mfu_hipblas`
(src/teamredbench/native/builtin.py:11-23) are registered as aliases of the
same executables so that unchanged suites (`native.kernel: hbm_hip`) run on
B200."""
from __future__ import annotations

from teamredbench_b200._native import HBM_EXECUTABLE, MFU_EXECUTABLE
from teamredbench_b200.native.registry import register_native_kernel

_HBM = "B200 STREAM copy/scale/triad kernels (vector and TMA-bulk paths), libtrb_b200."
_MFU = "B200 tcgen05/TMEM/TMA GEMM (bf16, f16, tf32, e4m3, int8), libtrb_b200."

register_native_kernel(name="hbm_b200", benchmark="hbm", description=_HBM, binary_path=HBM_EXECUTABLE)
register_native_kernel(name="mfu_b200", benchmark="mfu", description=_MFU, binary_path=MFU_EXECUTABLE)
register_native_kernel(name="hbm_hip", benchmark="hbm", description="alias of hbm_b200: " + _HBM,
                       binary_path=HBM_EXECUTABLE)
register_native_kernel(name="mfu_hipblas", benchmark="mfu", description="alias of mfu_b200: " + _MFU,
                       binary_path=MFU_EXECUTABLE)
