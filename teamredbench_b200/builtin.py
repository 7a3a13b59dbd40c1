"""Importing this module registers every built-in benchmark, metric, native
kernel and profiler engine (reference: src/teamredbench/builtin.py)."""
from teamredbench_b200.benchmarks import collective, hbm, mfu  # noqa: F401
from teamredbench_b200.metrics import common  # noqa: F401
from teamredbench_b200.native import builtin as _native_builtin  # noqa: F401
from teamredbench_b200.profiling import builtin as _profiling_builtin  # noqa: F401
