import teamredbench_b200.builtin  # noqa: F401
from teamredbench_b200.native.registry import list_native_kernels
from teamredbench_b200.profiling.registry import list_profile_engines
from teamredbench_b200.registry import list_benchmarks, list_metrics


def test_builtin_registrations_present():
    assert {"hbm", "collective", "mfu"} <= set(list_benchmarks())
    assert {"latency_us", "hbm_bandwidth_gbps", "hbm_efficiency_pct", "payload_bandwidth_gbps",
            "bus_bandwidth_gbps", "link_efficiency_pct", "achieved_tops", "mfu_pct"} <= set(list_metrics())


def test_native_kernels_include_reference_names_as_aliases():
    names = {d.name: d for d in list_native_kernels()}
    assert {"hbm_b200", "mfu_b200", "hbm_hip", "mfu_hipblas"} <= set(names)
    assert names["hbm_hip"].binary_path == names["hbm_b200"].binary_path
    assert names["mfu_hipblas"].benchmark == "mfu"


def test_ncu_engine_registered():
    assert "ncu" in {d.name for d in list_profile_engines()}
