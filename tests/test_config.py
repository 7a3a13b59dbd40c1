from pathlib import Path

from teamredbench_b200.config import load_hardware_profile, load_suite

SUITES = Path(__file__).resolve().parent.parent / "teamredbench_b200" / "configs" / "suites"
HW = SUITES.parent / "profiles" / "hardware"


def test_load_suite_resolves_profiles():
    suite = load_suite(SUITES / "smoke.yaml")
    assert suite.name == "smoke"
    assert suite.hardware_profile.family == "nvidia"
    assert suite.runtime_profile.cuda_version == "12.9"
    assert suite.outputs.directory.name == "smoke"
    assert suite.profiling.enabled is False


def test_baseline_suites_load():
    for name, bench in [("b200_hbm_stream.yaml", "hbm"), ("b200_gemm_sweep.yaml", "mfu"),
                        ("b200_gemm_mixed.yaml", "mfu"), ("b200_collective.yaml", "collective")]:
        suite = load_suite(SUITES / name)
        assert suite.benchmarks[0].benchmark == bench
        assert suite.hardware_profile.name == "nvidia-b200"


def test_native_smoke_keeps_reference_kernel_names():
    suite = load_suite(SUITES / "native_smoke.yaml")
    assert [b.params["native"]["kernel"] for b in suite.benchmarks] == ["hbm_hip", "mfu_hipblas"]


def test_ncu_suite_profiling_config():
    suite = load_suite(SUITES / "ncu_hbm_smoke.yaml")
    assert suite.profiling.enabled and suite.profiling.engine == "ncu"


def test_b200_profile_peaks():
    profile = load_hardware_profile(HW / "nvidia_b200.yaml")
    assert profile.peak_hbm_bandwidth_gbps == 8000.0
    assert profile.peak_link_bandwidth_gbps["xgmi"] == 900.0
    for dtype, peak in {"bfloat16": 2250.0, "float16": 2250.0, "tfloat32": 1125.0, "float8_e4m3fn": 4500.0,
                        "int8": 4500.0}.items():
        assert profile.peak_compute_tops[dtype] == peak
