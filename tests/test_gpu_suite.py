"""End-to-end on the GPU through the reference-facing plugin API: suites with
`backend: native` run the trb_hbm / trb_mfu launchers (subprocess + JSON
contract) over libtrb_b200.so, and the records carry sane metrics."""
from __future__ import annotations

from pathlib import Path

import pytest
import yaml

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200.runner import run_suite  # noqa: E402

ROOT = Path(__file__).resolve().parent.parent
HW = ROOT / "teamredbench_b200" / "configs" / "profiles" / "hardware" / "nvidia_b200.yaml"
RT = ROOT / "teamredbench_b200" / "configs" / "profiles" / "cuda" / "cuda_generic.yaml"


def _suite(tmp_path: Path, benchmarks: list[dict]) -> Path:
    suite = tmp_path / "suite.yaml"
    suite.write_text(yaml.safe_dump({"name": "gpu-suite", "device": {"profile": str(HW)}, "runtime": {"profile": str(RT)},
                                     "outputs": {"directory": str(tmp_path / "results"), "formats": ["json", "csv"]},
                                     "benchmarks": benchmarks}), encoding="utf-8")
    return suite


def test_native_hbm_and_mfu_through_reference_kernel_names(tmp_path):
    summary = run_suite(_suite(tmp_path, [
        {"benchmark": "hbm", "params": {"backend": "native", "dtypes": ["float32", "bfloat16", "float16", "float64",
                                                                        "int8"],
                                        "modes": ["copy", "scale", "triad"], "size_mib": 512, "scale": 3.0,
                                        "warmup": 2, "iterations": 5, "native": {"kernel": "hbm_hip"}}},
        {"benchmark": "mfu", "params": {"backend": "native", "dtypes": ["bfloat16", "float16", "tfloat32",
                                                                        "float8_e4m3fn", "int8", "float32",
                                                                        "float64"],
                                        "shapes": [[2048, 2048, 2048]], "warmup": 2, "iterations": 5,
                                        "native": {"kernel": "mfu_hipblas"}}}]))
    by_key = {(r.benchmark, r.case, r.dtype): r for r in summary.records}
    for dtype in ("float32", "bfloat16", "float16", "float64"):
        for mode in ("copy", "scale", "triad"):
            r = by_key[("hbm", f"{mode}_512MiB", dtype)]
            assert r.status == "ok", r.error
            assert 1000 < r.metrics["hbm_bandwidth_gbps"] < 9000, r.metrics
            assert r.metadata["backend_library"] == "libtrb_b200"
    assert by_key[("hbm", "copy_512MiB", "int8")].status == "ok"
    assert by_key[("hbm", "triad_512MiB", "int8")].status == "skipped"
    for dtype in ("bfloat16", "float16", "tfloat32", "float8_e4m3fn", "int8", "float32", "float64"):
        r = by_key[("mfu", "gemm_2048x2048x2048", dtype)]
        assert r.status == "ok", r.error
        assert r.metrics["achieved_tops"] > (5 if dtype == "float64" else 50) and 0 < r.metrics["mfu_pct"] < 100
        assert r.metadata["device_error"] == 0
    assert summary.outputs["csv"].exists()


def test_torch_backend_runs(tmp_path):
    summary = run_suite(_suite(tmp_path, [
        {"benchmark": "hbm", "params": {"backend": "torch", "dtypes": ["float32"], "modes": ["triad"], "size_mib": 256,
                                        "scale": 3.0, "warmup": 1, "iterations": 3, "seed": 0}},
        {"benchmark": "mfu", "params": {"backend": "torch", "dtypes": ["bfloat16", "tfloat32", "int8",
                                                                       "float8_e4m3fn"],
                                        "shapes": [[1024, 1024, 1024]], "warmup": 1, "iterations": 3, "seed": 0}}]))
    assert all(r.status == "ok" for r in summary.records), [(r.case, r.dtype, r.error) for r in summary.records]
