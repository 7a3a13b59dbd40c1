import json
from pathlib import Path

import yaml

from teamredbench_b200.benchmarks.base import Benchmark, BenchmarkRecord
from teamredbench_b200.registry import register_benchmark
from teamredbench_b200.runner import run_suite


@register_benchmark("test_dummy_callback")
class DummyCallbackBenchmark(Benchmark):
    default_metrics = ["latency_us", "mfu_pct"]

    def run(self) -> list[BenchmarkRecord]:
        return [self.emit_record(BenchmarkRecord(benchmark=self.name, case="single", dtype="float32",
                                                 raw_metrics={"elapsed_s": 0.001, "achieved_ops": 1e9}))]


def _write_suite(tmp_path: Path, extra: dict | None = None) -> Path:
    hardware, runtime, suite = tmp_path / "hardware.yaml", tmp_path / "runtime.yaml", tmp_path / "suite.yaml"
    hardware.write_text(yaml.safe_dump({"name": "test-hw", "family": "blackwell", "peak_hbm_bandwidth_gbps": 1,
                                        "peak_link_bandwidth_gbps": {"xgmi": 1, "network": 1},
                                        "peak_compute_tops": {"float32": 1}}), encoding="utf-8")
    runtime.write_text(yaml.safe_dump({"name": "test-runtime", "cuda_version": "test", "libraries": {},
                                       "env": {"TRB_TEST_RUNTIME_ENV": "applied"}}), encoding="utf-8")
    body = {"name": "callback-suite", "device": {"profile": str(hardware)}, "runtime": {"profile": str(runtime)},
            "outputs": {"directory": str(tmp_path / "results"), "formats": ["json", "csv"]},
            "benchmarks": [{"benchmark": "test_dummy_callback"}]}
    body.update(extra or {})
    suite.write_text(yaml.safe_dump(body), encoding="utf-8")
    return suite


def test_run_suite_invokes_record_callback_with_metrics(tmp_path: Path, monkeypatch):
    monkeypatch.delenv("TRB_TEST_RUNTIME_ENV", raising=False)
    seen: list[BenchmarkRecord] = []
    summary = run_suite(_write_suite(tmp_path), record_callback=seen.append)
    assert len(summary.records) == 1 and len(seen) == 1
    assert seen[0].metrics["latency_us"] == 1000.0
    assert seen[0].metrics["mfu_pct"] is None
    for key in ("json", "csv", "metadata"):
        assert summary.outputs[key].exists()
    records = json.loads(summary.outputs["json"].read_text(encoding="utf-8"))
    meta = json.loads(summary.outputs["metadata"].read_text(encoding="utf-8"))
    assert records[0]["benchmark"] == "test_dummy_callback"
    assert meta["record_count"] == 1
    assert meta["outputs"]["json"] == str(summary.outputs["json"])
    assert meta["run"]["configs"]["suite"]["raw"]["name"] == "callback-suite"
    assert meta["run"]["configs"]["hardware_profile"]["raw"]["name"] == "test-hw"
    assert meta["run"]["configs"]["runtime_profile"]["raw"]["name"] == "test-runtime"
    assert meta["run"]["python"]["version"]
    assert meta["run"]["reproduce"]["run_command"]
    import os

    assert os.environ["TRB_TEST_RUNTIME_ENV"] == "applied"


def test_same_second_runs_do_not_overwrite(tmp_path: Path):
    suite = _write_suite(tmp_path)
    a = run_suite(suite)
    b = run_suite(suite)
    assert a.outputs["json"] != b.outputs["json"]
    assert a.outputs["json"].exists() and b.outputs["json"].exists()
