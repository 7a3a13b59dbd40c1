"""Native-kernel boundary tests in the reference's style (tests/test_native.py):
fake executables written as Python scripts stand in for the kernels, so the
subprocess / JSON contract, metric plumbing and cache logic run without a GPU."""
import json
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import yaml

import teamredbench_b200.builtin  # noqa: F401
import teamredbench_b200.native.runtime as native_runtime
from teamredbench_b200.native.runtime import NativeKernelError, ResolvedNativeKernel, clear_native_cache
from teamredbench_b200.runner import run_suite


def _write_executable(path: Path, contents: str) -> None:
    path.write_text(contents, encoding="utf-8")
    path.chmod(0o755)


def _profiles(tmp_path: Path, tops: dict) -> tuple[Path, Path]:
    hardware, runtime = tmp_path / "hardware.yaml", tmp_path / "runtime.yaml"
    hardware.write_text(yaml.safe_dump({"name": "test-hw", "family": "blackwell", "peak_hbm_bandwidth_gbps": 4000,
                                        "peak_link_bandwidth_gbps": {"xgmi": 1, "network": 1},
                                        "peak_compute_tops": tops}), encoding="utf-8")
    runtime.write_text(yaml.safe_dump({"name": "test-runtime", "cuda_version": "test", "libraries": {}, "env": {}}),
                       encoding="utf-8")
    return hardware, runtime


def _fake(tmp_path: Path, name: str, payload: dict) -> Path:
    seen = tmp_path / f"{name}_args.json"
    _write_executable(tmp_path / f"{name}.py", "\n".join([
        f"#!{sys.executable}", "import json, sys",
        f"open({str(seen)!r}, 'w', encoding='utf-8').write(json.dumps(sys.argv[1:]))",
        "print('some log line')",
        f"print(json.dumps({payload!r}))"]))
    return seen


def _suite(tmp_path: Path, hardware: Path, runtime: Path, bench: dict) -> Path:
    suite = tmp_path / "suite.yaml"
    suite.write_text(yaml.safe_dump({"name": "native-suite", "device": {"profile": str(hardware)},
                                     "runtime": {"profile": str(runtime)},
                                     "outputs": {"directory": str(tmp_path / "results"), "formats": ["json"]},
                                     "benchmarks": [bench]}), encoding="utf-8")
    return suite


def test_clean_native_cache_removes_entries(tmp_path: Path):
    cache = tmp_path / "native-cache"
    cache.mkdir()
    (cache / "kernel-a").write_text("a", encoding="utf-8")
    (cache / "kernel-b").mkdir()
    (cache / "kernel-b" / "payload").write_text("b", encoding="utf-8")
    cleared, removed = clear_native_cache(cache)
    assert cleared == cache and removed == 2 and list(cache.iterdir()) == []


def test_run_suite_hbm_native_backend_uses_relative_binary(tmp_path: Path):
    hardware, runtime = _profiles(tmp_path, {"float32": 100})
    seen = _fake(tmp_path, "fake_hbm", {"status": "ok", "raw_metrics": {"elapsed_s": 0.002},
                                        "metadata": {"executor": "fake"}})
    suite = _suite(tmp_path, hardware, runtime, {"benchmark": "hbm", "params": {
        "backend": "native", "dtypes": ["float32"], "modes": ["copy"], "size_mib": 1024, "warmup": 2,
        "iterations": 5, "native": {"binary": "./fake_hbm.py"}}})
    summary = run_suite(suite)
    record = summary.records[0]
    assert record.status == "ok"
    assert record.metadata["backend"] == "native" and record.metadata["executor"] == "fake"
    assert record.metrics["hbm_bandwidth_gbps"] == pytest.approx(1073.741824)
    assert record.metrics["hbm_efficiency_pct"] == pytest.approx(26.8435456)
    argv = json.loads(seen.read_text(encoding="utf-8"))
    assert argv[:6] == ["--dtype", "float32", "--mode", "copy", "--size-mib", "1024"]
    assert "--scale" in argv and "--device-id" in argv


def test_run_suite_mfu_native_backend_uses_relative_binary(tmp_path: Path):
    hardware, runtime = _profiles(tmp_path, {"float32": 20})
    seen = _fake(tmp_path, "fake_mfu", {"status": "ok", "raw_metrics": {"elapsed_s": 0.001},
                                        "metadata": {"executor": "fake"}})
    suite = _suite(tmp_path, hardware, runtime, {"benchmark": "mfu", "params": {
        "backend": "native", "dtypes": ["float32"], "shapes": [[1024, 1024, 1024]], "warmup": 2, "iterations": 5,
        "native": {"binary": "./fake_mfu.py"}}})
    record = run_suite(suite).records[0]
    assert record.status == "ok"
    assert record.metrics["achieved_tops"] == pytest.approx(2.147483648)
    assert record.metrics["mfu_pct"] == pytest.approx(10.73741824)
    argv = json.loads(seen.read_text(encoding="utf-8"))
    for flag, value in (("--m", "1024"), ("--n", "1024"), ("--k", "1024"), ("--dtype", "float32")):
        assert argv[argv.index(flag) + 1] == value


def test_skipped_status_and_failures_become_skipped_records(tmp_path: Path):
    hardware, runtime = _profiles(tmp_path, {"float32": 20})
    _fake(tmp_path, "fake_skip", {"status": "skipped", "error": "unsupported dtype"})
    _write_executable(tmp_path / "fake_crash.py", f"#!{sys.executable}\nimport sys\nsys.exit(3)\n")
    for binary, expect in (("./fake_skip.py", "unsupported dtype"), ("./fake_crash.py", "failed")):
        suite = _suite(tmp_path, hardware, runtime, {"benchmark": "hbm", "params": {
            "backend": "native", "dtypes": ["float32"], "modes": ["triad"], "native": {"binary": binary}}})
        record = run_suite(suite).records[0]
        assert record.status == "skipped" and expect in record.error


def test_native_timeout_becomes_skipped_record(tmp_path: Path):
    hardware, runtime = _profiles(tmp_path, {"float32": 20})
    _write_executable(tmp_path / "fake_hang.py", f"#!{sys.executable}\nimport time\ntime.sleep(30)\n")
    suite = _suite(tmp_path, hardware, runtime, {"benchmark": "hbm", "params": {
        "backend": "native", "dtypes": ["float32"], "modes": ["copy"],
        "native": {"binary": "./fake_hang.py", "timeout_s": 1}}})
    record = run_suite(suite).records[0]
    assert record.status == "skipped" and "timed out" in record.error


def test_prepare_native_kernel_binary_rebuilds_when_local_include_changes(tmp_path: Path, monkeypatch):
    source, include = tmp_path / "kernel.cu", tmp_path / "kernel_impl.cuh"
    source.write_text('#include "kernel_impl.cuh"\nint main() { return kValue; }\n', encoding="utf-8")
    include.write_text("static constexpr int kValue = 0;\n", encoding="utf-8")
    monkeypatch.setattr(native_runtime, "_find_cuda_compiler", lambda preferred=None: "/usr/local/cuda/bin/nvcc")
    outputs, commands = [], []

    def fake_run(command, **_):
        target = Path(command[command.index("-o") + 1])
        target.write_text("fake-binary", encoding="utf-8")
        outputs.append(target)
        commands.append(command)
        return SimpleNamespace(returncode=0, stderr="", stdout="")

    monkeypatch.setattr(native_runtime.subprocess, "run", fake_run)
    kernel = ResolvedNativeKernel(benchmark="mfu", name="unit-test-kernel", description="cache test",
                                  source_path=source, cache_dir=tmp_path / "native-cache")
    first = native_runtime.prepare_native_kernel_binary(kernel)
    assert native_runtime.prepare_native_kernel_binary(kernel) == first  # cached
    include.write_text("static constexpr int kValue = 1;\n", encoding="utf-8")
    second = native_runtime.prepare_native_kernel_binary(kernel)
    assert first != second and outputs == [first, second]
    assert "arch=compute_100a,code=sm_100a" in commands[0]


def test_missing_binary_is_an_error(tmp_path: Path):
    kernel = ResolvedNativeKernel(benchmark="hbm", name="x", description="", binary_path=tmp_path / "nope")
    with pytest.raises(NativeKernelError):
        native_runtime.prepare_native_kernel_binary(kernel)


def test_builtin_kernel_resolves_to_in_tree_launcher(tmp_path: Path):
    from teamredbench_b200._native import HBM_EXECUTABLE

    kernel = native_runtime.resolve_native_kernel(benchmark="hbm", params={}, suite_path=None, repo_root=tmp_path,
                                                  default_kernel="hbm_b200")
    assert kernel.binary_path == HBM_EXECUTABLE
    with pytest.raises(ValueError):
        native_runtime.resolve_native_kernel(benchmark="mfu", params={"native": {"kernel": "hbm_b200"}},
                                             suite_path=None, repo_root=tmp_path)
