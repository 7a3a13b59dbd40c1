import json
import os
import sys
from pathlib import Path

import yaml

from teamredbench_b200.profiling.builtin import build_ncu_command
from teamredbench_b200.runner import run_suite

ROOT = Path(__file__).resolve().parent.parent


def test_run_suite_with_profile_engine_plugin(tmp_path: Path, monkeypatch):
    plugin_dir = tmp_path / "plugins"
    plugin_dir.mkdir()
    (plugin_dir / "fake_profile_plugin_b200.py").write_text("\n".join([
        "import sys",
        "from teamredbench_b200.profiling.registry import ProfilingLaunch, register_profile_engine",
        "def build_command(params, target_command, artifact_dir, base_dir):",
        "    code = ('from pathlib import Path; import subprocess, sys; '",
        "            'artifact = Path(sys.argv[1]); artifact.mkdir(parents=True, exist_ok=True); '",
        "            \"(artifact / 'marker.txt').write_text('profile', encoding='utf-8'); \"",
        "            'raise SystemExit(subprocess.run(sys.argv[2:]).returncode)')",
        "    return ProfilingLaunch(command=(sys.executable, '-c', code, str(artifact_dir), *target_command),",
        "                           artifact_dir=artifact_dir, metadata={'wrapper': 'fake'})",
        "register_profile_engine(name='fake-profiler', description='Fake profiler for tests.',",
        "                        build_command=build_command)"]), encoding="utf-8")
    monkeypatch.syspath_prepend(str(plugin_dir))
    monkeypatch.setenv("PYTHONPATH", os.pathsep.join([str(plugin_dir), str(ROOT), os.environ.get("PYTHONPATH", "")]))
    hardware, runtime, suite = tmp_path / "hardware.yaml", tmp_path / "runtime.yaml", tmp_path / "suite.yaml"
    hardware.write_text(yaml.safe_dump({"name": "test-hw", "family": "blackwell", "peak_hbm_bandwidth_gbps": 1,
                                        "peak_link_bandwidth_gbps": {"xgmi": 1, "network": 1},
                                        "peak_compute_tops": {"float32": 1}}), encoding="utf-8")
    runtime.write_text(yaml.safe_dump({"name": "test-runtime", "cuda_version": "test"}), encoding="utf-8")
    suite.write_text(yaml.safe_dump({
        "name": "profile-suite", "device": {"profile": str(hardware)}, "runtime": {"profile": str(runtime)},
        "plugins": ["fake_profile_plugin_b200"], "profiling": {"enabled": True, "engine": "fake-profiler"},
        "outputs": {"directory": str(tmp_path / "results"), "formats": ["json", "csv"]},
        "benchmarks": [{"benchmark": "hbm", "params": {"dtypes": ["float32"], "modes": ["copy"], "size_mib": 1,
                                                       "warmup": 0, "iterations": 1}}]}), encoding="utf-8")
    summary = run_suite(suite)
    assert (summary.outputs["profiling"] / "marker.txt").exists()
    meta = json.loads(summary.outputs["metadata"].read_text(encoding="utf-8"))
    assert meta["outputs"]["profiling"] == str(summary.outputs["profiling"])
    assert meta["run"]["profiling"]["engine"] == "fake-profiler"
    assert meta["run"]["profiling"]["engine_metadata"]["wrapper"] == "fake"


def test_ncu_engine_always_disables_clock_control(tmp_path: Path):
    launch = build_ncu_command({"kernel_name": "regex:gemm", "launch_count": 3}, ["python", "x.py"], tmp_path, None)
    cmd = list(launch.command)
    assert cmd[cmd.index("--clock-control") + 1] == "none"
    assert cmd[cmd.index("--metrics") + 1] == "gpu__time_duration.sum"
    assert cmd[-2:] == ["python", "x.py"] and "-k" in cmd and "-c" in cmd
    import pytest

    with pytest.raises(ValueError):
        build_ncu_command({"extra_args": ["--clock-control", "base"]}, ["x"], tmp_path, None)
    full = list(build_ncu_command({"set": "full", "csv": False}, ["x"], tmp_path, None).command)
    assert "--set" in full and "--metrics" not in full and "-o" in full
