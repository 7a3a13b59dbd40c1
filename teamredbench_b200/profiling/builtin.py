"""Built-in profiler engine: NVIDIA Nsight Compute (`ncu`).

Replaces the reference's rocprof engine (src/teamredbench/profiling/builtin.py:
37-150).  The engine wraps the whole suite run; since every native case is a
child process, `--target-processes all` is on.  Defaults keep a capture small
and safe on shared GPUs: `--clock-control none` is ALWAYS passed (ncu would
otherwise lock the GPU clocks), and the default metric list is the
one-pass `gpu__time_duration.sum` launch list.

params:
  binary            ncu executable (default: ncu on PATH / /usr/local/cuda/bin/ncu)
  metrics           list of metric names (default [gpu__time_duration.sum])
  sections          list of section names (e.g. SpeedOfLight, MemoryWorkloadAnalysis)
  set               section set name (e.g. full)
  kernel_name       -k filter (e.g. "regex:gemm_tcgen05")
  launch_skip       -s N
  launch_count      -c N
  csv               true -> text CSV log (ncu.csv) instead of an .ncu-rep report
  extra_args        list of extra ncu arguments
  env               mapping of extra environment variables
"""
from __future__ import annotations

import shutil
from pathlib import Path
from typing import Any

from teamredbench_b200.profiling.registry import ProfilingLaunch, register_profile_engine


def _ncu_binary(value: str) -> str:
    if Path(value).is_absolute():
        return value
    return shutil.which(value) or (str(Path("/usr/local/cuda/bin") / value)
                                   if (Path("/usr/local/cuda/bin") / value).exists() else value)


def build_ncu_command(params: dict[str, Any], target_command: list[str], artifact_dir: Path,
                      base_dir: Path | None) -> ProfilingLaunch:
    artifact_dir.mkdir(parents=True, exist_ok=True)
    binary = _ncu_binary(str(params.get("binary", "ncu")))
    command: list[str] = [binary, "--clock-control", "none", "--target-processes", "all"]
    if params.get("set"):
        command += ["--set", str(params["set"])]
    for section in params.get("sections") or []:
        command += ["--section", str(section)]
    metrics = params.get("metrics")
    if metrics is None and not params.get("set") and not params.get("sections"):
        metrics = ["gpu__time_duration.sum"]
    if metrics:
        command += ["--metrics", ",".join(str(m) for m in metrics)]
    if params.get("kernel_name"):
        command += ["-k", str(params["kernel_name"])]
    if params.get("launch_skip") is not None:
        command += ["-s", str(int(params["launch_skip"]))]
    if params.get("launch_count") is not None:
        command += ["-c", str(int(params["launch_count"]))]
    if params.get("csv", True):
        output = artifact_dir / "ncu.csv"
        command += ["--csv", "--log-file", str(output)]
    else:
        output = artifact_dir / "profile"
        command += ["-o", str(output)]
    extra = params.get("extra_args") or []
    if not isinstance(extra, list):
        raise ValueError("profiling.params.extra_args must be a list of strings.")
    if any(str(a) == "--clock-control" for a in extra):
        raise ValueError("profiling.params.extra_args must not override --clock-control (always 'none').")
    command += [str(a) for a in extra]
    env = {str(k): str(v) for k, v in (params.get("env") or {}).items()}
    command += list(target_command)
    return ProfilingLaunch(command=tuple(command), artifact_dir=artifact_dir, env=env,
                           metadata={"binary": binary, "output": str(output), "clock_control": "none"})


register_profile_engine(name="ncu", description="Profile a TeamRedBench run with NVIDIA Nsight Compute (ncu).",
                        build_command=build_ncu_command)
