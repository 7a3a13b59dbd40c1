"""Run provenance written into every *.metadata.json (reference:
src/teamredbench/provenance.py:249-306), with NVIDIA probes (nvidia-smi,
nvcc, driver) in place of the ROCm ones."""
from __future__ import annotations

import os
import platform
import shlex
import socket
import subprocess
import sys
from dataclasses import asdict
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

from teamredbench_b200 import __version__
from teamredbench_b200.benchmarks.base import BenchmarkContext
from teamredbench_b200.config import SuiteConfig
from teamredbench_b200.device import detect_runtime

_ENV_NAMES = {"CUDA_VISIBLE_DEVICES", "LD_LIBRARY_PATH", "LOCAL_RANK", "MASTER_ADDR", "MASTER_PORT",
              "OMP_NUM_THREADS", "PATH", "PYTHONPATH", "RANK", "VIRTUAL_ENV", "WORLD_SIZE", "LOCAL_WORLD_SIZE"}
_ENV_PREFIXES = ("CUDA_", "NCCL_", "NVIDIA_", "PYTORCH_", "TORCH_", "SLURM_", "TEAMREDBENCH_", "UCX_")


def _command(cmd: list[str]) -> str | None:
    try:
        done = subprocess.run(cmd, check=False, capture_output=True, text=True, timeout=10)
    except (OSError, subprocess.TimeoutExpired):
        return None
    return done.stdout.strip() or None if done.returncode == 0 else None


def _stamp(value: datetime) -> str:
    return value.astimezone(timezone.utc).isoformat().replace("+00:00", "Z")


def _git(repo_root: Path | None) -> dict[str, Any]:
    if repo_root is None:
        return {}
    top = _command(["git", "-C", str(repo_root), "rev-parse", "--show-toplevel"])
    if not top:
        return {}
    status = _command(["git", "-C", top, "status", "--short"])
    return {"commit": _command(["git", "-C", top, "rev-parse", "HEAD"]),
            "branch": _command(["git", "-C", top, "rev-parse", "--abbrev-ref", "HEAD"]),
            "dirty": bool(status), "status_short": status}


def _config(path: Path | None, raw: dict[str, Any]) -> dict[str, Any]:
    content = None
    if path is not None and path.exists():
        try:
            content = path.read_text(encoding="utf-8")
        except OSError:
            content = None
    return {"path": str(path) if path else None, "raw": raw, "content": content}


def build_run_metadata(*, suite: SuiteConfig, context: BenchmarkContext, requested_device_id: int,
                       output_dir: Path, output_formats: list[str], profile_note: str | None,
                       started_at: datetime, finished_at: datetime) -> dict[str, Any]:
    torch = context.torch_module
    run_cmd = ["python", "-m", "teamredbench_b200", "run"] + ([str(suite.path)] if suite.path else []) + [
        "--device-id", str(requested_device_id), "--output-dir", str(output_dir)]
    uname = platform.uname()
    return {
        "tool": {"name": "teamredbench_b200", "version": __version__},
        "timestamps": {"started_at_utc": _stamp(started_at), "finished_at_utc": _stamp(finished_at),
                       "duration_s": max((finished_at - started_at).total_seconds(), 0.0)},
        "invocation": {"argv": list(sys.argv), "shell_command": shlex.join(sys.argv), "working_directory": os.getcwd(),
                       "requested_device_id": requested_device_id, "resolved_device_id": context.device_id,
                       "rank": context.rank, "world_size": context.world_size, "output_dir": str(output_dir)},
        "reproduce": {"run_command": shlex.join(run_cmd)},
        "system": {"hostname": socket.gethostname(), "platform": platform.platform(), "machine": uname.machine,
                   "processor": uname.processor, "cpu_count": os.cpu_count()},
        "python": {"executable": sys.executable, "version": platform.python_version()},
        "torch": {} if torch is None else {"version": getattr(torch, "__version__", None),
                                           "cuda_version": getattr(getattr(torch, "version", None), "cuda", None)},
        "cuda": {"profile_name": context.runtime_profile.name,
                 "profile_cuda_version": context.runtime_profile.cuda_version,
                 "profile_libraries": dict(context.runtime_profile.libraries),
                 **detect_runtime(torch)},
        "device": asdict(context.device_info) if context.device_info is not None else None,
        "environment": {"variables": {k: v for k, v in sorted(os.environ.items())
                                      if k in _ENV_NAMES or k.startswith(_ENV_PREFIXES)}},
        "git": _git(context.repo_root),
        "configs": {"suite": _config(suite.path, suite.raw),
                    "hardware_profile": _config(context.hardware_profile.path, context.hardware_profile.raw),
                    "runtime_profile": _config(context.runtime_profile.path, context.runtime_profile.raw),
                    "profile_note": profile_note, "profiling": dict(suite.profiling.raw),
                    "plugins": list(suite.plugins), "output_formats": list(output_formats)},
    }
