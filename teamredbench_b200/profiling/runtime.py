"""Profiled suite runs: re-run the whole suite as a child process under the
selected engine and merge its results (reference:
src/teamredbench/profiling/runtime.py:24-184)."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

from teamredbench_b200.benchmarks.base import BenchmarkContext, BenchmarkRecord
from teamredbench_b200.config import ProfilingConfig, SuiteConfig
from teamredbench_b200.profiling.registry import get_profile_engine

INTERNAL_RUN_ENV = "TEAMREDBENCH_INTERNAL_RUN"
FORCE_JSON_OUTPUT_ENV = "TEAMREDBENCH_FORCE_JSON_OUTPUT"


class ProfilingError(RuntimeError):
    pass


def profiling_active() -> bool:
    return os.environ.get(INTERNAL_RUN_ENV) == "1"


def profiling_enabled(config: ProfilingConfig) -> bool:
    return bool(config.enabled and config.engine and not profiling_active())


def force_json_output_enabled() -> bool:
    return os.environ.get(FORCE_JSON_OUTPUT_ENV) == "1"


def effective_output_formats(formats: list[str]) -> list[str]:
    out = list(formats)
    if force_json_output_enabled() and "json" not in out:
        out.append("json")
    return out


def _record_from_json(payload: dict[str, Any]) -> BenchmarkRecord:
    return BenchmarkRecord(
        benchmark=str(payload["benchmark"]), case=str(payload["case"]), dtype=str(payload["dtype"]),
        status=str(payload.get("status", "ok")),
        error=str(payload["error"]) if payload.get("error") is not None else None,
        metrics=dict(payload.get("metrics", {})), raw_metrics=dict(payload.get("raw_metrics", {})),
        metadata=dict(payload.get("metadata", {})))


def run_profiled_suite(*, suite: SuiteConfig, context: BenchmarkContext, output_dir: Path, device_id: int,
                       record_callback):
    from teamredbench_b200.runner import RunSummary

    if suite.path is None:
        raise ProfilingError("Suite path is required for profiled runs.")
    if not suite.profiling.engine:
        raise ProfilingError("Profiling is enabled but no engine is configured.")
    engine = get_profile_engine(suite.profiling.engine)
    stamp = datetime.now(timezone.utc).strftime("%Y%m%dT%H%M%SZ")
    artifact_dir = output_dir / "profiling" / f"{suite.name}-{engine.name}-{stamp}"
    child = [sys.executable, "-m", "teamredbench_b200", "run", str(suite.path), "--device-id", str(device_id),
             "--output-dir", str(output_dir), "--quiet-records"]
    launch = engine.build_command(dict(suite.profiling.params), child, artifact_dir, suite.path.parent)
    env = {**os.environ, INTERNAL_RUN_ENV: "1", FORCE_JSON_OUTPUT_ENV: "1", **launch.env}
    before = set(output_dir.glob(f"{suite.name}-*.metadata.json")) if output_dir.exists() else set()
    completed = subprocess.run(list(launch.command), check=False, capture_output=True, text=True, env=env)
    if completed.returncode != 0:
        error = completed.stderr.strip() or completed.stdout.strip() or "unknown profiling failure"
        raise ProfilingError(f"Profile engine {engine.name} failed: {error}")
    new = sorted(set(output_dir.glob(f"{suite.name}-*.metadata.json")) - before)
    if not new:
        raise ProfilingError("Profiled run completed but no metadata file was produced.")
    metadata_path = new[-1]
    payload = json.loads(metadata_path.read_text(encoding="utf-8"))
    outputs = {name: Path(p) for name, p in payload.get("outputs", {}).items()}
    json_path = outputs.get("json")
    if json_path is None or not json_path.exists():
        raise ProfilingError("Profiled run did not produce a JSON results file.")
    records = [_record_from_json(item) for item in json.loads(json_path.read_text(encoding="utf-8"))]
    payload.setdefault("outputs", {})["profiling"] = str(launch.artifact_dir)
    payload.setdefault("run", {})["profiling"] = {
        "enabled": True, "engine": engine.name, "artifact_dir": str(launch.artifact_dir),
        "command": list(launch.command), "engine_metadata": dict(launch.metadata)}
    metadata_path.write_text(json.dumps(payload, indent=2), encoding="utf-8")
    outputs["profiling"] = launch.artifact_dir
    run_metadata = dict(payload.get("run", {}))
    if record_callback is not None:
        for record in records:
            record_callback(record)
    return RunSummary(suite=suite, context=context, records=records, outputs=outputs, run_metadata=run_metadata,
                      profile_note=run_metadata.get("configs", {}).get("profile_note"))
