"""Suite / hardware-profile / runtime-profile loading (YAML).

Mirrors the reference's schema (src/teamredbench/config.py:10-150) so its
suites and profiles load unchanged.  Additions: RuntimeProfile.cuda_version
(ROCm's `rocm_version` is kept for reference profiles) and an optional
suite-level `distributed:` mapping used by the multi-rank aggregation."""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import yaml


@dataclass
class HardwareProfile:
    name: str
    family: str
    peak_hbm_bandwidth_gbps: float | None = None
    peak_link_bandwidth_gbps: dict[str, float] = field(default_factory=dict)
    peak_compute_tops: dict[str, float] = field(default_factory=dict)
    notes: list[str] = field(default_factory=list)
    path: Path | None = None
    raw: dict[str, Any] = field(default_factory=dict)


@dataclass
class RuntimeProfile:
    name: str
    rocm_version: str = "unknown"
    cuda_version: str = "unknown"
    libraries: dict[str, str] = field(default_factory=dict)
    env: dict[str, str] = field(default_factory=dict)
    notes: list[str] = field(default_factory=list)
    path: Path | None = None
    raw: dict[str, Any] = field(default_factory=dict)


@dataclass
class OutputConfig:
    directory: Path
    formats: list[str] = field(default_factory=lambda: ["json", "csv"])


@dataclass
class ProfilingConfig:
    enabled: bool = False
    engine: str | None = None
    params: dict[str, Any] = field(default_factory=dict)
    raw: dict[str, Any] = field(default_factory=dict)


@dataclass
class BenchmarkInvocation:
    benchmark: str
    params: dict[str, Any] = field(default_factory=dict)
    metrics: list[str] = field(default_factory=list)


@dataclass
class SuiteConfig:
    name: str
    benchmarks: list[BenchmarkInvocation]
    hardware_profile: HardwareProfile
    runtime_profile: RuntimeProfile
    outputs: OutputConfig
    profiling: ProfilingConfig = field(default_factory=ProfilingConfig)
    plugins: list[str] = field(default_factory=list)
    distributed: dict[str, Any] = field(default_factory=dict)
    path: Path | None = None
    raw: dict[str, Any] = field(default_factory=dict)


def _read_mapping(path: Path) -> dict[str, Any]:
    with path.open("r", encoding="utf-8") as handle:
        data = yaml.safe_load(handle) or {}
    if not isinstance(data, dict):
        raise ValueError(f"Expected mapping in {path}")
    return data


def _relative_to(base: Path, target: str) -> Path:
    candidate = Path(target)
    return candidate if candidate.is_absolute() else (base / candidate).resolve()


def load_hardware_profile(path: Path) -> HardwareProfile:
    data = _read_mapping(Path(path))
    return HardwareProfile(
        name=str(data["name"]),
        family=str(data["family"]),
        peak_hbm_bandwidth_gbps=data.get("peak_hbm_bandwidth_gbps"),
        peak_link_bandwidth_gbps=dict(data.get("peak_link_bandwidth_gbps") or {}),
        peak_compute_tops={str(k): float(v) for k, v in (data.get("peak_compute_tops") or {}).items()
                           if v is not None},
        notes=list(data.get("notes") or []),
        path=Path(path),
        raw=data,
    )


def load_runtime_profile(path: Path) -> RuntimeProfile:
    data = _read_mapping(Path(path))
    return RuntimeProfile(
        name=str(data["name"]),
        rocm_version=str(data.get("rocm_version", "unknown")),
        cuda_version=str(data.get("cuda_version", "unknown")),
        libraries={str(k): str(v) for k, v in (data.get("libraries") or {}).items()},
        env={str(k): str(v) for k, v in (data.get("env") or {}).items()},
        notes=list(data.get("notes") or []),
        path=Path(path),
        raw=data,
    )


def load_suite(path: str | Path) -> SuiteConfig:
    suite_path = Path(path).resolve()
    data = _read_mapping(suite_path)
    base = suite_path.parent
    profiling = data.get("profiling") or {}
    if not isinstance(profiling, dict):
        raise ValueError(f"Expected mapping for profiling config in {suite_path}")
    outputs = data.get("outputs") or {}
    return SuiteConfig(
        name=str(data.get("name", suite_path.stem)),
        benchmarks=[
            BenchmarkInvocation(benchmark=str(item["benchmark"]), params=dict(item.get("params") or {}),
                                metrics=list(item.get("metrics") or []))
            for item in data.get("benchmarks") or []
        ],
        hardware_profile=load_hardware_profile(_relative_to(base, str(data["device"]["profile"]))),
        runtime_profile=load_runtime_profile(_relative_to(base, str(data["runtime"]["profile"]))),
        outputs=OutputConfig(directory=_relative_to(base, str(outputs.get("directory", "../../results"))),
                             formats=list(outputs.get("formats", ["json", "csv"]))),
        profiling=ProfilingConfig(enabled=bool(profiling.get("enabled", bool(profiling.get("engine")))),
                                  engine=str(profiling["engine"]) if profiling.get("engine") is not None else None,
                                  params=dict(profiling.get("params") or {}), raw=dict(profiling)),
        plugins=list(data.get("plugins") or []),
        distributed=dict(data.get("distributed") or {}),
        path=suite_path,
        raw=data,
    )
