"""Suite runner (reference: src/teamredbench/runner.py:31-178).

load suite -> load plugins -> build context -> run each benchmark (records
pass through the metric registry as they are emitted) -> provenance -> write.

Multi-GPU (one process per GPU under torchrun): LOCAL_RANK picks the device as
in the reference (runner.py:93).  Added here: the runtime profile's `env` is
applied before any benchmark runs; a process group is created
(`cpu:gloo,cuda:nccl`, or `gloo` without CUDA) when WORLD_SIZE > 1;
benchmarks barrier before each timed case so the replicas' timed windows
overlap; afterwards all records are gathered to rank 0, which adds one
"box" aggregate per (benchmark, case, dtype) and alone writes the result
files.  For replicated benchmarks (hbm, mfu, ...) the aggregate sums bytes /
ops over ranks and divides by the MAX device-timed elapsed_s over ranks; for
`collective` it keeps the payload and takes the max elapsed_s.
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass, replace
from datetime import datetime, timedelta, timezone
from pathlib import Path
from typing import Any, Callable

from teamredbench_b200 import builtin as _builtin  # noqa: F401
from teamredbench_b200.benchmarks.base import BenchmarkContext, BenchmarkRecord
from teamredbench_b200.config import HardwareProfile, SuiteConfig, load_hardware_profile, load_suite
from teamredbench_b200.device import detect_device, load_torch
from teamredbench_b200.dtypes import discover_dtypes
from teamredbench_b200.io import write_results
from teamredbench_b200.profiling.runtime import effective_output_formats, profiling_enabled, run_profiled_suite
from teamredbench_b200.provenance import build_run_metadata
from teamredbench_b200.registry import get_benchmark, get_metric, load_plugins

# Benchmarks whose per-rank work is independent (weak scaling): aggregate = sum / max time.
REPLICATED_SUM_KEYS = ("moved_bytes", "achieved_ops")
REPLICATED_PEAK_KEYS = ("peak_bandwidth_gbps", "peak_tops")


@dataclass
class RunSummary:
    suite: SuiteConfig
    context: BenchmarkContext
    records: list[BenchmarkRecord]
    outputs: dict[str, Path]
    run_metadata: dict[str, object]
    profile_note: str | None = None


def _apply_metrics(record: BenchmarkRecord, metric_names: list[str]) -> None:
    if record.status != "ok":
        return
    for name in metric_names:
        record.metrics[name] = get_metric(name).compute(record.raw_metrics)


# ---------------------------------------------------------------- SKU auto-profile
_SKU_PATTERN = re.compile(r"mi\d{3,4}x|\bb200\b|\bb300\b|\bgb200\b|\bh100\b|\bh200\b", re.IGNORECASE)


def _extract_sku_tokens(text: str | None) -> set[str]:
    if not text:
        return set()
    return {token.lower() for token in _SKU_PATTERN.findall(text.replace("_", " ").replace("-", " "))}


def _has_limits(profile: HardwareProfile) -> bool:
    return (profile.peak_hbm_bandwidth_gbps is not None and float(profile.peak_hbm_bandwidth_gbps) > 0
            and any(v is not None and float(v) > 0 for v in profile.peak_compute_tops.values()))


def _resolve_hardware_profile(profile: HardwareProfile, *, device_name: str | None,
                              repo_root: Path | None) -> tuple[HardwareProfile, str | None]:
    """A placeholder profile (no peaks) is swapped for the published profile
    whose SKU token matches the detected device (reference runner.py:57-89)."""
    if _has_limits(profile) or repo_root is None:
        return profile, None
    tokens = _extract_sku_tokens(device_name)
    hw_dir = repo_root / "configs" / "profiles" / "hardware"
    if not tokens or not hw_dir.exists():
        return profile, None
    for path in sorted(hw_dir.glob("*.yaml")):
        candidate = load_hardware_profile(path)
        if _extract_sku_tokens(f"{candidate.name} {path.stem}") & tokens and _has_limits(candidate):
            return candidate, (f"Auto-selected hardware profile {candidate.name} from detected device "
                               f"{device_name!r} because {profile.name} has no theoretical peak data.")
    return profile, None


def build_context(suite: SuiteConfig, device_id: int = 0) -> tuple[BenchmarkContext, str | None]:
    resolved = int(os.environ.get("LOCAL_RANK", device_id))
    torch_module = load_torch()
    device_info = detect_device(torch_module, device_id=resolved)
    repo_root = suite.path.parent.parent.parent if suite.path else None
    hardware, note = _resolve_hardware_profile(suite.hardware_profile,
                                               device_name=device_info.name if device_info else None,
                                               repo_root=repo_root)
    return BenchmarkContext(hardware_profile=hardware, runtime_profile=suite.runtime_profile,
                            device_info=device_info, torch_module=torch_module,
                            dtype_specs=discover_dtypes(torch_module), device_id=resolved, repo_root=repo_root,
                            suite_path=suite.path, rank=int(os.environ.get("RANK", 0)),
                            world_size=int(os.environ.get("WORLD_SIZE", 1))), note


# ---------------------------------------------------------------- multi-rank
def ensure_process_group(context: BenchmarkContext, suite: SuiteConfig):
    """Default process group for replica sync / aggregation (WORLD_SIZE > 1)."""
    if context.world_size <= 1 or context.torch_module is None:
        return None
    dist = context.torch_module.distributed
    if not dist.is_available():
        return None
    if not dist.is_initialized():
        has_cuda = bool(context.torch_module.cuda.is_available())
        backend = suite.distributed.get("backend") or ("cpu:gloo,cuda:nccl" if has_cuda else "gloo")
        kwargs: dict[str, Any] = {"backend": backend, "init_method": "env://",
                                  "timeout": timedelta(seconds=float(suite.distributed.get("timeout_s", 600)))}
        dist.init_process_group(**kwargs)
    return dist


def aggregate_records(per_rank: list[list[BenchmarkRecord]], metric_names: dict[str, list[str]]
                      ) -> list[BenchmarkRecord]:
    """Per-rank records (tagged with their rank) followed by one box aggregate
    per (benchmark, case, dtype) that every rank reported as ok."""
    world = len(per_rank)
    out: list[BenchmarkRecord] = []
    for rank, records in enumerate(per_rank):
        for r in records:
            out.append(replace(r, metadata={**r.metadata, "rank": rank}, metrics=dict(r.metrics)))
    keys = [(r.benchmark, r.case, r.dtype) for r in per_rank[0]]
    index = [{(r.benchmark, r.case, r.dtype): r for r in records} for records in per_rank]
    for key in keys:
        group = [table.get(key) for table in index]
        if any(r is None or r.status != "ok" or r.raw_metrics.get("elapsed_s") is None for r in group):
            continue
        first = group[0]
        elapsed = [float(r.raw_metrics["elapsed_s"]) for r in group]
        raw = dict(first.raw_metrics)
        raw["elapsed_s"] = max(elapsed)
        if first.benchmark != "collective":
            for k in REPLICATED_SUM_KEYS:
                if k in raw and all(r.raw_metrics.get(k) is not None for r in group):
                    raw[k] = sum(float(r.raw_metrics[k]) for r in group)
            for k in REPLICATED_PEAK_KEYS:
                if raw.get(k) is not None:
                    raw[k] = float(raw[k]) * world
        agg = BenchmarkRecord(benchmark=first.benchmark, case=first.case, dtype=first.dtype, raw_metrics=raw,
                              metadata={**first.metadata, "aggregate": "box", "world_size": world,
                                        "per_rank_elapsed_s": elapsed,
                                        "scaling": "replicated" if first.benchmark != "collective" else "collective"})
        _apply_metrics(agg, metric_names.get(first.benchmark, []))
        out.append(agg)
    return out


def _gather_records(dist, records: list[BenchmarkRecord], world: int) -> list[list[BenchmarkRecord]]:
    gathered: list[Any] = [None] * world
    dist.all_gather_object(gathered, records)
    return gathered


# ---------------------------------------------------------------- run
def run_suite(suite_path: str | Path, output_dir: str | Path | None = None, device_id: int = 0,
              record_callback: Callable[[BenchmarkRecord], None] | None = None) -> RunSummary:
    started = datetime.now(timezone.utc)
    suite = load_suite(suite_path)
    for key, value in suite.runtime_profile.env.items():
        os.environ.setdefault(key, value)
    load_plugins(suite.plugins)
    target = Path(output_dir).resolve() if output_dir else suite.outputs.directory
    context, note = build_context(suite, device_id=device_id)
    suite.hardware_profile = context.hardware_profile
    if profiling_enabled(suite.profiling):
        return run_profiled_suite(suite=suite, context=context, output_dir=target.resolve(), device_id=device_id,
                                  record_callback=record_callback)

    dist = ensure_process_group(context, suite)
    records: list[BenchmarkRecord] = []
    metric_names: dict[str, list[str]] = {}
    for invocation in suite.benchmarks:
        cls = get_benchmark(invocation.benchmark)
        names = invocation.metrics or list(cls.default_metrics)
        metric_names[invocation.benchmark] = names

        def sink(record: BenchmarkRecord, names: list[str] = names) -> None:
            _apply_metrics(record, names)
            if record_callback is not None:
                record_callback(record)

        records.extend(cls(context=context, params=invocation.params, record_sink=sink).run())

    write_here = True
    if dist is not None and context.world_size > 1:
        per_rank = _gather_records(dist, records, context.world_size)
        write_here = context.rank == 0
        if write_here:
            records = aggregate_records(per_rank, metric_names)

    finished = datetime.now(timezone.utc)
    formats = effective_output_formats(suite.outputs.formats)
    metadata = build_run_metadata(suite=suite, context=context, requested_device_id=device_id,
                                  output_dir=target.resolve(), output_formats=formats, profile_note=note,
                                  started_at=started, finished_at=finished)
    outputs: dict[str, Path] = {}
    if write_here:
        outputs = write_results(records=records, suite_name=suite.name, output_dir=target.resolve(),
                                formats=formats, run_metadata=metadata)
    return RunSummary(suite=suite, context=context, records=records, outputs=outputs, run_metadata=metadata,
                      profile_note=note)
