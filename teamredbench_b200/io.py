"""Result files: records JSON, flattened CSV and a metadata JSON
(reference: src/teamredbench/io.py:42-87).  A numeric suffix is added when a
file of the same name exists, so that runs started in the same second (for
example one per rank) never overwrite each other."""
from __future__ import annotations

import csv
import json
from datetime import datetime, timezone
from pathlib import Path
from typing import Iterable

from teamredbench_b200.benchmarks.base import BenchmarkRecord


def serialize_record(record: BenchmarkRecord) -> dict[str, object]:
    return {"benchmark": record.benchmark, "case": record.case, "dtype": record.dtype, "status": record.status,
            "error": record.error, "metrics": record.metrics, "raw_metrics": record.raw_metrics,
            "metadata": record.metadata}


def flatten_record(record: BenchmarkRecord) -> dict[str, object]:
    row: dict[str, object] = {"benchmark": record.benchmark, "case": record.case, "dtype": record.dtype,
                              "status": record.status, "error": record.error or ""}
    for prefix, table in (("metric", record.metrics), ("raw", record.raw_metrics), ("meta", record.metadata)):
        for key in sorted(table):
            row[f"{prefix}_{key}"] = table[key]
    return row


def _unique_stem(output_dir: Path, stem: str) -> str:
    candidate, n = stem, 1
    while any((output_dir / f"{candidate}{ext}").exists() for ext in (".json", ".csv", ".metadata.json")):
        candidate = f"{stem}-{n}"
        n += 1
    return candidate


def write_results(records: Iterable[BenchmarkRecord], suite_name: str, output_dir: Path, formats: list[str],
                  run_metadata: dict[str, object] | None = None, tag: str | None = None) -> dict[str, Path]:
    records = list(records)
    output_dir.mkdir(parents=True, exist_ok=True)
    stamp = datetime.now(timezone.utc).strftime("%Y%m%dT%H%M%SZ")
    stem = _unique_stem(output_dir, f"{suite_name}-{stamp}" + (f"-{tag}" if tag else ""))
    outputs: dict[str, Path] = {}
    if "json" in formats:
        path = output_dir / f"{stem}.json"
        path.write_text(json.dumps([serialize_record(r) for r in records], indent=2), encoding="utf-8")
        outputs["json"] = path
    if "csv" in formats:
        path = output_dir / f"{stem}.csv"
        rows = [flatten_record(r) for r in records]
        with path.open("w", encoding="utf-8", newline="") as handle:
            writer = csv.DictWriter(handle, fieldnames=sorted({k for row in rows for k in row}))
            writer.writeheader()
            writer.writerows(rows)
        outputs["csv"] = path
    meta_path = output_dir / f"{stem}.metadata.json"
    outputs["metadata"] = meta_path
    counts: dict[str, int] = {}
    for r in records:
        counts[r.status] = counts.get(r.status, 0) + 1
    meta_path.write_text(json.dumps({
        "schema_version": 1,
        "suite_name": suite_name,
        "generated_at_utc": datetime.now(timezone.utc).isoformat().replace("+00:00", "Z"),
        "record_count": len(records),
        "record_status_counts": counts,
        "outputs": {name: str(p) for name, p in outputs.items()},
        "run": run_metadata or {},
    }, indent=2), encoding="utf-8")
    return outputs
