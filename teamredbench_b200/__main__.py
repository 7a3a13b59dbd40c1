"""`python -m teamredbench_b200 run <suite.yaml>` -- the entry the profiler
engines re-execute (reference: src/teamredbench/cli.py:85-107), plus listing
commands.  Output: one line per record, then the written file paths."""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path


def _format_record(record) -> str:
    head = f"[{record.status.upper()}] {record.benchmark} case={record.case} dtype={record.dtype}"
    if record.status != "ok":
        return f"{head} error={record.error}"
    values = record.metrics or record.raw_metrics
    parts = []
    for name, value in sorted(values.items()):
        text = "n/a" if value is None else (f"{value:.6g}" if isinstance(value, float) else str(value))
        parts.append(f"{name}={text}{'%' if name.endswith('_pct') and value is not None else ''}")
    return f"{head} {', '.join(parts)}".rstrip()


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(prog="teamredbench_b200")
    sub = parser.add_subparsers(dest="command", required=True)
    run = sub.add_parser("run")
    run.add_argument("suite", type=Path)
    run.add_argument("--output-dir", type=Path, default=None)
    run.add_argument("--device-id", type=int, default=0)
    run.add_argument("--quiet-records", action="store_true")
    for name in ("list-benchmarks", "list-metrics", "list-native-kernels", "list-profile-engines", "list-dtypes"):
        sub.add_parser(name)
    args = parser.parse_args(argv)

    from teamredbench_b200 import builtin  # noqa: F401
    from teamredbench_b200 import registry
    from teamredbench_b200.native.registry import list_native_kernels
    from teamredbench_b200.profiling.registry import list_profile_engines

    if args.command == "run":
        from teamredbench_b200.profiling.runtime import profiling_active
        from teamredbench_b200.runner import run_suite

        summary = run_suite(args.suite, output_dir=args.output_dir, device_id=args.device_id,
                            record_callback=None if args.quiet_records else (lambda r: print(_format_record(r))))
        if profiling_active() or os.environ.get("TEAMREDBENCH_SUPPRESS_CLI_OUTPUT") == "1":
            return 0
        print(f"Suite: {summary.suite.name}")
        print(f"Hardware Profile: {summary.context.hardware_profile.name}")
        if summary.profile_note:
            print(summary.profile_note)
        print(f"Records: {len(summary.records)}")
        for fmt, path in summary.outputs.items():
            print(f"{fmt.upper()}: {path}")
    elif args.command == "list-benchmarks":
        print("\n".join(registry.list_benchmarks()))
    elif args.command == "list-metrics":
        print("\n".join(registry.list_metrics()))
    elif args.command == "list-native-kernels":
        print("\n".join(f"{d.name} [{d.benchmark}]" for d in list_native_kernels()))
    elif args.command == "list-profile-engines":
        print("\n".join(f"{d.name}: {d.description}" for d in list_profile_engines()))
    elif args.command == "list-dtypes":
        from teamredbench_b200.device import load_torch
        from teamredbench_b200.dtypes import discover_dtypes

        print("\n".join(sorted(discover_dtypes(load_torch()))))
    return 0


if __name__ == "__main__":
    sys.exit(main())
