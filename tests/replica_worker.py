"""One rank of the CPU multi-process runner tests (run as `python -m tests.replica_worker`).

Registers a replicated dummy benchmark whose device time depends on the rank,
then runs the given suite through the real runner (gloo process group)."""
from __future__ import annotations

import json
import os
import sys

from teamredbench_b200.benchmarks.base import Benchmark, BenchmarkRecord
from teamredbench_b200.registry import register_benchmark


@register_benchmark("test_replica")
class ReplicaBenchmark(Benchmark):
    default_metrics = ["hbm_bandwidth_gbps", "hbm_efficiency_pct", "latency_us"]

    def run(self) -> list[BenchmarkRecord]:
        if self.params.get("fail_rank") == self.context.rank:
            raise RuntimeError(f"rank {self.context.rank} fails on purpose (host-side)")
        self.sync_ranks()
        return [self.emit_record(BenchmarkRecord(
            benchmark=self.name, case="triad_4096MiB", dtype="float32",
            raw_metrics={"elapsed_s": 0.001 * (self.context.rank + 1), "moved_bytes": 1e9,
                         "peak_bandwidth_gbps": 8000.0}))]


def main() -> int:
    from teamredbench_b200.runner import run_suite

    summary = run_suite(sys.argv[1])
    out = {"rank": int(os.environ["RANK"]), "outputs": {k: str(v) for k, v in summary.outputs.items()},
           "records": [[r.case, r.status, r.metadata.get("aggregate"), r.metrics.get("hbm_bandwidth_gbps"),
                        r.metrics.get("hbm_efficiency_pct"), r.raw_metrics.get("elapsed_s")] for r in summary.records]}
    print("RESULT " + json.dumps(out), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
