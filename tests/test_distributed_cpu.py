"""Multi-rank runner logic on CPU: world_size-2 gloo process groups, one
subprocess per rank (no GPU).  Covers the replica barrier, the rank-0 box
aggregate (sum of bytes / max device time), single-writer output, and a rank
that fails on the host making the other rank error out (bounded by the
process-group timeout) instead of hanging."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import yaml

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _suite(tmp_path: Path, params: dict) -> Path:
    hardware, runtime, suite = tmp_path / "hw.yaml", tmp_path / "rt.yaml", tmp_path / "suite.yaml"
    hardware.write_text(yaml.safe_dump({"name": "test-hw", "family": "blackwell", "peak_hbm_bandwidth_gbps": 8000.0,
                                        "peak_compute_tops": {"float32": 1}}), encoding="utf-8")
    runtime.write_text(yaml.safe_dump({"name": "rt"}), encoding="utf-8")
    suite.write_text(yaml.safe_dump({
        "name": "replicas", "device": {"profile": str(hardware)}, "runtime": {"profile": str(runtime)},
        "plugins": ["tests.replica_worker"], "distributed": {"backend": "gloo", "timeout_s": 8},
        "outputs": {"directory": str(tmp_path / "results"), "formats": ["json"]},
        "benchmarks": [{"benchmark": "test_replica", "params": params}]}), encoding="utf-8")
    return suite


def _launch(suite: Path, world: int = 2, timeout: float = 120):
    port = _free_port()
    procs = []
    for rank in range(world):
        env = {**os.environ, "RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
               "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": "",
               "PYTHONPATH": str(ROOT)}
        procs.append(subprocess.Popen([sys.executable, "-m", "tests.replica_worker", str(suite)], cwd=ROOT, env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    results = []
    for p in procs:
        try:
            out, err = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            out, err = p.communicate()
        results.append((p.returncode, out, err))
    return results


def _parse(out: str) -> dict:
    line = [ln for ln in out.splitlines() if ln.startswith("RESULT ")][-1]
    return json.loads(line[len("RESULT "):])


def test_two_rank_box_aggregate(tmp_path: Path):
    results = _launch(_suite(tmp_path, {}))
    assert all(rc == 0 for rc, _, _ in results), [e[-2000:] for _, _, e in results]
    r0, r1 = _parse(results[0][1]), _parse(results[1][1])
    assert r1["outputs"] == {}                      # only rank 0 writes
    written = json.loads(Path(r0["outputs"]["json"]).read_text())
    aggregates = [r for r in written if r["metadata"].get("aggregate") == "box"]
    assert len(written) == 3 and len(aggregates) == 1
    agg = aggregates[0]
    assert agg["raw_metrics"]["elapsed_s"] == pytest.approx(0.002)       # max over ranks
    assert agg["raw_metrics"]["moved_bytes"] == pytest.approx(2e9)       # sum over ranks
    assert agg["metrics"]["hbm_bandwidth_gbps"] == pytest.approx(1000.0)
    assert agg["metrics"]["hbm_efficiency_pct"] == pytest.approx(1000.0 / 16000.0 * 100)
    assert agg["metadata"]["per_rank_elapsed_s"] == [0.001, 0.002]
    assert sorted(r["metadata"]["rank"] for r in written if "rank" in r["metadata"]) == [0, 1]


def test_failing_rank_does_not_hang_the_other(tmp_path: Path):
    results = _launch(_suite(tmp_path, {"fail_rank": 1}), timeout=90)
    assert results[1][0] != 0 and "fails on purpose" in results[1][2]
    assert results[0][0] != 0                       # errors out (timeout / connection), not hung
