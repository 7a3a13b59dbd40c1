"""Two-GPU runs (skipped with fewer than 2 GPUs): replicas through the suite
runner with a box aggregate on rank 0, the NCCL collective sweep, and
bench.py's max-over-ranks whole-job value.  Processes are launched with
torch.distributed.run on 127.0.0.1, bounded by `timeout`."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import yaml

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if torch.cuda.device_count() < 2:  # pragma: no cover - single-GPU or CPU hosts
    pytest.skip("needs 2 GPUs", allow_module_level=True)

ROOT = Path(__file__).resolve().parent.parent
HW = ROOT / "teamredbench_b200" / "configs" / "profiles" / "hardware" / "nvidia_b200.yaml"
RT = ROOT / "teamredbench_b200" / "configs" / "profiles" / "cuda" / "cuda_generic.yaml"


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(args: list[str], timeout: int = 600) -> subprocess.CompletedProcess:
    cmd = ["timeout", "-k", "60", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()), *args]
    env = {**os.environ, "PYTHONPATH": str(ROOT), "NCCL_NVLS_ENABLE": "0"}
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout + 120)


def test_suite_replicas_aggregate_and_collective(tmp_path):
    suite = tmp_path / "suite.yaml"
    out = tmp_path / "results"
    suite.write_text(yaml.safe_dump({
        "name": "two-gpu", "device": {"profile": str(HW)}, "runtime": {"profile": str(RT)},
        "distributed": {"timeout_s": 300},
        "outputs": {"directory": str(out), "formats": ["json"]},
        "benchmarks": [
            {"benchmark": "hbm", "params": {"backend": "native", "dtypes": ["float32"], "modes": ["triad"],
                                            "size_mib": 1024, "scale": 3.0, "warmup": 2, "iterations": 10}},
            {"benchmark": "mfu", "params": {"backend": "native", "dtypes": ["bfloat16"],
                                            "shapes": [[4096, 4096, 4096]], "warmup": 2, "iterations": 5}},
            {"benchmark": "collective", "params": {"backend": "nccl", "dtypes": ["bfloat16"],
                                                   "operations": ["all_reduce", "all_gather", "broadcast"],
                                                   "sizes_bytes": [1024, 1 << 20, 256 << 20], "warmup": 2,
                                                   "iterations": 5}},
        ]}), encoding="utf-8")
    done = _torchrun(["-m", "teamredbench_b200", "run", str(suite), "--quiet-records"])
    assert done.returncode == 0, done.stderr[-3000:]
    files = sorted(out.glob("two-gpu-*.json"))
    files = [f for f in files if not f.name.endswith(".metadata.json")]
    assert len(files) == 1  # rank 0 alone writes
    records = json.loads(files[0].read_text())
    agg = {(r["benchmark"], r["case"]): r for r in records if r["metadata"].get("aggregate") == "box"}
    per_rank = [r for r in records if r["benchmark"] == "hbm" and "rank" in r["metadata"]]
    assert len(per_rank) == 2 and all(r["status"] == "ok" for r in per_rank)
    hbm = agg[("hbm", "triad_1024MiB")]
    assert hbm["metadata"]["world_size"] == 2
    single = max(r["metrics"]["hbm_bandwidth_gbps"] for r in per_rank)
    assert 1.6 * single < hbm["metrics"]["hbm_bandwidth_gbps"] <= 2.0 * single * 1.001
    mfu = agg[("mfu", "gemm_4096x4096x4096")]
    assert mfu["metrics"]["achieved_tops"] > 1000  # two B200s
    coll = [r for r in records if r["benchmark"] == "collective" and "rank" in r["metadata"]]
    assert len(coll) == 2 * 9 and all(r["status"] == "ok" for r in coll), [r.get("error") for r in coll]
    big = [r for r in coll if r["case"] == "all_reduce_256MiB"][0]
    assert big["metrics"]["bus_bandwidth_gbps"] > 100
    assert big["metadata"]["world_size"] == 2


def test_bench_two_gpus_whole_job_value():
    done = _torchrun(["bench.py", "--gpus", "2", "--steps", "5", "--warmup", "3", "--no-extras", "--e2e-steps", "1"])
    assert done.returncode == 0, done.stderr[-3000:]
    line = json.loads([ln for ln in done.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["n_gpus"] == 2 and line["scaling"] == "weak"
    assert line["value"] > 1.8 * line["roofline"]["achieved"] * 0.95  # sum over replicas
    assert line["cpu_baseline"] is None  # rank 0 at N=1 only
