"""NCCL collective bandwidth sweep (reference:
src/teamredbench/benchmarks/collective.py).

Kept on torch.distributed + NCCL over NVLink 5 / NVSwitch: no native kernel
replaces it.  Additions over the reference:
  * `sizes_bytes` (any byte count, e.g. 1 KiB .. 4 GiB) next to the
    reference's integer `sizes_mib`, which cannot express sub-MiB sizes;
  * tensor values uniform[-1,1) seeded by rank (`seed`, default 0);
  * `bus_factor_nccl_tests` (all_gather's (n-1)/n applied to the gathered
    total, as nccl-tests does) beside the reference's per-rank convention;
  * `preallocate_outputs: true` to keep all_gather's output allocation out of
    the timed loop (the reference allocates inside it);
  * `elapsed_s` is device time (CUDA events around the timed loop), the max
    over ranks; the reference's host timing of the same loop is kept as
    `host_elapsed_s`.
Bus factors (reference :12-16): all_reduce 2(n-1)/n, all_gather (n-1)/n,
broadcast 1."""
from __future__ import annotations

import socket
import time
from typing import Any

from teamredbench_b200.benchmarks.base import Benchmark, BenchmarkRecord
from teamredbench_b200.device import cuda_device_available
from teamredbench_b200.registry import register_benchmark

BUS_FACTORS = {
    "all_reduce": lambda world_size: 2 * (world_size - 1) / world_size,
    "all_gather": lambda world_size: (world_size - 1) / world_size,
    "broadcast": lambda world_size: 1.0,
}
NCCL_TESTS_BUS_FACTORS = {
    "all_reduce": lambda world_size: 2 * (world_size - 1) / world_size,
    "all_gather": lambda world_size: float(world_size - 1),  # (n-1)/n of the n-times-larger total
    "broadcast": lambda world_size: 1.0,
}


def format_size(size_bytes: int) -> str:
    for unit, shift in (("GiB", 30), ("MiB", 20), ("KiB", 10)):
        if size_bytes >= 1 << shift and size_bytes % (1 << shift) == 0:
            return f"{size_bytes >> shift}{unit}"
    return f"{size_bytes}B"


@register_benchmark("collective")
class CollectiveBandwidthBenchmark(Benchmark):
    default_metrics = ["payload_bandwidth_gbps", "bus_bandwidth_gbps", "link_efficiency_pct", "latency_us"]

    @staticmethod
    def _normalize_backend(backend: str) -> str:
        normalized = backend.strip().lower()
        return "nccl" if normalized == "rccl" else normalized

    def _ensure_process_group(self, backend: str):
        dist = self.torch.distributed
        if not dist.is_available():
            raise RuntimeError("torch.distributed is not available in this build.")
        if not dist.is_initialized():
            dist.init_process_group(backend=backend, init_method="env://")
        return dist

    def _scope(self, dist: Any) -> str:
        hosts = [None] * dist.get_world_size()
        dist.all_gather_object(hosts, socket.gethostname())
        return "inter-node" if len(set(hosts)) > 1 else "intra-node"

    def _run_collective(self, op_name: str, dist: Any, tensor: Any, gather_list: list | None = None) -> None:
        if op_name == "all_reduce":
            dist.all_reduce(tensor)
        elif op_name == "all_gather":
            outputs = gather_list if gather_list is not None else [
                self.torch.empty_like(tensor) for _ in range(dist.get_world_size())]
            dist.all_gather(outputs, tensor)
        elif op_name == "broadcast":
            dist.broadcast(tensor, src=0)
        else:
            raise KeyError(f"Unknown collective operation: {op_name}")

    def _sizes(self) -> list[tuple[int, Any]]:
        """(bytes, label used in case names and metadata) per requested size."""
        if self.params.get("sizes_bytes") is not None:
            return [(int(b), format_size(int(b))) for b in self.params["sizes_bytes"]]
        return [(int(m) * 1024 * 1024, m) for m in self.params.get("sizes_mib", [8, 64, 256])]

    def _make_tensor(self, spec, numel: int, seed: int):
        torch = self.torch
        g = torch.Generator(device=self.device).manual_seed(seed)
        dtype = getattr(torch, spec.torch_attr)
        if spec.kind in ("integer", "bool"):
            return torch.randint(-8 if spec.name != "uint8" else 0, 9, (numel,), device=self.device, generator=g,
                                 dtype=dtype)
        return (torch.rand(numel, device=self.device, generator=g) * 2 - 1).to(dtype)

    def _time_loop(self, dist: Any, fn, warmup: int, iterations: int) -> tuple[float, float]:
        """Mean seconds per collective, max over ranks: device time from CUDA
        events on the current stream (which NCCL's blocking collectives make
        wait for their own stream), and the reference's host timing of the same
        loop (timed_iterations' rule: perf_counter between two synchronizes,
        src/teamredbench/utils.py:14-29)."""
        torch = self.torch
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        start.record()
        for _ in range(iterations):
            fn()
        stop.record()
        torch.cuda.synchronize()
        host = (time.perf_counter() - t0) / max(iterations, 1)
        device = start.elapsed_time(stop) / 1e3 / max(iterations, 1)
        both = torch.tensor([device, host], dtype=torch.float64, device=self.device)
        dist.all_reduce(both, op=dist.ReduceOp.MAX)
        return float(both[0].item()), float(both[1].item())

    def run(self) -> list[BenchmarkRecord]:
        if self.context.torch_module is None:
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a", error="PyTorch is not installed."))]
        torch = self.torch
        if not cuda_device_available(torch):
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a",
                                                         error="No CUDA device visible to PyTorch."))]
        self.set_device()
        backend = self._normalize_backend(str(self.params.get("backend", "nccl")))
        try:
            dist = self._ensure_process_group(backend=backend)
        except Exception as exc:  # noqa: BLE001
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a", error=str(exc)))]
        world_size = dist.get_world_size()
        if world_size < 2:
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a",
                                                         error="Collective benchmark requires WORLD_SIZE >= 2."))]
        operations = list(self.params.get("operations", ["all_reduce"]))
        warmup = int(self.params.get("warmup", 20))
        iterations = int(self.params.get("iterations", 100))
        seed = int(self.params.get("seed", 0))
        preallocate = bool(self.params.get("preallocate_outputs", False))
        scope = self._scope(dist)
        records: list[BenchmarkRecord] = []
        for spec in self.selected_dtype_specs():
            for size_bytes, label in self._sizes():
                numel = max(size_bytes // spec.bytes_per_element, 1)
                for op_name in operations:
                    case = f"{op_name}_{label}" if isinstance(label, str) else f"{op_name}_{label}MiB"
                    meta_size = {"size_bytes": numel * spec.bytes_per_element}
                    if not isinstance(label, str):
                        meta_size["size_mib"] = label
                    try:
                        tensor = self._make_tensor(spec, numel, seed + dist.get_rank())
                        gather = ([torch.empty_like(tensor) for _ in range(world_size)]
                                  if preallocate and op_name == "all_gather" else None)
                        dist.barrier()
                        elapsed_s, host_s = self._time_loop(
                            dist, lambda: self._run_collective(op_name, dist, tensor, gather), warmup, iterations)
                        dist.barrier()
                        del tensor, gather
                    except Exception as exc:  # noqa: BLE001
                        records.append(self.emit_record(self.skipped_record(
                            case=case, dtype=spec.name, error=str(exc),
                            metadata={"operation": op_name, "scope": scope, **meta_size})))
                        continue
                    records.append(self.emit_record(BenchmarkRecord(
                        benchmark=self.name, case=case, dtype=spec.name,
                        raw_metrics={
                            "elapsed_s": elapsed_s,
                            "host_elapsed_s": host_s,
                            "payload_bytes": numel * spec.bytes_per_element,
                            "bus_factor": BUS_FACTORS[op_name](world_size),
                            "bus_factor_nccl_tests": NCCL_TESTS_BUS_FACTORS[op_name](world_size),
                            "peak_link_bandwidth_gbps": self.context.hardware_profile.peak_link_bandwidth_gbps.get(
                                "network" if scope == "inter-node" else "xgmi"),
                        },
                        metadata={"operation": op_name, "scope": scope, "world_size": world_size,
                                  "preallocated_outputs": preallocate, **meta_size})))
        return records
