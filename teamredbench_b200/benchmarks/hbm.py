"""STREAM copy / scale / triad benchmark (reference:
src/teamredbench/benchmarks/hbm.py).

backend: native (default kernel ``hbm_b200``) runs the B200 launcher once per
(dtype, mode) case through the native runtime's subprocess contract;
backend: torch runs the same ops as torch calls (the reference semantics).
Records, case names, metadata and raw metrics are the reference's."""
from __future__ import annotations

from dataclasses import replace
from typing import Any

from teamredbench_b200.benchmarks.base import Benchmark, BenchmarkRecord
from teamredbench_b200.device import cuda_device_available
from teamredbench_b200.native.runtime import (
    NativeKernelError,
    prepare_native_kernel_binary,
    resolve_native_kernel,
    run_native_kernel,
)
from teamredbench_b200.registry import register_benchmark
from teamredbench_b200.utils import make_tensor, timed_iterations

MODE_BYTE_FACTORS = {"copy": 2, "scale": 2, "triad": 3}


@register_benchmark("hbm")
class HbmBandwidthBenchmark(Benchmark):
    default_metrics = ["hbm_bandwidth_gbps", "hbm_efficiency_pct", "latency_us"]

    def _run_mode(self, mode: str, src: Any, dst: Any, aux: Any, scale: float) -> None:
        torch = self.torch
        if mode == "copy":
            dst.copy_(src)
        elif mode == "scale":
            torch.mul(src, scale, out=dst)
        elif mode == "triad":
            torch.add(src, aux, alpha=scale, out=dst)
        else:
            raise KeyError(f"Unknown HBM mode: {mode}")

    def _common_params(self) -> tuple[int, int, int, list[str], float]:
        p = self.params
        return (int(p.get("size_mib", 1024)), int(p.get("warmup", 10)), int(p.get("iterations", 50)),
                list(p.get("modes", ["copy"])), float(p.get("scale", 1.0)))

    def _skip_all(self, modes: list[str], size_mib: int, kernel_name: str, error: str) -> list[BenchmarkRecord]:
        return [
            self.emit_record(self.skipped_record(
                case=f"{mode}_{size_mib}MiB", dtype=spec.name, error=error,
                metadata={"backend": "native", "kernel": kernel_name, "mode": mode, "size_mib": size_mib}))
            for spec in self.selected_dtype_specs() for mode in modes
        ]

    def _run_native(self) -> list[BenchmarkRecord]:
        size_mib, warmup, iterations, modes, scale = self._common_params()
        total_bytes = size_mib * 1024 * 1024
        kernel = resolve_native_kernel(benchmark=self.name, params=self.params, suite_path=self.context.suite_path,
                                       repo_root=self.context.repo_root, default_kernel="hbm_b200")
        try:
            kernel = replace(kernel, binary_path=prepare_native_kernel_binary(kernel))
        except NativeKernelError as exc:
            return self._skip_all(modes, size_mib, kernel.name, str(exc))

        records: list[BenchmarkRecord] = []
        for spec in self.selected_dtype_specs():
            numel = max(total_bytes // spec.bytes_per_element, 1)
            for mode in modes:
                case = f"{mode}_{size_mib}MiB"
                metadata: dict[str, Any] = {"backend": "native", "kernel": kernel.name, "mode": mode,
                                            "size_mib": size_mib, "elements": numel}
                args = ["--dtype", spec.name, "--mode", mode, "--size-mib", str(size_mib), "--warmup", str(warmup),
                        "--iterations", str(iterations), "--device-id", str(self.context.device_id),
                        "--scale", str(scale)]
                if self.params.get("blocks_per_cu") is not None:
                    args += ["--blocks-per-cu", str(int(self.params["blocks_per_cu"]))]
                    metadata["blocks_per_cu"] = int(self.params["blocks_per_cu"])
                if self.params.get("variant") is not None:
                    args += ["--variant", str(self.params["variant"])]
                self.sync_ranks()
                try:
                    result = run_native_kernel(kernel, args)
                except NativeKernelError as exc:
                    records.append(self.emit_record(self.skipped_record(case=case, dtype=spec.name, error=str(exc),
                                                                        metadata=metadata)))
                    continue
                metadata.update(result.metadata)
                if result.status != "ok":
                    records.append(self.emit_record(self.skipped_record(
                        case=case, dtype=spec.name, error=result.error or "Native kernel did not report success.",
                        metadata=metadata)))
                    continue
                raw = dict(result.raw_metrics)
                raw.setdefault("elapsed_s", raw.get("elapsed_seconds"))
                if raw.get("elapsed_s") is None:
                    records.append(self.emit_record(self.skipped_record(
                        case=case, dtype=spec.name, error="Native kernel did not report elapsed_s.", metadata=metadata)))
                    continue
                raw.setdefault("moved_bytes", MODE_BYTE_FACTORS[mode] * numel * spec.bytes_per_element)
                raw.setdefault("peak_bandwidth_gbps", self.context.hardware_profile.peak_hbm_bandwidth_gbps)
                records.append(self.emit_record(BenchmarkRecord(benchmark=self.name, case=case, dtype=spec.name,
                                                                raw_metrics=raw, metadata=metadata)))
        return records

    def _run_torch(self) -> list[BenchmarkRecord]:
        if self.context.torch_module is None:
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a", error="PyTorch is not installed."))]
        torch = self.torch
        if not cuda_device_available(torch):
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a",
                                                         error="No CUDA device visible to PyTorch."))]
        self.set_device()
        size_mib, warmup, iterations, modes, scale = self._common_params()
        total_bytes = size_mib * 1024 * 1024
        generator = None
        if self.params.get("seed") is not None:
            generator = torch.Generator(device=self.device).manual_seed(int(self.params["seed"]))
        records: list[BenchmarkRecord] = []
        for spec in self.selected_dtype_specs():
            numel = max(total_bytes // spec.bytes_per_element, 1)
            for mode in modes:
                case = f"{mode}_{size_mib}MiB"
                try:
                    src = make_tensor(torch, spec, (numel,), self.device, generator)
                    dst = torch.empty_like(src)
                    aux = make_tensor(torch, spec, (numel,), self.device, generator) if mode == "triad" else None
                    self.sync_ranks()
                    elapsed_s = timed_iterations(lambda: self._run_mode(mode, src, dst, aux, scale),
                                                 torch_module=torch, warmup=warmup, iterations=iterations)
                except Exception as exc:  # noqa: BLE001 - any failure becomes a skipped record
                    records.append(self.emit_record(self.skipped_record(
                        case=case, dtype=spec.name, error=str(exc),
                        metadata={"backend": "torch", "mode": mode, "size_mib": size_mib})))
                    continue
                records.append(self.emit_record(BenchmarkRecord(
                    benchmark=self.name, case=case, dtype=spec.name,
                    raw_metrics={"elapsed_s": elapsed_s,
                                 "moved_bytes": MODE_BYTE_FACTORS[mode] * numel * spec.bytes_per_element,
                                 "peak_bandwidth_gbps": self.context.hardware_profile.peak_hbm_bandwidth_gbps},
                    metadata={"backend": "torch", "mode": mode, "size_mib": size_mib, "elements": numel})))
        return records

    def run(self) -> list[BenchmarkRecord]:
        backend = str(self.params.get("backend", "torch")).lower()
        if backend == "torch":
            return self._run_torch()
        if backend == "native":
            return self._run_native()
        raise KeyError(f"Unknown HBM backend: {backend}")
