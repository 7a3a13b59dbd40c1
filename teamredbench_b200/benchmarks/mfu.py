"""Dense GEMM throughput / MFU benchmark (reference:
src/teamredbench/benchmarks/mfu.py).

backend: native (default kernel ``mfu_b200``) runs the tcgen05 GEMM launcher
per (dtype, shape); backend: torch runs torch.mm with the output in the input
dtype, as the reference does, plus the torch calls for the dtypes the
reference's torch path cannot express (tfloat32 = fp32 mm with TF32 enabled,
int8 = torch._int_mm with int32 output, float8_e4m3fn = torch._scaled_mm with
per-tensor scales and bf16 output)."""
from __future__ import annotations

import math
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

DEFAULT_SHAPES = [[4096, 4096, 4096], [8192, 8192, 8192]]


@register_benchmark("mfu")
class MfuBenchmark(Benchmark):
    default_metrics = ["achieved_tops", "mfu_pct", "latency_us"]

    def _common_params(self) -> tuple[int, int, list[list[int]]]:
        p = self.params
        return int(p.get("warmup", 10)), int(p.get("iterations", 50)), list(p.get("shapes", DEFAULT_SHAPES))

    def _precheck(self, spec, peak_tops, case: str, metadata: dict[str, Any]) -> BenchmarkRecord | None:
        if spec.matmul_ops_factor == 0:
            return self.emit_record(self.skipped_record(case=case, dtype=spec.name,
                                                        error="MFU is not defined for this dtype.", metadata=metadata))
        if peak_tops is None:
            return self.emit_record(self.skipped_record(
                case=case, dtype=spec.name, error="Missing peak_compute_tops entry for dtype in hardware profile.",
                metadata=metadata))
        return None

    def _run_native(self) -> list[BenchmarkRecord]:
        warmup, iterations, shapes = self._common_params()
        kernel = resolve_native_kernel(benchmark=self.name, params=self.params, suite_path=self.context.suite_path,
                                       repo_root=self.context.repo_root, default_kernel="mfu_b200")
        try:
            kernel = replace(kernel, binary_path=prepare_native_kernel_binary(kernel))
        except NativeKernelError as exc:
            out = []
            for spec in self.selected_dtype_specs():
                for shape in shapes:
                    m, n, k = (int(d) for d in shape)
                    out.append(self.emit_record(self.skipped_record(
                        case=f"gemm_{m}x{n}x{k}", dtype=spec.name, error=str(exc),
                        metadata={"backend": "native", "kernel": kernel.name, "m": m, "n": n, "k": k})))
            return out

        records: list[BenchmarkRecord] = []
        for spec in self.selected_dtype_specs():
            peak_tops = self.context.hardware_profile.peak_compute_tops.get(spec.name)
            for shape in shapes:
                m, n, k = (int(d) for d in shape)
                case = f"gemm_{m}x{n}x{k}"
                metadata: dict[str, Any] = {"backend": "native", "kernel": kernel.name, "m": m, "n": n, "k": k}
                skipped = self._precheck(spec, peak_tops, case, metadata)
                if skipped is not None:
                    records.append(skipped)
                    continue
                self.sync_ranks()
                try:
                    result = run_native_kernel(kernel, [
                        "--dtype", spec.name, "--m", str(m), "--n", str(n), "--k", str(k), "--warmup", str(warmup),
                        "--iterations", str(iterations), "--device-id", str(self.context.device_id)])
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
                raw.setdefault("achieved_ops", spec.matmul_ops_factor * m * n * k)
                raw.setdefault("peak_tops", peak_tops)
                records.append(self.emit_record(BenchmarkRecord(benchmark=self.name, case=case, dtype=spec.name,
                                                                raw_metrics=raw, metadata=metadata)))
        return records

    def _torch_operands(self, spec, m: int, n: int, k: int, generator):
        """Operands and the callable computing one product, per dtype."""
        torch = self.torch
        dev = self.device
        kw = {"device": dev} if generator is None else {"device": dev, "generator": generator}
        if spec.name == "int8":
            a = torch.randint(-127, 128, (m, k), dtype=torch.int8, **kw)
            b = torch.randint(-127, 128, (n, k), dtype=torch.int8, **kw).t()
            return lambda: torch._int_mm(a, b)
        if spec.name == "float8_e4m3fn":
            a32 = torch.randn(m, k, **kw) / math.sqrt(k)
            b32 = torch.randn(n, k, **kw) / math.sqrt(k)
            sa = (a32.abs().max() / 448.0).float()
            sb = (b32.abs().max() / 448.0).float()
            a = (a32 / sa).to(torch.float8_e4m3fn)
            b = (b32 / sb).to(torch.float8_e4m3fn).t()
            return lambda: torch._scaled_mm(a, b, scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
        if spec.name == "tfloat32":
            torch.backends.cuda.matmul.allow_tf32 = True
        a = make_tensor(torch, spec, (m, k), dev, generator)
        b = make_tensor(torch, spec, (k, n), dev, generator)
        out = torch.empty((m, n), device=dev, dtype=getattr(torch, spec.torch_attr))
        return lambda: torch.mm(a, b, out=out)

    def _run_torch(self) -> list[BenchmarkRecord]:
        if self.context.torch_module is None:
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a", error="PyTorch is not installed."))]
        torch = self.torch
        if not cuda_device_available(torch):
            return [self.emit_record(self.skipped_record(case="global", dtype="n/a",
                                                         error="No CUDA device visible to PyTorch."))]
        self.set_device()
        warmup, iterations, shapes = self._common_params()
        generator = None
        if self.params.get("seed") is not None:
            generator = torch.Generator(device=self.device).manual_seed(int(self.params["seed"]))
        records: list[BenchmarkRecord] = []
        for spec in self.selected_dtype_specs():
            peak_tops = self.context.hardware_profile.peak_compute_tops.get(spec.name)
            for shape in shapes:
                m, n, k = (int(d) for d in shape)
                case = f"gemm_{m}x{n}x{k}"
                metadata = {"backend": "torch", "m": m, "n": n, "k": k}
                skipped = self._precheck(spec, peak_tops, case, metadata)
                if skipped is not None:
                    records.append(skipped)
                    continue
                allow_tf32 = torch.backends.cuda.matmul.allow_tf32
                try:
                    fn = self._torch_operands(spec, m, n, k, generator)
                    self.sync_ranks()
                    elapsed_s = timed_iterations(fn, torch_module=torch, warmup=warmup, iterations=iterations)
                except Exception as exc:  # noqa: BLE001
                    records.append(self.emit_record(self.skipped_record(case=case, dtype=spec.name, error=str(exc),
                                                                        metadata=metadata)))
                    continue
                finally:
                    torch.backends.cuda.matmul.allow_tf32 = allow_tf32
                records.append(self.emit_record(BenchmarkRecord(
                    benchmark=self.name, case=case, dtype=spec.name,
                    raw_metrics={"elapsed_s": elapsed_s, "achieved_ops": spec.matmul_ops_factor * m * n * k,
                                 "peak_tops": peak_tops},
                    metadata=metadata)))
        return records

    def run(self) -> list[BenchmarkRecord]:
        backend = str(self.params.get("backend", "torch")).lower()
        if backend == "torch":
            return self._run_torch()
        if backend == "native":
            return self._run_native()
        raise KeyError(f"Unknown MFU backend: {backend}")
