"""Registry of native kernels (reference: src/teamredbench/native/registry.py:7-48).

A definition names the benchmark it serves and how to obtain an executable:
a source file compiled on demand, and/or (added here) a prebuilt binary such
as the in-tree trb_hbm / trb_mfu launchers."""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path


@dataclass(frozen=True)
class NativeKernelDefinition:
    name: str
    benchmark: str
    description: str
    source_path: Path | None = None
    compile_args: tuple[str, ...] = ()
    binary_path: Path | None = None


NATIVE_KERNEL_REGISTRY: dict[str, NativeKernelDefinition] = {}


def register_native_kernel(*, name: str, benchmark: str, description: str, source_path: Path | None = None,
                           compile_args: tuple[str, ...] = (), binary_path: Path | None = None
                           ) -> NativeKernelDefinition:
    definition = NativeKernelDefinition(name=name, benchmark=benchmark, description=description,
                                        source_path=source_path, compile_args=tuple(compile_args),
                                        binary_path=binary_path)
    NATIVE_KERNEL_REGISTRY[name] = definition
    return definition


def get_native_kernel(name: str) -> NativeKernelDefinition:
    if name not in NATIVE_KERNEL_REGISTRY:
        raise KeyError(f"Unknown native kernel: {name}")
    return NATIVE_KERNEL_REGISTRY[name]


def list_native_kernels(benchmark: str | None = None) -> list[NativeKernelDefinition]:
    items = sorted(NATIVE_KERNEL_REGISTRY.values(), key=lambda d: d.name)
    return items if benchmark is None else [d for d in items if d.benchmark == benchmark]
