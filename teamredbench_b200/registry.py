"""Benchmark / metric registries and plugin loading.

Same API as the reference (src/teamredbench/registry.py:13-56): decorators
populate module-level dicts keyed by name; later registrations replace earlier
ones, which is how a suite plugin overrides a built-in.
"""
from __future__ import annotations

import importlib
from typing import Any, Callable

from teamredbench_b200.metrics.base import MetricDefinition

BENCHMARK_REGISTRY: dict[str, type] = {}
METRIC_REGISTRY: dict[str, MetricDefinition] = {}


def register_benchmark(name: str) -> Callable[[type], type]:
    def wrap(cls: type) -> type:
        cls.name = name
        BENCHMARK_REGISTRY[name] = cls
        return cls

    return wrap


def register_metric(name: str, description: str) -> Callable:
    def wrap(fn: Callable[[dict[str, Any]], float | None]):
        METRIC_REGISTRY[name] = MetricDefinition(name=name, description=description, compute=fn)
        return fn

    return wrap


def _lookup(table: dict, kind: str, name: str):
    try:
        return table[name]
    except KeyError:
        raise KeyError(f"Unknown {kind}: {name}") from None


def get_benchmark(name: str) -> type:
    return _lookup(BENCHMARK_REGISTRY, "benchmark", name)


def get_metric(name: str) -> MetricDefinition:
    return _lookup(METRIC_REGISTRY, "metric", name)


def list_benchmarks() -> list[str]:
    return sorted(BENCHMARK_REGISTRY)


def list_metrics() -> list[str]:
    return sorted(METRIC_REGISTRY)


def load_plugins(module_names: list[str]) -> None:
    """Import each module; importing is what registers its contents."""
    for module_name in module_names:
        importlib.import_module(module_name)
