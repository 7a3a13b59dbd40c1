"""Derived metrics.  Formulas are the reference's
(src/teamredbench/metrics/common.py:14-83): GB/s = bytes / s / 1e9,
TOPS = ops / s / 1e12, efficiency = value / peak * 100.  Any missing input, or
a zero denominator, yields None."""
from __future__ import annotations

from typing import Any

from teamredbench_b200.registry import register_metric


def _num(raw: dict[str, Any], key: str) -> float | None:
    value = raw.get(key)
    return None if value is None else float(value)


def _ratio(numerator: float | None, denominator: float | None, scale: float) -> float | None:
    if numerator is None or denominator is None or denominator == 0:
        return None
    return numerator / denominator / scale


@register_metric("latency_us", "Average iteration latency in microseconds.")
def latency_us(raw: dict[str, Any]) -> float | None:
    elapsed = _num(raw, "elapsed_s")
    return None if elapsed is None else elapsed * 1e6


@register_metric("hbm_bandwidth_gbps", "Device memory bandwidth derived from moved bytes.")
def hbm_bandwidth_gbps(raw: dict[str, Any]) -> float | None:
    return _ratio(_num(raw, "moved_bytes"), _num(raw, "elapsed_s"), 1e9)


@register_metric("hbm_efficiency_pct", "HBM bandwidth as a percentage of configured peak.")
def hbm_efficiency_pct(raw: dict[str, Any]) -> float | None:
    pct = _ratio(hbm_bandwidth_gbps(raw), _num(raw, "peak_bandwidth_gbps"), 0.01)
    return pct


@register_metric("payload_bandwidth_gbps", "Collective payload bandwidth in GB/s.")
def payload_bandwidth_gbps(raw: dict[str, Any]) -> float | None:
    return _ratio(_num(raw, "payload_bytes"), _num(raw, "elapsed_s"), 1e9)


@register_metric("bus_bandwidth_gbps", "Collective link bandwidth in GB/s after bus factor.")
def bus_bandwidth_gbps(raw: dict[str, Any]) -> float | None:
    payload = payload_bandwidth_gbps(raw)
    factor = _num(raw, "bus_factor")
    if payload is None or factor is None:
        return None
    return payload * factor


@register_metric("link_efficiency_pct", "Collective bandwidth as a percentage of configured peak link bandwidth.")
def link_efficiency_pct(raw: dict[str, Any]) -> float | None:
    return _ratio(bus_bandwidth_gbps(raw), _num(raw, "peak_link_bandwidth_gbps"), 0.01)


@register_metric("achieved_tops", "Achieved throughput in tera-ops per second.")
def achieved_tops(raw: dict[str, Any]) -> float | None:
    return _ratio(_num(raw, "achieved_ops"), _num(raw, "elapsed_s"), 1e12)


@register_metric("mfu_pct", "Measured throughput as a percentage of configured peak.")
def mfu_pct(raw: dict[str, Any]) -> float | None:
    return _ratio(achieved_tops(raw), _num(raw, "peak_tops"), 0.01)


@register_metric("bus_bandwidth_nccl_tests_gbps",
                 "Collective bus bandwidth in the nccl-tests convention (all_gather factor on the total size).")
def bus_bandwidth_nccl_tests_gbps(raw: dict[str, Any]) -> float | None:
    payload = payload_bandwidth_gbps(raw)
    factor = _num(raw, "bus_factor_nccl_tests")
    if payload is None or factor is None:
        return None
    return payload * factor
