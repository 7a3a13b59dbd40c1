from types import SimpleNamespace

from teamredbench_b200.benchmarks.base import BenchmarkContext
from teamredbench_b200.benchmarks.collective import (
    BUS_FACTORS,
    NCCL_TESTS_BUS_FACTORS,
    CollectiveBandwidthBenchmark,
    format_size,
)
from teamredbench_b200.config import HardwareProfile, RuntimeProfile


class _FakeCuda:
    def is_available(self) -> bool:
        return True

    def set_device(self, device_id: int) -> None:
        self.device_id = device_id


class _FakeTorch:
    def __init__(self):
        self.cuda = _FakeCuda()

    def device(self, spec: str) -> str:
        return spec


def _context():
    return BenchmarkContext(hardware_profile=HardwareProfile(name="test-hw", family="blackwell",
                                                             peak_link_bandwidth_gbps={"xgmi": 1.0, "network": 1.0}),
                            runtime_profile=RuntimeProfile(name="test-runtime"), device_info=None,
                            torch_module=_FakeTorch(), dtype_specs={})


def test_collective_accepts_rccl_backend_alias(monkeypatch):
    benchmark = CollectiveBandwidthBenchmark(context=_context(), params={"backend": "rccl"}, record_sink=None)
    seen: list[str] = []
    monkeypatch.setattr(benchmark, "_ensure_process_group",
                        lambda backend: seen.append(backend) or SimpleNamespace(get_world_size=lambda: 2))
    monkeypatch.setattr(benchmark, "_scope", lambda dist: "intra-node")
    monkeypatch.setattr(benchmark, "selected_dtype_specs", lambda: [])
    assert benchmark.run() == [] and seen == ["nccl"]


def test_byte_sizes_and_labels():
    bench = CollectiveBandwidthBenchmark(context=_context(), params={"sizes_bytes": [1024, 4096, 3 << 20, 4 << 30, 100]})
    assert [label for _, label in bench._sizes()] == ["1KiB", "4KiB", "3MiB", "4GiB", "100B"]
    bench = CollectiveBandwidthBenchmark(context=_context(), params={"sizes_mib": [8]})
    assert bench._sizes() == [(8 << 20, 8)]
    assert format_size(1 << 30) == "1GiB"


def test_bus_factors():
    assert BUS_FACTORS["all_reduce"](8) == 1.75
    assert BUS_FACTORS["all_gather"](8) == 0.875
    assert NCCL_TESTS_BUS_FACTORS["all_gather"](8) == 7.0
    assert BUS_FACTORS["broadcast"](4) == 1.0
