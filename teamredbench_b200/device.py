"""Device discovery through torch.cuda plus NVIDIA tool probes.

Mirrors src/teamredbench/device.py:9-127.  The reference's ROCm helper names
(rocm_device_available, rocm_device, set_rocm_device, synchronize_rocm_device)
are kept as aliases: PyTorch exposes NVIDIA GPUs through the same torch.cuda
API, so benchmark code written against the reference keeps working."""
from __future__ import annotations

import shutil
import subprocess
from dataclasses import asdict, dataclass
from typing import Any


@dataclass
class DeviceInfo:
    index: int
    name: str
    total_memory_bytes: int | None = None
    multiprocessor_count: int | None = None
    clock_rate_khz: int | None = None
    gcn_arch_name: str | None = None
    compute_capability: str | None = None


def load_torch():
    try:
        import torch
    except ImportError:
        return None
    return torch


def cuda_device_available(torch_module: Any) -> bool:
    return torch_module is not None and bool(torch_module.cuda.is_available())


def cuda_device(torch_module: Any, device_id: int):
    return torch_module.device(f"cuda:{device_id}")


def set_cuda_device(torch_module: Any, device_id: int) -> None:
    if cuda_device_available(torch_module):
        torch_module.cuda.set_device(device_id)


def synchronize_cuda_device(torch_module: Any) -> None:
    if cuda_device_available(torch_module):
        torch_module.cuda.synchronize()


# reference-compatible names
rocm_device_available = cuda_device_available
rocm_device = cuda_device
set_rocm_device = set_cuda_device
synchronize_rocm_device = synchronize_cuda_device


def _run_command(command: list[str]) -> str | None:
    if shutil.which(command[0]) is None:
        return None
    try:
        completed = subprocess.run(command, check=False, capture_output=True, text=True, timeout=20)
    except (OSError, subprocess.TimeoutExpired):
        return None
    if completed.returncode != 0:
        return None
    return completed.stdout.strip() or None


def detect_device(torch_module: Any, device_id: int = 0) -> DeviceInfo | None:
    if not cuda_device_available(torch_module):
        return None
    props = torch_module.cuda.get_device_properties(device_id)
    major, minor = getattr(props, "major", None), getattr(props, "minor", None)
    return DeviceInfo(
        index=device_id,
        name=str(props.name),
        total_memory_bytes=getattr(props, "total_memory", None),
        multiprocessor_count=getattr(props, "multi_processor_count", None),
        clock_rate_khz=getattr(props, "clock_rate", None),
        gcn_arch_name=getattr(props, "gcnArchName", None) or None,
        compute_capability=f"{major}.{minor}" if major is not None else None,
    )


def detect_runtime(torch_module: Any) -> dict[str, Any]:
    torch_info: dict[str, Any] = {}
    if torch_module is not None:
        version = getattr(torch_module, "version", None)
        torch_info = {"torch_version": getattr(torch_module, "__version__", "unknown"),
                      "cuda_version": getattr(version, "cuda", None)}
    smi = _run_command(["nvidia-smi", "--query-gpu=name,driver_version,clocks.max.sm,memory.total",
                        "--format=csv,noheader"])
    nvcc = _run_command(["nvcc", "--version"])
    return {
        "torch": torch_info,
        "nvcc_version": nvcc.splitlines()[-1] if nvcc else None,
        "nvidia_smi": smi,
    }


def discover_environment(torch_module: Any, device_id: int = 0) -> dict[str, Any]:
    device = detect_device(torch_module, device_id=device_id)
    return {
        "device": asdict(device) if device else None,
        "runtime": detect_runtime(torch_module),
        "suggested_hardware_profile": {
            "name": device.name if device else "fill-me",
            "family": "blackwell",
            "peak_hbm_bandwidth_gbps": None,
            "peak_link_bandwidth_gbps": {"xgmi": None, "nvlink": None, "network": None},
            "peak_compute_tops": {},
            "notes": ["Fill in theoretical peak values before using MFU or efficiency metrics."],
        },
    }
