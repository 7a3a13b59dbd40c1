"""Timing and tensor helpers (reference: src/teamredbench/utils.py:14-48)."""
from __future__ import annotations

import time
from typing import Any, Callable

from teamredbench_b200.device import synchronize_cuda_device
from teamredbench_b200.dtypes import DTypeSpec


def synchronize(torch_module: Any) -> None:
    synchronize_cuda_device(torch_module)


def timed_iterations(fn: Callable[[], None], *, torch_module: Any, warmup: int, iterations: int) -> float:
    """Mean host seconds per call of `fn` after `warmup` calls, device-synchronised
    on both sides of the timed loop (the torch backend's timing rule)."""
    for _ in range(warmup):
        fn()
    synchronize(torch_module)
    start = time.perf_counter()
    for _ in range(iterations):
        fn()
    synchronize(torch_module)
    return (time.perf_counter() - start) / max(iterations, 1)


def make_tensor(torch_module: Any, spec: DTypeSpec, shape: tuple[int, ...], device: Any,
                generator: Any | None = None):
    """Random tensor of `spec` (randn for floats, randint[0,17) for integers, as
    the reference); pass a seeded `generator` for reproducible inputs."""
    torch = torch_module
    dtype = getattr(torch, spec.torch_attr)
    kw = {"device": device} if generator is None else {"device": device, "generator": generator}
    if spec.kind == "bool":
        return torch.randint(0, 2, shape, dtype=torch.uint8, **kw).to(dtype=dtype)
    if spec.kind == "integer":
        return torch.randint(0, 17, shape, dtype=dtype, **kw)
    if spec.kind == "complex":
        real_dtype = torch.float32 if spec.name == "complex64" else torch.float64
        return torch.complex(torch.randn(shape, dtype=real_dtype, **kw),
                             torch.randn(shape, dtype=real_dtype, **kw)).to(dtype=dtype)
    return torch.randn(shape, dtype=torch.float32, **kw).to(dtype=dtype)


def tensor_nbytes(tensor: Any) -> int:
    return int(tensor.numel() * tensor.element_size())
