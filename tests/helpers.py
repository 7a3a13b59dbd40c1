"""Shared helpers for the GPU parity tests (torch <-> raw numpy storage)."""
from __future__ import annotations

import math

import numpy as np

import oracle

TORCH_DTYPE = {
    "float32": "float32",
    "tfloat32": "float32",
    "float64": "float64",
    "bfloat16": "bfloat16",
    "float16": "float16",
    "int8": "int8",
    "float8_e4m3fn": "float8_e4m3fn",
    "int32": "int32",
}

GEMM_OUT = {"bfloat16": "bfloat16", "float16": "float16", "tfloat32": "float32", "float8_e4m3fn": "bfloat16",
            "int8": "int32", "float32": "float32", "float64": "float64"}
# rel-to-max tolerances of the reference's native GEMM harness
# (tests/native/gemm_parity.hip.cpp:174-178: 1e-10 for double, 1e-4 for float,
# 1e-2 for 16-bit), tightened to 1e-5 for tf32-exact inputs (the BASELINE
# bound for fp32-accumulate tf32), against the fp64 CPU oracle at every K.
GEMM_TOLERANCE = {"bfloat16": 1e-2, "float16": 1e-2, "float8_e4m3fn": 1e-2, "tfloat32": 1e-5,
                  "float32": 1e-4, "float64": 1e-10, "int8": 0.0}  # int8: bit-exact


def torch_dtype(name: str):
    import torch

    return getattr(torch, TORCH_DTYPE[name])


def to_raw(tensor) -> np.ndarray:
    """Tensor (any device) -> numpy array in the oracle's storage convention."""
    import torch

    t = tensor.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def from_raw(array: np.ndarray, name: str, device: str = "cuda"):
    import torch

    array = np.ascontiguousarray(array)
    if name == "bfloat16":
        return torch.from_numpy(array.view(np.int16)).view(torch.bfloat16).to(device)
    if name == "float8_e4m3fn":
        return torch.from_numpy(array.view(np.uint8)).view(torch.float8_e4m3fn).to(device)
    return torch.from_numpy(array).to(device)


def uniform_pm1(n: int, name: str, seed: int = 0, device: str = "cuda"):
    """BASELINE stream inputs: b then c ~ uniform[-1, 1) from `seed`, cast to dtype."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    if name == "float64":
        b = torch.rand(n, generator=g, device=device, dtype=torch.float64) * 2 - 1
        c = torch.rand(n, generator=g, device=device, dtype=torch.float64) * 2 - 1
        return b, c
    if name == "int8":
        b = torch.randint(-128, 128, (n,), generator=g, device=device, dtype=torch.int8)
        return b, b.clone()
    b = (torch.rand(n, generator=g, device=device) * 2 - 1).to(torch_dtype(name))
    c = (torch.rand(n, generator=g, device=device) * 2 - 1).to(torch_dtype(name))
    return b, c


def gemm_operands(name: str, m: int, n: int, k: int, seed: int = 0, device: str = "cuda"):
    """BASELINE GEMM inputs (A drawn before B).  Returns (a, b, scale_a, scale_b)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    if name == "int8":
        a = torch.randint(-127, 128, (m, k), generator=g, device=device, dtype=torch.int8)
        b = torch.randint(-127, 128, (k, n), generator=g, device=device, dtype=torch.int8)
        return a, b, 1.0, 1.0
    if name == "float64":
        a = torch.randn(m, k, generator=g, device=device, dtype=torch.float64) / math.sqrt(k)
        b = torch.randn(k, n, generator=g, device=device, dtype=torch.float64) / math.sqrt(k)
        return a, b, 1.0, 1.0
    a32 = torch.randn(m, k, generator=g, device=device) / math.sqrt(k)
    b32 = torch.randn(k, n, generator=g, device=device) / math.sqrt(k)
    if name in ("bfloat16", "float16", "float32"):
        return a32.to(torch_dtype(name)), b32.to(torch_dtype(name)), 1.0, 1.0
    if name == "tfloat32":
        from teamredbench_b200 import _native

        a32, b32 = a32.contiguous(), b32.contiguous()
        _native.round_tf32(a32.data_ptr(), a32.numel(), torch.cuda.current_stream().cuda_stream)
        _native.round_tf32(b32.data_ptr(), b32.numel(), torch.cuda.current_stream().cuda_stream)
        return a32, b32, 1.0, 1.0
    sa = float(a32.abs().max()) / 448.0
    sb = float(b32.abs().max()) / 448.0
    return (a32 / sa).to(torch.float8_e4m3fn), (b32 / sb).to(torch.float8_e4m3fn), sa, sb


def gemm_result_f64(name: str, c) -> np.ndarray:
    raw = to_raw(c)
    if GEMM_OUT[name] == "bfloat16":
        return oracle.bf16_to_f32(raw).astype(np.float64)
    return raw.astype(np.float64)
