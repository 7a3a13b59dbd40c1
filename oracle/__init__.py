"""CPU oracle for the TeamRedBench B200 hot path.

TEST INFRASTRUCTURE ONLY.  The product package (``teamredbench_b200``) never
imports this module.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, as the
checker or as the timed CPU baseline.

The arithmetic lives in ``trb_oracle.c`` (built by ``oracle/Makefile`` into
``libtrb_oracle.so``); its header states, per operation, which reference
file:line it restates and how the restatement was pinned.  This wrapper only
marshals numpy arrays.

Element storage conventions (all numpy arrays are C-contiguous):
    float32 / tfloat32 -> np.float32
    float64            -> np.float64
    bfloat16           -> np.uint16 (raw bf16 bits)
    float16            -> np.float16 (raw IEEE half)
    int8               -> np.int8
    float8_e4m3fn      -> np.uint8 (raw e4m3 bits)
    int32              -> np.int32
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "libtrb_oracle.so"

# codes shared with include/trb_b200.h
DTYPE_CODES = {
    "float32": 0,
    "bfloat16": 1,
    "float16": 2,
    "float64": 3,
    "int8": 4,
    "float8_e4m3fn": 5,
    "tfloat32": 6,
    "int32": 7,
}
MODE_CODES = {"copy": 0, "scale": 1, "triad": 2}
NUMPY_STORAGE = {
    "float32": np.float32,
    "tfloat32": np.float32,
    "float64": np.float64,
    "bfloat16": np.uint16,
    "float16": np.float16,
    "int8": np.int8,
    "float8_e4m3fn": np.uint8,
    "int32": np.int32,
}

_lib = None


def build(verbose: bool = False) -> Path:
    """Compile libtrb_oracle.so with the committed Makefile."""
    completed = subprocess.run(["make", "-C", str(ORACLE_DIR)], capture_output=True, text=True)
    if completed.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{completed.stdout}\n{completed.stderr}")
    if verbose:
        print(completed.stdout)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        build()
    handle = ctypes.CDLL(str(LIB_PATH))
    vp, i64, dbl, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_double, ctypes.c_int
    handle.trbo_hbm.argtypes = [i32, i32, vp, vp, vp, i64, dbl, i32]
    handle.trbo_hbm.restype = i32
    handle.trbo_hbm_torch_tail.argtypes = [i32, i32, vp, vp, vp, i64, dbl]
    handle.trbo_hbm_torch_tail.restype = i32
    handle.trbo_gemm_rows.argtypes = [i32, i64, i64, i64, vp, vp, vp, i64, dbl, dbl, vp, i32]
    handle.trbo_gemm_rows.restype = i32
    handle.trbo_convert_f32.argtypes = [i32, vp, vp, i64]
    handle.trbo_convert_f32.restype = i32
    handle.trbo_e4m3_to_f32.argtypes = [ctypes.c_uint8]
    handle.trbo_e4m3_to_f32.restype = ctypes.c_float
    handle.trbo_round_tf32.argtypes = [ctypes.c_float]
    handle.trbo_round_tf32.restype = ctypes.c_float
    _lib = handle
    return handle


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1))


def _ptr(array: np.ndarray | None) -> int | None:
    if array is None:
        return None
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data


def hbm(dtype: str, mode: str, src: np.ndarray, aux: np.ndarray | None, scale: float,
        nthreads: int | None = None, out: np.ndarray | None = None) -> np.ndarray:
    """dst = op(src, aux) with torch-CPU (vector body) semantics; see trb_oracle.c."""
    storage = NUMPY_STORAGE[dtype]
    src = np.ascontiguousarray(src, dtype=storage)
    if aux is not None:
        aux = np.ascontiguousarray(aux, dtype=storage)
        assert aux.shape == src.shape
    dst = np.empty_like(src) if out is None else out
    status = lib().trbo_hbm(DTYPE_CODES[dtype], MODE_CODES[mode], _ptr(dst), _ptr(src), _ptr(aux),
                            src.size, float(scale), int(nthreads or default_threads()))
    if status != 0:
        raise ValueError(f"oracle hbm({dtype}, {mode}) returned {status}")
    return dst


def hbm_torch_tail(dtype: str, mode: str, src: np.ndarray, aux: np.ndarray | None, scale: float) -> np.ndarray:
    """torch's scalar-remainder formula (differs from hbm() only for bf16/f16 triad)."""
    storage = NUMPY_STORAGE[dtype]
    src = np.ascontiguousarray(src, dtype=storage)
    aux = None if aux is None else np.ascontiguousarray(aux, dtype=storage)
    dst = np.empty_like(src)
    status = lib().trbo_hbm_torch_tail(DTYPE_CODES[dtype], MODE_CODES[mode], _ptr(dst), _ptr(src), _ptr(aux),
                                       src.size, float(scale))
    if status != 0:
        raise ValueError(f"oracle hbm_torch_tail({dtype}, {mode}) returned {status}")
    return dst


def gemm_rows(dtype: str, a: np.ndarray, b: np.ndarray, rows: np.ndarray | list[int],
              scale_a: float = 1.0, scale_b: float = 1.0, nthreads: int | None = None) -> np.ndarray:
    """fp64 reference of (A @ B)[rows, :] for row-major A (m x k) and B (k x n)."""
    storage = NUMPY_STORAGE[dtype]
    a = np.ascontiguousarray(a, dtype=storage)
    b = np.ascontiguousarray(b, dtype=storage)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2, (a.shape, b.shape)
    rows = np.ascontiguousarray(np.asarray(rows, dtype=np.int64))
    out = np.empty((rows.size, n), dtype=np.float64)
    status = lib().trbo_gemm_rows(DTYPE_CODES[dtype], m, n, k, _ptr(a), _ptr(b), _ptr(rows), rows.size,
                                  float(scale_a), float(scale_b), _ptr(out), int(nthreads or default_threads()))
    if status != 0:
        raise ValueError(f"oracle gemm_rows({dtype}) returned {status}")
    return out


def from_f32(dtype: str, values: np.ndarray) -> np.ndarray:
    """RNE conversion of float32 values into dtype storage (bf16/f16/tf32/f32)."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(values.shape, dtype=NUMPY_STORAGE[dtype])
    status = lib().trbo_convert_f32(DTYPE_CODES[dtype], _ptr(values), _ptr(out), values.size)
    if status != 0:
        raise ValueError(f"unsupported conversion to {dtype}")
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def e4m3_to_f32(bits: np.ndarray) -> np.ndarray:
    table = np.array([lib().trbo_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
    return table[np.asarray(bits, dtype=np.uint8)]


def rel_to_max_error(result: np.ndarray, reference: np.ndarray) -> float:
    """max|C - ref| / max|ref|, the reference harness's error metric
    (tests/native/gemm_parity.hip.cpp:163-178)."""
    result = np.asarray(result, dtype=np.float64)
    reference = np.asarray(reference, dtype=np.float64)
    denom = float(np.max(np.abs(reference))) if reference.size else 0.0
    err = float(np.max(np.abs(result - reference))) if reference.size else 0.0
    return err / denom if denom > 0 else err
