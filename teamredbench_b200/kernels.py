"""torch-tensor front end of the native kernels.

Thin: it checks shapes / dtypes / devices, takes raw device pointers and the
current CUDA stream, and calls libtrb_b200 through ``_native``.  torch provides
device memory and streams only; all arithmetic happens in the CUDA kernels.
"""
from __future__ import annotations

from typing import Any

from teamredbench_b200 import _native

_TORCH_TO_TRB = {
    "torch.float32": "float32",
    "torch.bfloat16": "bfloat16",
    "torch.float16": "float16",
    "torch.float64": "float64",
    "torch.int8": "int8",
    "torch.uint8": "int8",
    "torch.float8_e4m3fn": "float8_e4m3fn",
}


_DTYPE_CACHE: dict[Any, str] = {}  # torch.dtype object -> library dtype name, filled on first use


def trb_dtype(tensor: Any) -> str:
    name = _DTYPE_CACHE.get(tensor.dtype)
    if name is None:
        name = _TORCH_TO_TRB.get(str(tensor.dtype))
        if name is None:
            raise _native.NativeSkipped(1, f"unsupported tensor dtype {tensor.dtype}")
        _DTYPE_CACHE[tensor.dtype] = name
    return name


def _stream_handle(tensor: Any, stream: Any | None) -> int:
    """Raw cudaStream_t of ``stream``, or of the device's current stream.

    The current stream is read through torch's raw-handle query (one C call,
    no Stream object built), which keeps the per-call host cost of a small
    GEMM close to the bare ctypes call; torch builds without it take the
    public ``torch.cuda.current_stream``."""
    import torch

    if stream is not None:
        return int(stream.cuda_stream)
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    if raw is not None:
        return int(raw(tensor.get_device()))
    return int(torch.cuda.current_stream(tensor.device).cuda_stream)


def _require_cuda_contiguous(*tensors: Any) -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("tensor must live on a CUDA device")
        if not t.is_contiguous():
            raise ValueError("tensor must be contiguous")


def stream_op(mode: str, dst: Any, src: Any, aux: Any | None = None, scale: float = 1.0, variant: str = "auto",
              blocks_per_sm: int = 0, stream: Any | None = None) -> Any:
    """dst = copy / scale / triad of src (and aux) -- the hbm benchmark's op
    (reference src/teamredbench/benchmarks/hbm.py:29-39), on the GPU."""
    _require_cuda_contiguous(dst, src, aux)
    if src.dtype != dst.dtype or (aux is not None and aux.dtype != src.dtype):
        raise ValueError("dst, src and aux must share one dtype")
    if src.numel() != dst.numel() or (aux is not None and aux.numel() != src.numel()):
        raise ValueError("dst, src and aux must have the same number of elements")
    if mode == "triad" and aux is None:
        raise ValueError("triad needs aux")
    _native.hbm_launch(trb_dtype(src), mode, dst.data_ptr(), src.data_ptr(),
                       aux.data_ptr() if aux is not None else None, src.numel(), float(scale), variant,
                       blocks_per_sm, _stream_handle(src, stream))
    return dst


def gemm(a: Any, b: Any, out: Any, *, dtype: str | None = None, scale_a: float = 1.0, scale_b: float = 1.0,
         splits: int = 0, cta_pair: int = -1, b_transposed: bool = False, stream: Any | None = None,
         tile_n: int = 0) -> Any:
    """out = a @ b on the tcgen05 kernel; a (m x k) and b (k x n) row-major.
    With b_transposed=True, `b` holds B^T as a row-major (n x k) tensor.

    dtype defaults to the tensors' dtype; pass ``dtype="tfloat32"`` to run
    float32 tensors on the tf32 tensor-core path (float32 itself runs as three
    tf32 products, float64 on the DMMA tensor path).  Output dtypes: bf16 for bf16 /
    e4m3 inputs, f16 for f16, f32 for tf32 and float32, f64 for float64, int32
    for int8.
    splits: 0 = automatic split-K, >= 1 forces that many K splits reduced
    through a global workspace, -2 / -4 / -8 that many splits reduced inside a
    thread-block cluster (distributed shared memory).
    cta_pair: -1 automatic, 0 single-CTA 128x256 kernel, 1 CTA-pair 256x256 kernel,
    2 CTA pair with 256x512 tiles (bf16 / f16 / e4m3 inputs, no split-K; bit-identical
    to cta_pair=1).
    tile_n: 0 automatic, 64/128/256 single-CTA tile width, -1 the
    swapped-operand skinny kernel (C^T = B^T A^T, m <= 64; automatic for
    m <= 64)."""
    _require_cuda_contiguous(a, b, out)
    if a.dim() != 2 or b.dim() != 2:
        raise ValueError(f"gemm operands must be 2-D, got {tuple(a.shape)} x {tuple(b.shape)}")
    m, k = a.shape
    n, bk = b.shape if b_transposed else reversed(b.shape)
    if bk != k:
        raise ValueError(f"incompatible shapes {tuple(a.shape)} x {tuple(b.shape)} (b_transposed={b_transposed})")
    if out.shape != (m, n):
        raise ValueError(f"out must be {(m, n)}, got {tuple(out.shape)}")
    name = dtype or trb_dtype(a)
    _native.gemm_launch_ex(name, m, n, k, a.data_ptr(), b.data_ptr(), out.data_ptr(), float(scale_a),
                           float(scale_b), int(splits), int(cta_pair), "k_major" if b_transposed else "row_major",
                           _stream_handle(a, stream), int(tile_n))
    return out
