"""ctypes binding of libtrb_b200.so (declared in include/trb_b200.h).

This is the only way the Python package reaches the GPU.  There is no CPU or
library fallback: if the shared library is missing, every call raises
``NativeLibraryMissing`` (build it with ``python -m teamredbench_b200.build``).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_DIR = PKG / "lib"
LIBRARY_PATH = LIB_DIR / "libtrb_b200.so"
HBM_EXECUTABLE = LIB_DIR / "trb_hbm"
MFU_EXECUTABLE = LIB_DIR / "trb_mfu"

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
VARIANT_CODES = {"auto": 0, "vec": 1, "bulk": 2, "memcpy": 3}
VARIANT_NAMES = {v: k for k, v in VARIANT_CODES.items()}

TRB_OK = 0
TRB_SKIPPED = 1

# Every symbol include/trb_b200.h declares.
EXPORTED_SYMBOLS = (
    "trb_abi_version",
    "trb_last_error",
    "trb_device_error",
    "trb_hbm_run",
    "trb_hbm_launch",
    "trb_hbm_host",
    "trb_gemm_run",
    "trb_gemm_launch",
    "trb_gemm_launch_ex",
    "trb_gemm_launch_noalloc",
    "trb_gemm_host",
    "trb_round_tf32",
    "trb_selftest_bounded_wait",
)


class NativeLibraryMissing(RuntimeError):
    pass


class NativeError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"libtrb_b200 status {status}: {message}")
        self.status = status
        self.message = message


class NativeSkipped(NativeError):
    """Unsupported dtype / mode / shape (the reference's status "skipped")."""


class TrbResult(ctypes.Structure):
    _fields_ = [
        ("elapsed_s", ctypes.c_double),
        ("moved_bytes", ctypes.c_double),
        ("achieved_ops", ctypes.c_double),
        ("h2d_bytes", ctypes.c_double),
        ("d2h_bytes", ctypes.c_double),
        ("device_id", ctypes.c_int32),
        ("sm_count", ctypes.c_int32),
        ("grid", ctypes.c_int32),
        ("block", ctypes.c_int32),
        ("blocks_per_sm", ctypes.c_int32),
        ("variant", ctypes.c_int32),
        ("device_error", ctypes.c_int32),
        ("launches", ctypes.c_int32),
        ("split_k", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("implementation", ctypes.c_char * 64),
    ]

    def as_dict(self) -> dict:
        out = {name: getattr(self, name) for name, _ in self._fields_}
        out["implementation"] = self.implementation.decode()
        return out


class HbmArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("variant", ctypes.c_int32),
        ("device_id", ctypes.c_int32),
        ("size_bytes", ctypes.c_uint64),
        ("warmup", ctypes.c_int32),
        ("iterations", ctypes.c_int32),
        ("scale", ctypes.c_double),
        ("blocks_per_sm", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("m", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("k", ctypes.c_int32),
        ("warmup", ctypes.c_int32),
        ("iterations", ctypes.c_int32),
        ("device_id", ctypes.c_int32),
        ("b_layout", ctypes.c_int32),
    ]


class GemmOptions(ctypes.Structure):
    _fields_ = [
        ("splits", ctypes.c_int32),
        ("cta_pair", ctypes.c_int32),
        ("b_layout", ctypes.c_int32),
        ("tile_n", ctypes.c_int32),
    ]


B_LAYOUTS = {"row_major": 0, "k_major": 1}


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load (once) and type the library; raise NativeLibraryMissing if absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY_PATH.exists():
        raise NativeLibraryMissing(
            f"{LIBRARY_PATH} not found: build the native backend with `python -m teamredbench_b200.build`"
        )
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    vp, u64, i32, dbl, flt = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_double, ctypes.c_float
    res_p = ctypes.POINTER(TrbResult)
    lib.trb_abi_version.argtypes = []
    lib.trb_abi_version.restype = i32
    lib.trb_last_error.argtypes = []
    lib.trb_last_error.restype = ctypes.c_char_p
    lib.trb_device_error.argtypes = [i32, i32]
    lib.trb_device_error.restype = i32
    lib.trb_hbm_run.argtypes = [ctypes.POINTER(HbmArgs), res_p]
    lib.trb_hbm_run.restype = i32
    lib.trb_hbm_launch.argtypes = [i32, i32, vp, vp, vp, u64, dbl, i32, i32, vp]
    lib.trb_hbm_launch.restype = i32
    lib.trb_hbm_host.argtypes = [i32, i32, vp, vp, vp, u64, dbl, i32, res_p]
    lib.trb_hbm_host.restype = i32
    lib.trb_gemm_run.argtypes = [ctypes.POINTER(GemmArgs), res_p]
    lib.trb_gemm_run.restype = i32
    lib.trb_gemm_launch.argtypes = [i32, i32, i32, i32, vp, vp, vp, flt, flt, vp]
    lib.trb_gemm_launch.restype = i32
    lib.trb_gemm_launch_ex.argtypes = [i32, i32, i32, i32, vp, vp, vp, flt, flt, ctypes.POINTER(GemmOptions), vp]
    lib.trb_gemm_launch_ex.restype = i32
    lib.trb_gemm_launch_noalloc.argtypes = [i32, i32, i32, i32, vp, vp, vp, flt, flt, i32, vp]
    lib.trb_gemm_launch_noalloc.restype = i32
    lib.trb_gemm_host.argtypes = [i32, i32, i32, i32, vp, vp, vp, flt, flt, i32, res_p]
    lib.trb_gemm_host.restype = i32
    lib.trb_round_tf32.argtypes = [vp, u64, vp]
    lib.trb_round_tf32.restype = i32
    lib.trb_selftest_bounded_wait.argtypes = [ctypes.c_uint32, i32, res_p]
    lib.trb_selftest_bounded_wait.restype = i32
    _lib = lib
    return lib


def last_error() -> str:
    return (load().trb_last_error() or b"").decode(errors="replace")


def check(status: int) -> int:
    if status == TRB_OK:
        return status
    message = last_error()
    if status > 0:
        raise NativeSkipped(status, message)
    raise NativeError(status, message)


def hbm_run(dtype: str, mode: str, size_bytes: int, warmup: int, iterations: int, device_id: int = 0,
            scale: float = 1.0, variant: str = "auto", blocks_per_sm: int = 0) -> TrbResult:
    args = HbmArgs(DTYPE_CODES[dtype], MODE_CODES[mode], VARIANT_CODES[variant], device_id, size_bytes, warmup,
                   iterations, scale, blocks_per_sm, 0)
    result = TrbResult()
    check(load().trb_hbm_run(ctypes.byref(args), ctypes.byref(result)))
    return result


def hbm_launch(dtype: str, mode: str, dst: int, src: int, aux: int | None, count: int, scale: float,
               variant: str = "auto", blocks_per_sm: int = 0, stream: int = 0) -> None:
    check(load().trb_hbm_launch(DTYPE_CODES[dtype], MODE_CODES[mode], dst, src, aux, count, scale,
                                VARIANT_CODES[variant], blocks_per_sm, stream or None))


def hbm_host(dtype: str, mode: str, dst: int, src: int, aux: int | None, count: int, scale: float,
             device_id: int = 0) -> TrbResult:
    result = TrbResult()
    check(load().trb_hbm_host(DTYPE_CODES[dtype], MODE_CODES[mode], dst, src, aux, count, scale, device_id,
                              ctypes.byref(result)))
    return result


def gemm_run(dtype: str, m: int, n: int, k: int, warmup: int, iterations: int, device_id: int = 0,
             b_layout: str = "row_major") -> TrbResult:
    args = GemmArgs(DTYPE_CODES[dtype], m, n, k, warmup, iterations, device_id, B_LAYOUTS[b_layout])
    result = TrbResult()
    check(load().trb_gemm_run(ctypes.byref(args), ctypes.byref(result)))
    return result


def gemm_launch(dtype: str, m: int, n: int, k: int, a: int, b: int, c: int, scale_a: float = 1.0,
                scale_b: float = 1.0, stream: int = 0) -> None:
    check(load().trb_gemm_launch(DTYPE_CODES[dtype], m, n, k, a, b, c, scale_a, scale_b, stream or None))


def gemm_launch_ex(dtype: str, m: int, n: int, k: int, a: int, b: int, c: int, scale_a: float = 1.0,
                   scale_b: float = 1.0, splits: int = 0, cta_pair: int = -1, b_layout: str = "row_major",
                   stream: int = 0, tile_n: int = 0) -> None:
    opts = GemmOptions(splits, cta_pair, B_LAYOUTS[b_layout], tile_n)
    check(load().trb_gemm_launch_ex(DTYPE_CODES[dtype], m, n, k, a, b, c, scale_a, scale_b, ctypes.byref(opts),
                                    stream or None))


def gemm_launch_noalloc(dtype: str, m: int, n: int, k: int, a: int, b: int, c: int, scale_a: float = 1.0,
                        scale_b: float = 1.0, splits: int = 0, stream: int = 0) -> None:
    """Split-K GEMM whose scratch is a fixed array in the library (no device
    allocation); see trb_gemm_launch_noalloc in include/trb_b200.h."""
    check(load().trb_gemm_launch_noalloc(DTYPE_CODES[dtype], m, n, k, a, b, c, scale_a, scale_b, splits,
                                         stream or None))


def gemm_host(dtype: str, m: int, n: int, k: int, a: int, b: int, c: int, scale_a: float = 1.0,
              scale_b: float = 1.0, device_id: int = 0) -> TrbResult:
    result = TrbResult()
    check(load().trb_gemm_host(DTYPE_CODES[dtype], m, n, k, a, b, c, scale_a, scale_b, device_id,
                               ctypes.byref(result)))
    return result


def round_tf32(data: int, count: int, stream: int = 0) -> None:
    check(load().trb_round_tf32(data, count, stream or None))


def selftest_bounded_wait(limit_us: int, device_id: int = 0) -> tuple[int, TrbResult, str]:
    """Run the bounded-wait self-test kernel (trb_selftest_bounded_wait);
    returns (status, result, last error message) without raising, since the
    expected status is TRB_ERR_DEVICE_TIMEOUT."""
    result = TrbResult()
    status = load().trb_selftest_bounded_wait(limit_us, device_id, ctypes.byref(result))
    return status, result, last_error()


def device_error(device_id: int = 0, clear: bool = False) -> int:
    status = load().trb_device_error(device_id, int(clear))
    if status < 0:
        check(status)
    return status
