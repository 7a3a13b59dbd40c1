"""GPU parity of the HBM stream kernels (through the C ABI) against the CPU
oracle and the reference-generated golden vectors.  Bit-exact throughout."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from tests.helpers import from_raw, to_raw, torch_dtype, uniform_pm1

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200 import _native  # noqa: E402
from teamredbench_b200.kernels import stream_op  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
FLOAT_DTYPES = ["float32", "bfloat16", "float16", "float64"]
VARIANTS = ["vec", "bulk"]


def _run(dtype, mode, b, c, scale, variant):
    dst = torch.empty_like(b)
    stream_op(mode, dst, b if mode != "scale" else c, c if mode == "triad" else None, scale, variant=variant)
    torch.cuda.synchronize()
    return dst


def _expected(dtype, mode, b, c, scale):
    src = to_raw(b if mode != "scale" else c)
    aux = to_raw(c) if mode == "triad" else None
    return oracle.hbm(dtype, mode, src, aux, scale)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("dtype", FLOAT_DTYPES)
def test_golden_vectors_through_c_abi(dtype, variant):
    g = np.load(GOLDEN / "hbm_golden.npz")
    b = from_raw(g[f"{dtype}/b"], dtype)
    c = from_raw(g[f"{dtype}/c"], dtype)
    assert np.array_equal(to_raw(_run(dtype, "copy", b, c, 1.0, variant)).view(np.uint8),
                          g[f"{dtype}/copy"].view(np.uint8))
    n = int(g["n"])
    for s in g["scales"]:
        s = float(s)
        got = to_raw(_run(dtype, "scale", b, c, s, variant))
        assert np.array_equal(got.view(np.uint8), g[f"{dtype}/scale/{s}"].view(np.uint8)), (dtype, s)
        got = to_raw(_run(dtype, "triad", b, c, s, variant))
        want = g[f"{dtype}/triad/{s}"]
        if dtype in ("bfloat16", "float16"):
            # torch's single-threaded scalar remainder (last n % 32 elements) uses a
            # different formula; the kernel follows torch's vector body everywhere.
            body = n - n % 32
            assert np.array_equal(got.view(np.uint16)[:body], want.view(np.uint16)[:body]), (dtype, s)
            assert np.array_equal(got, _expected(dtype, "triad", b, c, s)), (dtype, s)
        else:
            assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (dtype, s)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("mode", ["copy", "scale", "triad"])
@pytest.mark.parametrize("dtype", FLOAT_DTYPES)
def test_seeded_ragged_sizes_bit_exact(dtype, mode, variant):
    for n in (1, 7, 4099, (1 << 22) + 13):
        b, c = uniform_pm1(n, dtype, seed=n)
        for scale in (3.0, -0.37):
            got = to_raw(_run(dtype, mode, b, c, scale, variant))
            assert np.array_equal(got.view(np.uint8), _expected(dtype, mode, b, c, scale).view(np.uint8)), (n, scale)


@pytest.mark.parametrize("variant", ["vec", "bulk", "memcpy"])
def test_int8_copy(variant):
    b, _ = uniform_pm1(100003, "int8")
    got = _run("int8", "copy", b, b, 1.0, variant)
    assert torch.equal(got, b)


def test_int8_scale_is_skipped():
    b, _ = uniform_pm1(64, "int8")
    with pytest.raises(_native.NativeSkipped):
        _run("int8", "scale", b, b, 2.0, "vec")


def test_unaligned_pointers_take_scalar_path():
    base_b, base_c = uniform_pm1(10001, "float32")
    b, c = base_b[1:], base_c[1:]  # 4-byte offset: not 16-byte aligned
    dst = torch.empty(10001, device="cuda")[1:]
    stream_op("triad", dst, b, c, 3.0)
    torch.cuda.synchronize()
    want = oracle.hbm("float32", "triad", to_raw(b), to_raw(c), 3.0)
    assert np.array_equal(to_raw(dst), want)


def test_argument_errors():
    x = torch.zeros(16, device="cuda")
    with pytest.raises(_native.NativeError):
        _native.hbm_launch("float32", "triad", x.data_ptr(), x.data_ptr(), None, 16, 1.0)
    with pytest.raises(_native.NativeError):
        _native.hbm_launch("float32", "copy", x.data_ptr(), x.data_ptr(), None, 0, 1.0)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_baseline_full_size_triad_bit_exact(dtype):
    """BASELINE config: 2^30 elements, uniform[-1,1) seed 0, s = 3.0, full compare."""
    n = 1 << 30
    b, c = uniform_pm1(n, dtype, seed=0)
    dst = torch.empty_like(b)
    stream_op("triad", dst, b, c, 3.0)
    torch.cuda.synchronize()
    want = oracle.hbm(dtype, "triad", to_raw(b), to_raw(c), 3.0)
    got = to_raw(dst)
    del dst, b, c
    torch.cuda.empty_cache()
    assert np.array_equal(got, want)


def test_bulk_variant_full_size_copy_and_scale():
    n = 1 << 28
    b, c = uniform_pm1(n, "float32", seed=0)
    for mode in ("copy", "scale"):
        got = to_raw(_run("float32", mode, b, c, 3.0, "bulk"))
        assert np.array_equal(got, _expected("float32", mode, b, c, 3.0)), mode


@pytest.mark.parametrize("mode", ["copy", "scale", "triad"])
def test_host_entry_point_round_trip(mode):
    n = (1 << 25) + 5  # spans several 64 MiB pipeline chunks of f32
    b, c = uniform_pm1(n, "float32", seed=7)
    hb, hc = b.cpu().pin_memory(), c.cpu().pin_memory()
    hd = torch.empty_like(hb).pin_memory()
    src, aux = (hb, hc) if mode != "scale" else (hc, None)
    res = _native.hbm_host("float32", mode, hd.data_ptr(), src.data_ptr(), aux.data_ptr() if aux is not None else None,
                           n, 3.0)
    assert res.elapsed_s > 0 and res.device_error == 0
    want = oracle.hbm("float32", mode, src.numpy(), aux.numpy() if aux is not None else None, 3.0)
    assert np.array_equal(hd.numpy(), want)


def test_run_entry_point_reports_timing():
    res = _native.hbm_run("float32", "triad", 256 << 20, 2, 5, scale=3.0)
    assert res.elapsed_s > 0
    assert res.moved_bytes == 3 * (256 << 20)
    assert res.device_error == 0
    assert res.launches == 5
    res = _native.hbm_run("bfloat16", "copy", 64 << 20, 1, 2, variant="memcpy")
    assert res.implementation.decode() == "cudaMemcpyAsync_d2d"


def test_device_error_word_clear():
    assert _native.device_error(0, clear=True) == 0
