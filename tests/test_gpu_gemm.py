"""GPU parity of the tcgen05 GEMM (through the C ABI) against the fp64 CPU
oracle and the reference-generated torch golden vectors.

Pass rule: max|C - ref| <= tol * max|ref| (the reference harness's metric,
tests/native/gemm_parity.hip.cpp:163-178) with tol = 1e-2 for bf16 / f16 /
e4m3, 1e-5 for tf32, 1e-4 for float32 and 1e-10 for float64; int8 must be
bit-exact."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle
from tests.helpers import (GEMM_OUT, GEMM_TOLERANCE, from_raw, gemm_operands, gemm_result_f64,
                           to_raw, torch_dtype)

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from teamredbench_b200 import _native  # noqa: E402
from teamredbench_b200.kernels import gemm  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = ["bfloat16", "float16", "tfloat32", "float8_e4m3fn", "int8"]


def _run(name, a, b, sa=1.0, sb=1.0, splits=0, cta_pair=-1):
    m, n = a.shape[0], b.shape[1]
    out = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
    gemm(a, b, out, dtype=name, scale_a=sa, scale_b=sb, splits=splits, cta_pair=cta_pair)
    torch.cuda.synchronize()
    return out


def _check(name, a, b, c, sa, sb, rows, tol=None):
    ref = oracle.gemm_rows(name, to_raw(a), to_raw(b), rows, sa, sb)
    got = gemm_result_f64(name, c)[rows]
    if name == "int8":
        assert np.array_equal(got.astype(np.int64), ref.astype(np.int64))
        return 0.0
    err = oracle.rel_to_max_error(got, ref)
    assert err <= (tol if tol is not None else GEMM_TOLERANCE[name]), (name, err)
    return err


@pytest.mark.parametrize("key", ["square/bfloat16", "square/float16", "square/tfloat32", "square/float8_e4m3fn",
                                 "square/int8", "square/float32", "square/float64", "ragged/bfloat16"])
def test_golden_vectors(key):
    g = np.load(GOLDEN / "gemm_golden.npz")
    name = key.split("/")[1]
    m, n, k = (int(v) for v in g[f"{key}/shape"])
    a = from_raw(g[f"{key}/a"].reshape(m, k), name if name != "tfloat32" else "float32")
    b = from_raw(g[f"{key}/b"].reshape(k, n), name if name != "tfloat32" else "float32")
    sa, sb = (float(x) for x in g[f"{key}/scales"]) if name == "float8_e4m3fn" else (1.0, 1.0)
    c = _run(name, a, b, sa, sb)
    golden = g[f"{key}/c"].reshape(m, n)
    got = gemm_result_f64(name, c)
    if name == "int8":
        assert np.array_equal(got.astype(np.int64), golden.astype(np.int64))
    else:
        want = (oracle.bf16_to_f32(golden) if GEMM_OUT[name] == "bfloat16" else golden).astype(np.float64)
        assert oracle.rel_to_max_error(got, want) <= GEMM_TOLERANCE[name]
    _check(name, a, b, c, sa, sb, np.arange(m))


@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("shape", [(128, 256, 128), (256, 512, 1024), (1024, 1024, 1024), (300, 528, 208),
                                   (1, 16, 16), (129, 272, 144)])
def test_shapes_full_compare(name, shape):
    m, n, k = shape
    if (n * (4 if name == "tfloat32" else 2 if name in ("bfloat16", "float16") else 1)) % 16:
        pytest.skip("row stride not 16-byte aligned")
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=m + n + k)
    c = _run(name, a, b, sa, sb)
    _check(name, a, b, c, sa, sb, np.arange(m))


@pytest.mark.parametrize("name", ["bfloat16", "float16", "float8_e4m3fn", "int8"])
def test_baseline_8192_sampled_rows(name):
    """BASELINE mixed-dtype sweep shape M=N=K=8192, 48 sampled rows vs fp64."""
    m = n = k = 8192
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=0)
    c = _run(name, a, b, sa, sb)
    rows = np.random.default_rng(0).choice(m, size=48, replace=False)
    _check(name, a, b, c, sa, sb, np.sort(rows))


@pytest.mark.parametrize("cta_pair", [-1, 0])
def test_baseline_8192_tf32_within_1e5(cta_pair):
    """BASELINE tf32 at M = N = K = 8192 against the fp64 oracle, bound 1e-5.
    One fp32 accumulation chain over K = 8192 measures 2.2e-5 on B200 (cuBLAS's
    tf32 GEMM too); the kernels accumulate chains of 2048 K elements in TMEM
    and fold them in fp32, which measures ~5e-6."""
    m = n = k = 8192
    a, b, _, _ = gemm_operands("tfloat32", m, n, k, seed=0)
    c = _run("tfloat32", a, b, cta_pair=cta_pair)
    rows = np.sort(np.random.default_rng(0).choice(m, size=48, replace=False))
    err = _check("tfloat32", a, b, c, 1.0, 1.0, rows)
    print(f"tf32 8192^3 (cta_pair {cta_pair}) rel-to-max error {err:.3e}")


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (1024, 1024, 16384), (256, 384, 12288), (2048, 512, 6144)])
def test_tf32_long_k_chains_within_1e5(shape):
    """K >= 4096 through every automatic kernel choice (pair, single CTA,
    workspace split-K at very long K), each within 1e-5 of the fp64 oracle,
    and deterministic."""
    m, n, k = shape
    a, b, _, _ = gemm_operands("tfloat32", m, n, k, seed=k + m)
    c1 = _run("tfloat32", a, b)
    c2 = _run("tfloat32", a, b)
    assert torch.equal(c1, c2)
    rows = np.arange(m) if m <= 256 else np.sort(np.random.default_rng(2).choice(m, 64, replace=False))
    _check("tfloat32", a, b, c1, 1.0, 1.0, rows)


def test_baseline_16384_bf16_sampled_rows():
    """The largest square shape of the BASELINE bf16 sweep (16384^3), 48 sampled
    rows against the fp64 oracle."""
    m = n = k = 16384
    a, b, sa, sb = gemm_operands("bfloat16", m, n, k, seed=0)
    c = _run("bfloat16", a, b, sa, sb)
    rows = np.sort(np.random.default_rng(16384).choice(m, size=48, replace=False))
    _check("bfloat16", a, b, c, sa, sb, rows)
    del a, b, c
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("shape,splits", [((128, 256, 1024), 4), ((300, 528, 2048), 3), ((16, 8192, 8192), 4),
                                          ((1024, 768, 4096), 8), ((129, 272, 144), 2)])
def test_split_k_fixup(name, shape, splits):
    """Split-K partials summed by the last CTA of each tile, vs the oracle; the
    result is deterministic across launches (and bit-exact for int8)."""
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=11)
    c1 = _run(name, a, b, sa, sb, splits=splits)
    c2 = _run(name, a, b, sa, sb, splits=splits)
    assert torch.equal(c1, c2)
    rows = np.arange(m) if m <= 512 else np.sort(np.random.default_rng(1).choice(m, 64, replace=False))
    _check(name, a, b, c1, sa, sb, rows, tol=GEMM_TOLERANCE[name])


@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("cta_pair", [0, 1])
@pytest.mark.parametrize("shape,splits", [((300, 528, 208), 1), ((520, 784, 1024), 1), ((1, 16, 16), 1),
                                          ((257, 272, 512), 3), ((384, 1024, 2048), 0)])
def test_single_cta_and_pair_kernels(name, cta_pair, shape, splits):
    """Both kernel shapes (1 CTA 128x256 / CTA pair 256x256), ragged M / N / K
    tails, with and without split-K, against the oracle."""
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=m * 7 + n)
    c = _run(name, a, b, sa, sb, splits=splits, cta_pair=cta_pair)
    _check(name, a, b, c, sa, sb, np.arange(m))


def test_pair_and_single_agree_bitwise_for_int8():
    a, b, _, _ = gemm_operands("int8", 1000, 1040, 3008, seed=9)
    assert torch.equal(_run("int8", a, b, cta_pair=0), _run("int8", a, b, cta_pair=1))


@pytest.mark.parametrize("name", ["bfloat16", "float16", "float8_e4m3fn"])
@pytest.mark.parametrize("b_transposed", [False, True])
@pytest.mark.parametrize("shape", [(300, 528, 208), (520, 1104, 1024), (1, 16, 16), (768, 1536, 4096),
                                   (2048, 4096, 512)])
def test_wide_pair_kernel_matches_pair_bitwise(name, b_transposed, shape):
    """cta_pair = 2, the CTA pair with 256 x 512 tiles: each accumulator sums its
    k-blocks in the pair kernel's order with the same instructions, so the bits
    agree; ragged M / N / K tails, a tile whose second half lies past N, and
    several tiles per SM pair (the accumulator handed from tile to tile)."""
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=m + 3 * n)
    bb = b.t().contiguous() if b_transposed else b
    outs = []
    for cta_pair in (1, 2):
        out = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
        gemm(a, bb, out, dtype=name, scale_a=sa, scale_b=sb, splits=1, cta_pair=cta_pair, b_transposed=b_transposed)
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    rows = np.unique(np.linspace(0, m - 1, min(m, 64)).astype(np.int64))
    _check(name, a, b, outs[1], sa, sb, rows)


def test_wide_pair_kernel_option_errors():
    x = torch.zeros((512, 512), device="cuda", dtype=torch.float32)
    with pytest.raises(_native.NativeError, match="cta_pair = 2"):  # tf32 folds K chunks: the pair kernel's job
        gemm(x, x, torch.empty_like(x), dtype="tfloat32", cta_pair=2)
    y = torch.zeros((512, 512), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_native.NativeError, match="cta_pair = 2"):  # whole tiles only
        gemm(y, y, torch.empty_like(y), splits=2, cta_pair=2)
    z = torch.zeros((512, 512), device="cuda", dtype=torch.int8)
    with pytest.raises(_native.NativeError, match="cta_pair = 2"):  # 32-bit results do not fit in registers
        gemm(z, z, torch.empty((512, 512), device="cuda", dtype=torch.int32), dtype="int8", cta_pair=2)


def test_split_k_run_entry_reports_splits():
    res = _native.gemm_run("bfloat16", 16, 1024, 8192, 1, 3)  # 8 swapped panels x clusters of 8 K splits
    assert res.split_k == 8 and res.device_error == 0
    assert res.implementation.decode() == "tcgen05_swap_128x16_cluster8"
    res = _native.gemm_run("bfloat16", 16, 8192, 8192, 1, 3)  # 64 panels x clusters of 2
    assert res.split_k == 2 and res.implementation.decode() == "tcgen05_swap_128x16_cluster2"
    res = _native.gemm_run("bfloat16", 128, 8192, 8192, 1, 3)  # 64 tiles x clusters of 2 K splits
    assert res.split_k == 2 and res.implementation.decode() == "tcgen05_1cta_128x128_cluster2"
    res = _native.gemm_run("bfloat16", 4096, 4096, 4096, 1, 3)
    assert res.split_k == 1 and res.implementation.decode() == "tcgen05_cta_pair_256x512"
    res = _native.gemm_run("float8_e4m3fn", 4096, 4096, 4096, 1, 3)
    assert res.split_k == 1 and res.implementation.decode() == "tcgen05_cta_pair_256x256"


@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("shape", [(16, 8192, 8192), (128, 8192, 4096), (77, 2064, 3072), (64, 1024, 8192),
                                   (1, 512, 2048)])
@pytest.mark.parametrize("b_transposed", [False, True])
def test_skinny_narrow_tiles(name, shape, b_transposed):
    """M <= 128: narrow single-CTA tiles (BN = 64, 8-bit MN-major B: 128), with
    split-K on top when even those leave SMs idle (small N)."""
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=n + k)
    c = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
    bb = b.t().contiguous() if b_transposed else b
    gemm(a, bb, c, dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed)
    torch.cuda.synchronize()
    _check(name, a, b, c, sa, sb, np.arange(m), tol=GEMM_TOLERANCE[name])


@pytest.mark.parametrize("m", [16, 128])
def test_baseline_skinny_shapes(m):
    a, b, sa, sb = gemm_operands("bfloat16", m, 8192, 8192, seed=1)
    c = _run("bfloat16", a, b)
    _check("bfloat16", a, b, c, 1.0, 1.0, np.arange(m))


@pytest.mark.parametrize("size", [2048, 4096])
def test_baseline_square_bf16_sweep_sampled(size):
    a, b, _, _ = gemm_operands("bfloat16", size, size, size, seed=0)
    c = _run("bfloat16", a, b)
    rows = np.random.default_rng(size).choice(size, size=64, replace=False)
    _check("bfloat16", a, b, c, 1.0, 1.0, np.sort(rows))


def test_repeated_launches_are_deterministic():
    a, b, _, _ = gemm_operands("bfloat16", 1024, 2048, 512, seed=3)
    first = _run("bfloat16", a, b)
    for _ in range(3):
        assert torch.equal(_run("bfloat16", a, b), first)


def test_host_entry_point():
    m, n, k = 512, 768, 384
    a, b, _, _ = gemm_operands("bfloat16", m, n, k, seed=5)
    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    res = _native.gemm_host("bfloat16", m, n, k, ha.data_ptr(), hb.data_ptr(), hc.data_ptr())
    assert res.elapsed_s > 0 and res.device_error == 0
    _check("bfloat16", a, b, hc, 1.0, 1.0, np.arange(m))


def test_alignment_and_dtype_errors():
    a = torch.zeros((64, 20), device="cuda", dtype=torch.bfloat16)  # 40-byte rows
    b = torch.zeros((20, 64), device="cuda", dtype=torch.bfloat16)
    out = torch.empty((64, 64), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_native.NativeError):
        gemm(a, b, out)
    x = torch.zeros((64, 64), device="cuda", dtype=torch.int32)
    with pytest.raises(_native.NativeSkipped):
        gemm(x, x, torch.empty_like(x), dtype="int32")
    d = torch.zeros(64 * 64 + 1, device="cuda", dtype=torch.float64)
    with pytest.raises(_native.NativeError):  # float64 needs 8-byte aligned operands
        _native.gemm_launch("float64", 64, 64, 64, d.data_ptr() + 4, d.data_ptr(), d.data_ptr())


def test_run_entry_point_reports_timing():
    res = _native.gemm_run("bfloat16", 2048, 2048, 2048, 1, 3)
    assert res.elapsed_s > 0 and res.achieved_ops == 2 * 2048 ** 3 and res.device_error == 0
    res = _native.gemm_run("float8_e4m3fn", 1024, 1024, 1024, 1, 2)
    assert res.elapsed_s > 0 and res.device_error == 0


# ---------------------------------------------------------------------------
# float32 (three tf32 products on the tensor cores) and float64 (CUDA cores):
# the reference's native mfu covers float16/bfloat16/float32/float64
# (src/teamredbench/native/kernels/mfu_gemm.hip.cpp:9-21).
# ---------------------------------------------------------------------------
HIGH_PRECISION = ["float32", "float64"]


@pytest.mark.parametrize("name", HIGH_PRECISION)
@pytest.mark.parametrize("shape", [(128, 256, 128), (256, 512, 1024), (300, 528, 208), (1, 16, 16),
                                   (129, 272, 144), (1024, 1024, 4096)])
@pytest.mark.parametrize("b_transposed", [False, True])
def test_high_precision_shapes(name, shape, b_transposed):
    m, n, k = shape
    a, b, _, _ = gemm_operands(name, m, n, k, seed=m + n + k)
    c = torch.empty((m, n), device="cuda", dtype=torch_dtype(name))
    gemm(a, b.t().contiguous() if b_transposed else b, c, dtype=name, b_transposed=b_transposed)
    torch.cuda.synchronize()
    _check(name, a, b, c, 1.0, 1.0, np.arange(m))


@pytest.mark.parametrize("shape", [(77, 131, 61), (1, 1, 1), (3, 5, 7), (130, 129, 257), (513, 95, 33)])
@pytest.mark.parametrize("b_transposed", [False, True])
def test_float64_ragged_unaligned_shapes(shape, b_transposed):
    """float64 has no TMA stride rule: any m, n, k, only 8-byte alignment (odd
    rows take the 8-byte copy path)."""
    m, n, k = shape
    a, b, _, _ = gemm_operands("float64", m, n, k, seed=m * n + k)
    c = torch.empty((m, n), device="cuda", dtype=torch.float64)
    gemm(a, b.t().contiguous() if b_transposed else b, c, b_transposed=b_transposed)
    torch.cuda.synchronize()
    # the DMMA tensor path rounds like fp64 FMAs: a few ulps from the oracle's
    # k-ordered fma chain, far inside the reference's 1e-10
    _check("float64", a, b, c, 1.0, 1.0, np.arange(m), tol=1e-14)


def test_float64_matches_cublas_dgemm():
    a, b, _, _ = gemm_operands("float64", 1000, 1100, 900, seed=4)
    c = torch.empty((1000, 1100), device="cuda", dtype=torch.float64)
    gemm(a, b, c)
    ref = a @ b
    assert torch.allclose(c, ref, rtol=0, atol=1e-13 * float(ref.abs().max()))


@pytest.mark.parametrize("name", HIGH_PRECISION)
def test_high_precision_baseline_8192_sampled_rows(name):
    m = n = k = 8192
    a, b, _, _ = gemm_operands(name, m, n, k, seed=0)
    c = _run(name, a, b)
    rows = np.sort(np.random.default_rng(1).choice(m, size=32, replace=False))
    # float32 at K = 8192 measures ~2.1e-5: the split removes the input
    # rounding, what is left is the tensor core's fp32 accumulation over the
    # long K (a single tf32 product on tf32-exact inputs, and cuBLAS's, show
    # the same 2.2e-5); the reference's float bound 1e-4 holds.
    _check(name, a, b, c, 1.0, 1.0, rows)


def test_float32_beats_single_tf32_accuracy():
    """The split keeps the low bits a single tf32 product drops."""
    m, n, k = 256, 512, 2048
    a, b, _, _ = gemm_operands("float32", m, n, k, seed=9)
    c3 = _run("float32", a, b)
    c1 = torch.empty_like(c3)
    gemm(a, b, c1, dtype="tfloat32")   # tf32 path truncates the inputs' low 13 bits
    torch.cuda.synchronize()
    ref = oracle.gemm_rows("float64", to_raw(a).astype(np.float64), to_raw(b).astype(np.float64), np.arange(m))
    e3 = oracle.rel_to_max_error(gemm_result_f64("float32", c3), ref)
    e1 = oracle.rel_to_max_error(gemm_result_f64("float32", c1), ref)
    assert e3 < 1e-5 and e3 * 20 < e1, (e3, e1)


@pytest.mark.parametrize("name", HIGH_PRECISION)
def test_high_precision_run_entry(name):
    res = _native.gemm_run(name, 2048, 2048, 2048, 1, 2)
    assert res.elapsed_s > 0 and res.device_error == 0 and res.achieved_ops == 2 * 2048 ** 3
    impl = res.implementation.decode()
    if name == "float32":
        assert impl.startswith("fp32x3_tcgen05") and res.launches == 3 * 2, (impl, res.launches)
    else:
        assert impl == "fp64_dmma_128x128" and res.launches == 2, (impl, res.launches)


@pytest.mark.parametrize("name", HIGH_PRECISION)
def test_high_precision_host_entry(name):
    m, n, k = 384, 640, 320
    a, b, _, _ = gemm_operands(name, m, n, k, seed=12)
    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.empty((m, n), dtype=torch_dtype(name)).pin_memory()
    res = _native.gemm_host(name, m, n, k, ha.data_ptr(), hb.data_ptr(), hc.data_ptr())
    assert res.device_error == 0
    _check(name, a, b, hc, 1.0, 1.0, np.arange(m))


# ---------------------------------------------------------------------------
# Swapped-operand skinny kernel (M <= 64): C^T = B^T A^T with the rows of A as
# the MMA's N (16 / 32 / 64).
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("shape", [(1, 256, 512), (16, 8192, 8192), (17, 640, 1024), (32, 4096, 2048),
                                   (48, 1040, 4096), (64, 2048, 8192), (5, 144, 96)])
@pytest.mark.parametrize("b_transposed", [False, True])
@pytest.mark.parametrize("splits", [0, 1, 5])
def test_swap_kernel(name, shape, b_transposed, splits):
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=3 * m + n + k)
    bb = b.t().contiguous() if b_transposed else b
    out = lambda: torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))  # noqa: E731
    c1, c2 = out(), out()
    for c in (c1, c2):
        gemm(a, bb, c, dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed, splits=splits, tile_n=-1)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)  # deterministic, split-K included
    num_kb = -(-k * b.element_size() // 128)
    per_split = k if splits <= 1 else k * -(-num_kb // splits) // num_kb
    _check(name, a, b, c1, sa, sb, np.arange(m), tol=GEMM_TOLERANCE[name])


@pytest.mark.parametrize("b_transposed", [False, True])
def test_swap_and_tile_kernels_agree_bitwise_for_int8(b_transposed):
    a, b, _, _ = gemm_operands("int8", 40, 2048, 4096, seed=2)
    bb = b.t().contiguous() if b_transposed else b
    outs = []
    for kw in ({"tile_n": -1}, {"tile_n": 128}, {"cta_pair": 1}):
        c = torch.empty((40, 2048), device="cuda", dtype=torch.int32)
        gemm(a, bb, c, b_transposed=b_transposed, **kw)
        outs.append(c)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_swap_kernel_is_automatic_for_m_le_64_and_validates_options():
    a, b, _, _ = gemm_operands("bfloat16", 65, 512, 256, seed=1)
    c = torch.empty((65, 512), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(_native.NativeError):
        gemm(a, b, c, tile_n=-1)  # the swapped kernel takes m <= 64
    with pytest.raises(_native.NativeError):
        gemm(a, b, c, tile_n=96)
    gemm(a, b, c, tile_n=64)
    torch.cuda.synchronize()
    _check("bfloat16", a, b, c, 1.0, 1.0, np.arange(65))
    res = _native.gemm_run("float8_e4m3fn", 64, 4096, 4096, 1, 2)
    assert res.implementation.decode().startswith("tcgen05_swap_128x64") and res.device_error == 0
    res = _native.gemm_run("float32", 32, 4096, 4096, 1, 2)
    assert res.implementation.decode().startswith("fp32x3_tcgen05_swap_128x32") and res.device_error == 0


@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("shape", [(16, 8192, 8192), (32, 1024, 4096), (64, 2048, 2048), (5, 256, 1024),
                                   (48, 528, 3072)])
@pytest.mark.parametrize("cluster", [2, 4, 8])
@pytest.mark.parametrize("b_transposed", [False, True])
def test_swap_cluster_split_k(name, shape, cluster, b_transposed):
    """Cluster split-K (partials reduced through distributed shared memory)
    against the oracle, and bit-identical to the workspace split-K with the
    same split count (same K partition, same summation order)."""
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=m + 2 * n + k)
    bb = b.t().contiguous() if b_transposed else b
    c_cl = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
    c_ws = torch.empty_like(c_cl)
    num_kb = -(-k * b.element_size() // 128)
    kbps = -(-num_kb // cluster)
    if (cluster - 1) * kbps >= num_kb:
        with pytest.raises(_native.NativeError):
            gemm(a, bb, c_cl, dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed, tile_n=-1, splits=-cluster)
        return
    gemm(a, bb, c_cl, dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed, tile_n=-1, splits=-cluster)
    gemm(a, bb, c_ws, dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed, tile_n=-1, splits=cluster)
    torch.cuda.synchronize()
    assert torch.equal(c_cl, c_ws)
    _check(name, a, b, c_cl, sa, sb, np.arange(m), tol=GEMM_TOLERANCE[name])  # splitting only shortens the chains


@pytest.mark.parametrize("name", DTYPES)
@pytest.mark.parametrize("shape", [(128, 8192, 8192), (100, 2048, 4096), (65, 528, 3072), (256, 1024, 2048),
                                   (129, 272, 1024)])
@pytest.mark.parametrize("cluster", [2, 4, 8])
@pytest.mark.parametrize("b_transposed", [False, True])
@pytest.mark.parametrize("tile_n", [256, 128])
def test_tile_kernel_cluster_split_k(name, shape, cluster, b_transposed, tile_n):
    """Cluster split-K of the 128 x 256 / 128 x 128 single-CTA kernel (column
    blocks of the tile reduced through distributed shared memory) vs the
    oracle, and bit-identical to the workspace split-K with the same split
    count."""
    m, n, k = shape
    a, b, sa, sb = gemm_operands(name, m, n, k, seed=m + 3 * n + k)
    bb = b.t().contiguous() if b_transposed else b
    c_cl = torch.empty((m, n), device="cuda", dtype=torch_dtype(GEMM_OUT[name]))
    c_ws = torch.empty_like(c_cl)
    num_kb = -(-k * b.element_size() // 128)
    kbps = -(-num_kb // cluster)
    kw = dict(dtype=name, scale_a=sa, scale_b=sb, b_transposed=b_transposed, cta_pair=0, tile_n=tile_n)
    if (cluster - 1) * kbps >= num_kb or (tile_n // cluster) % 32:
        with pytest.raises(_native.NativeError):
            gemm(a, bb, c_cl, splits=-cluster, **kw)
        return
    gemm(a, bb, c_cl, splits=-cluster, **kw)
    gemm(a, bb, c_ws, splits=cluster, **kw)
    torch.cuda.synchronize()
    assert torch.equal(c_cl, c_ws)
    rows = np.arange(m) if m <= 256 else np.sort(np.random.default_rng(0).choice(m, 128, replace=False))
    _check(name, a, b, c_cl, sa, sb, rows, tol=GEMM_TOLERANCE[name])  # splitting only shortens the chains


def test_cluster_split_k_option_errors():
    a, b, _, _ = gemm_operands("bfloat16", 128, 512, 256, seed=1)  # 4 k-blocks
    c = torch.empty((128, 512), device="cuda", dtype=torch.bfloat16)
    for kw in ({"splits": -3}, {"splits": -8}, {"splits": -2, "cta_pair": 1}, {"splits": -2, "tile_n": 64},
               {"splits": -8, "tile_n": 128}):
        with pytest.raises(_native.NativeError):
            gemm(a, b, c, **kw)


@pytest.mark.parametrize("size,impl", [(1024, "tcgen05_1cta_128x64"), (1536, "tcgen05_1cta_128x128"),
                                       (2048, "tcgen05_1cta_128x256"), (3072, "tcgen05_cta_pair_256x256"),
                                       (8192, "tcgen05_cta_pair_256x512"), (16384, "tcgen05_cta_pair_256x512")])
def test_automatic_kernel_choice_for_square_sizes(size, impl):
    """The wave model's picks for the BASELINE square sweep (tiles that fill
    the SMs in whole waves; the pair once the grid is large; its 256 x 512
    tiles for bf16 once K reaches 64 k-blocks)."""
    res = _native.gemm_run("bfloat16", size, size, size, 0, 1)
    assert res.implementation.decode() == impl and res.split_k == 1 and res.device_error == 0


@pytest.mark.parametrize("name,shape,impl", [("float8_e4m3fn", (8192, 8192, 8192), "tcgen05_cta_pair_256x256"),
                                             ("bfloat16", (8192, 8192, 2048), "tcgen05_cta_pair_256x256"),
                                             ("float16", (8192, 8192, 8192), "tcgen05_cta_pair_256x512"),
                                             ("bfloat16", (8192, 8448, 4096), "tcgen05_cta_pair_256x256")])
def test_automatic_wide_pair_rule(name, shape, impl):
    """The 256 x 512 pair is picked for bf16 / f16 with >= 64 k-blocks when its
    tiles fill the SM pairs as well as 256 x 256 ones; e4m3, short K and a
    width that wastes part of a 512-wide tile keep the 256 x 256 pair."""
    m, n, k = shape
    res = _native.gemm_run(name, m, n, k, 0, 1)
    assert res.implementation.decode() == impl and res.device_error == 0


@pytest.mark.parametrize("shape", [(1024, 1024, 1024), (1536, 1536, 1536), (2048, 2048, 2048)])
def test_small_square_auto_choice_matches_oracle(shape):
    m, n, k = shape
    a, b, _, _ = gemm_operands("bfloat16", m, n, k, seed=k)
    c = _run("bfloat16", a, b)
    _check("bfloat16", a, b, c, 1.0, 1.0, np.sort(np.random.default_rng(k).choice(m, 96, replace=False)))
