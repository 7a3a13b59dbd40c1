"""The drop-in routes of the integration guide, driven by the reference's OWN
runtime and runner (CPU only; nothing here launches GPU work).

The reference reaches native kernels by spawning an executable with its flags
and parsing the last stdout line as JSON (src/teamredbench/native/runtime.py:
201-291; argv built at benchmarks/hbm.py:95-114 and benchmarks/mfu.py:107-125).
These tests import the reference package from a checkout named by the
TEAMREDBENCH_REFERENCE environment variable (default: a `reference` directory
beside this repository) and skip when there is none.  They check that:
  * route 1, an unchanged reference suite whose params.native.binary points at
    the B200 launchers, runs through the reference's run_suite: its argv is
    accepted and our JSON line becomes the reference's records, with this
    repository's nvidia_b200.yaml as the suite's hardware profile;
  * route 2, a one-line C++ shim registered under the reference's kernel names
    (hbm_hip / mfu_hipblas), is compiled by the reference's
    prepare_native_kernel_binary with g++ and execs the prebuilt launcher, so
    suites that name no binary at all run the B200 code.
Cases the launchers reject before any device work (int8 scale, an fp8 e5m2
GEMM) must come back as the reference's "skipped" records carrying our error
text.  On a host without a GPU every other case is skipped with "no CUDA device
visible"; with one, it must be "ok" and carry the reference's derived metrics.
"""
from __future__ import annotations

import os
import shutil
import sys
from pathlib import Path

import pytest

yaml = pytest.importorskip("yaml")

ROOT = Path(__file__).resolve().parent.parent
LIB = ROOT / "teamredbench_b200" / "lib"
HW_PROFILE = ROOT / "teamredbench_b200" / "configs" / "profiles" / "hardware" / "nvidia_b200.yaml"


def _reference_src() -> Path | None:
    base = Path(os.environ.get("TEAMREDBENCH_REFERENCE", ROOT.parent / "reference"))
    src = base / "src"
    return src if (src / "teamredbench" / "native" / "runtime.py").exists() else None


@pytest.fixture(scope="module")
def ref():
    src = _reference_src()
    if src is None:
        pytest.skip("no reference checkout (set TEAMREDBENCH_REFERENCE)")
    for exe in ("trb_hbm", "trb_mfu"):
        if not (LIB / exe).exists():
            pytest.skip(f"{exe} not built (python -m teamredbench_b200.build)")
    saved_path = list(sys.path)
    sys.path.insert(0, str(src))
    try:
        import teamredbench.builtin  # noqa: F401  (registers hbm_hip / mfu_hipblas and the benchmarks)
        import teamredbench.native.registry as registry
        import teamredbench.runner as runner
    except ImportError as exc:  # the reference's own dependencies are missing
        sys.path[:] = saved_path
        pytest.skip(f"reference package not importable: {exc}")
    saved_registry = dict(registry.NATIVE_KERNEL_REGISTRY)
    yield {"run_suite": runner.run_suite, "registry": registry}
    registry.NATIVE_KERNEL_REGISTRY.clear()
    registry.NATIVE_KERNEL_REGISTRY.update(saved_registry)
    sys.path[:] = saved_path
    for name in [m for m in sys.modules if m == "teamredbench" or m.startswith("teamredbench.")]:
        del sys.modules[name]


def _write_suite(tmp_path: Path, benchmarks: list[dict]) -> Path:
    runtime = tmp_path / "runtime.yaml"
    runtime.write_text(yaml.safe_dump({"name": "cuda-test", "rocm_version": "n/a", "libraries": {}, "env": {}}))
    suite = tmp_path / "suite.yaml"
    suite.write_text(yaml.safe_dump({
        "name": "b200-drop-in",
        "device": {"profile": str(HW_PROFILE)},
        "runtime": {"profile": str(runtime)},
        "outputs": {"directory": str(tmp_path / "results"), "formats": ["json"]},
        "benchmarks": benchmarks,
    }))
    return suite


def _hbm_case(native: dict) -> dict:
    return {"benchmark": "hbm", "params": {"backend": "native", "dtypes": ["float32", "int8"],
                                           "modes": ["copy", "scale"], "size_mib": 1, "warmup": 1,
                                           "iterations": 2, "scale": 3.0, "native": native}}


def _mfu_case(native: dict) -> dict:
    return {"benchmark": "mfu", "params": {"backend": "native", "dtypes": ["bfloat16", "float8_e5m2"],
                                           "shapes": [[256, 256, 256]], "warmup": 1, "iterations": 2,
                                           "native": native}}


def _check_records(records, gpu_visible_ok: bool = True):
    by_case = {(r.benchmark, r.dtype, r.case): r for r in records}
    # rejected by the launchers before any device work, whatever the host
    hbm_int8_scale = by_case[("hbm", "int8", "scale_1MiB")]
    assert hbm_int8_scale.status == "skipped"
    assert "unsupported dtype or mode for native HBM kernel" in (hbm_int8_scale.error or "")
    mfu_e5m2 = [r for (b, d, _), r in by_case.items() if b == "mfu" and d == "float8_e5m2"][0]
    assert mfu_e5m2.status == "skipped"
    assert "unsupported dtype for native MFU kernel: float8_e5m2" in (mfu_e5m2.error or "")
    for (bench, dtype, case), r in by_case.items():
        if r.status == "ok":
            assert r.metadata.get("backend_library") == "libtrb_b200", (bench, dtype, case)
            assert r.metrics.get("hbm_bandwidth_gbps" if bench == "hbm" else "achieved_tflops", 0) > 0
        else:
            assert r.status == "skipped", (bench, dtype, case, r.status)
            assert r.error, (bench, dtype, case)


def test_reference_suite_runs_b200_launchers_through_native_binary(ref, tmp_path):
    suite = _write_suite(tmp_path, [_hbm_case({"binary": str(LIB / "trb_hbm")}),
                                    _mfu_case({"binary": str(LIB / "trb_mfu")})])
    summary = ref["run_suite"](suite)
    assert len(summary.records) == 2 * 2 + 2
    _check_records(summary.records)


def test_reference_plugin_shim_compiled_by_reference_runtime(ref, tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    registry = ref["registry"]
    for name, bench, exe in (("hbm_hip", "hbm", "trb_hbm"), ("mfu_hipblas", "mfu", "trb_mfu")):
        shim = tmp_path / f"{exe}_shim.cpp"
        shim.write_text('#include <unistd.h>\n'
                        f'int main(int c, char** v) {{ v[0] = (char*)"{LIB / exe}"; execv(v[0], v); return 127; }}\n')
        registry.register_native_kernel(name=name, benchmark=bench, description=f"B200 {exe}", source_path=shim)
    native = {"compiler": gxx, "cache_dir": str(tmp_path / "native-cache")}  # no kernel/binary: the defaults
    suite = _write_suite(tmp_path, [_hbm_case(dict(native)), _mfu_case(dict(native))])
    summary = ref["run_suite"](suite)
    assert len(summary.records) == 2 * 2 + 2
    built = sorted(p.name for p in (tmp_path / "native-cache").iterdir())
    assert any(n.startswith("hbm_hip-") for n in built) and any(n.startswith("mfu_hipblas-") for n in built)
    _check_records(summary.records)
