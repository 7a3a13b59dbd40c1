"""The C-ABI library loads (no GPU needed), exports every entry point that
include/trb_b200.h declares, and its structs have the layout the ctypes
binding assumes (checked against a gcc-compiled probe of the header)."""
import re
import subprocess
from pathlib import Path

import pytest

from teamredbench_b200 import _native

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "trb_b200.h"


def _declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:int|const char\*)\s+(trb_\w+)\s*\(", text, flags=re.MULTILINE))


def test_header_declarations_match_binding():
    assert _declared_functions() == set(_native.EXPORTED_SYMBOLS)


def test_library_loads_and_exports_every_symbol():
    lib = _native.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    assert lib.trb_abi_version() == 1
    assert _native.last_error() == ""


def test_struct_layout_matches_c(tmp_path: Path):
    probe = tmp_path / "probe.c"
    probe.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "trb_b200.h"\n'
                     'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(trb_result), '
                     'offsetof(trb_result, implementation), sizeof(trb_hbm_args), offsetof(trb_hbm_args, scale), '
                     'sizeof(trb_gemm_args), offsetof(trb_result, launches), sizeof(trb_gemm_options), '
                     'offsetof(trb_gemm_options, b_layout), offsetof(trb_gemm_options, tile_n)); return 0;}\n')
    exe = tmp_path / "probe"
    subprocess.run(["gcc", f"-I{ROOT / 'include'}", str(probe), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    import ctypes

    assert got == [ctypes.sizeof(_native.TrbResult), _native.TrbResult.implementation.offset,
                   ctypes.sizeof(_native.HbmArgs), _native.HbmArgs.scale.offset, ctypes.sizeof(_native.GemmArgs),
                   _native.TrbResult.launches.offset, ctypes.sizeof(_native.GemmOptions),
                   _native.GemmOptions.b_layout.offset, _native.GemmOptions.tile_n.offset]


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setattr(_native, "LIBRARY_PATH", tmp_path / "absent.so")
    with pytest.raises(_native.NativeLibraryMissing):
        _native.load()


def test_launcher_reports_skipped_json_on_bad_input():
    """The launcher's argv/JSON contract on inputs rejected before any device work."""
    for exe, args in ((_native.HBM_EXECUTABLE, ["--dtype", "float32", "--mode", "bogus"]),
                      (_native.MFU_EXECUTABLE, ["--dtype", "float64", "--m", "64", "--n", "64", "--k", "64"]),
                      (_native.HBM_EXECUTABLE, ["--size-mib"])):
        done = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=60)
        assert done.returncode == 0
        import json

        payload = json.loads(done.stdout.strip().splitlines()[-1])
        assert payload["status"] == "skipped" and payload["error"]


_MFU_SHAPE = ["--dtype", "bfloat16", "--m", "64", "--n", "64", "--k", "64"]


@pytest.mark.parametrize("exe_name, args, error", [
    # mfu_gemm_common.hip.hpp:92-104: unknown keys, non-positive sizes, negative counts
    ("mfu", ["--dtype", "bfloat16", "--m", "0", "--n", "64", "--k", "64"], "matrix dimensions must be positive"),
    ("mfu", ["--dtype", "bfloat16", "--m", "64", "--n", "-1", "--k", "64"], "matrix dimensions must be positive"),
    ("mfu", _MFU_SHAPE + ["--warmup", "-1"], "warmup and iterations must be non-negative"),
    ("mfu", _MFU_SHAPE + ["--iterations", "-1"], "warmup and iterations must be non-negative"),
    ("mfu", _MFU_SHAPE + ["--blocks-per-cu", "-1"], "blocks-per-cu must be non-negative"),
    ("mfu", _MFU_SHAPE + ["--bogus", "1"], "unknown argument --bogus"),
    # hbm_bandwidth.hip.cpp:139-162: unknown keys and missing values
    ("hbm", ["--dtype", "float32", "--mode", "triad", "--bogus", "1"], "unknown argument --bogus"),
    ("hbm", ["--dtype", "float32", "--mode", "triad", "--warmup"], "missing value for argument --warmup"),
    # an addition: the reference parses --size-mib 0 and goes on to an empty launch
    ("hbm", ["--dtype", "float32", "--mode", "triad", "--size-mib", "0"], "size-mib must be positive"),
])
def test_launcher_argument_errors_match_reference(exe_name, args, error):
    """Rejected argv gives the reference's skipped record and message, exit 0, no device work."""
    import json

    exe = _native.MFU_EXECUTABLE if exe_name == "mfu" else _native.HBM_EXECUTABLE
    done = subprocess.run([str(exe), *args], capture_output=True, text=True, timeout=60)
    assert done.returncode == 0
    payload = json.loads(done.stdout.strip().splitlines()[-1])
    assert payload == {"status": "skipped", "error": error}
