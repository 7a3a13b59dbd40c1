"""Build recipe for the native backend (sm_100a only).

Produces, in-tree under ``teamredbench_b200/lib/``:
    libtrb_b200.so  -- the C-ABI library (include/trb_b200.h)
    trb_hbm, trb_mfu -- launcher executables that keep the reference's
                        argv / last-line-JSON contract

``python -m teamredbench_b200.build`` or ``build()`` from Python.  nvcc
cross-compiles without a GPU.  Objects are rebuilt only when a source or
header is newer than the object.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
OBJ_DIR = LIB_DIR / "obj"
INCLUDE = ROOT / "include"

CUDA_SOURCES = ["trb_abi.cu", "hbm_stream.cu", "gemm_tcgen05.cu", "gemm_fp64.cu"]
HEADERS = [CSRC / "trb_common.cuh", INCLUDE / "trb_b200.h"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
              f"-I{INCLUDE}", "-Xptxas", "-warn-spills"]

LIBRARY = LIB_DIR / "libtrb_b200.so"
EXECUTABLES = {"trb_hbm": "TRB_BENCH_HBM", "trb_mfu": "TRB_BENCH_MFU"}


def find_nvcc() -> str:
    for candidate in (os.environ.get("TEAMREDBENCH_NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return str(candidate)
    raise RuntimeError("nvcc not found; set TEAMREDBENCH_NVCC")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    completed = subprocess.run(cmd, capture_output=True, text=True)
    if completed.returncode != 0:
        raise RuntimeError(f"command failed ({completed.returncode}): {' '.join(cmd)}\n{completed.stdout}\n{completed.stderr}")
    return completed.stdout + completed.stderr


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = find_nvcc()
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    jobs = []
    for src in CUDA_SOURCES:
        obj = OBJ_DIR / (Path(src).stem + ".o")
        if ptxas_verbose or _stale(obj, [CSRC / src, *HEADERS]):
            jobs.append([nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-c", str(CSRC / src), "-o", str(obj)])
    logs: list[str] = []
    if jobs:
        with ThreadPoolExecutor(max_workers=len(jobs)) as pool:
            logs = list(pool.map(lambda cmd: _run(cmd, verbose), jobs))
    if ptxas_verbose:
        for log in logs:
            print(log)
    objs = [OBJ_DIR / (Path(s).stem + ".o") for s in CUDA_SOURCES]
    if _stale(LIBRARY, objs):
        _run([nvcc, *ARCH_FLAGS, "-shared", "-o", str(LIBRARY), *map(str, objs)], verbose)
    main_src = CSRC / "trb_native_main.cpp"
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    for exe, define in EXECUTABLES.items():
        target = LIB_DIR / exe
        if _stale(target, [main_src, INCLUDE / "trb_b200.h", LIBRARY]):
            _run([cxx, "-O2", "-std=c++17", f"-D{define}", f"-I{INCLUDE}", str(main_src), "-o", str(target),
                  f"-L{LIB_DIR}", "-ltrb_b200", "-Wl,-rpath,$ORIGIN"], verbose)
    return LIBRARY


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv)
    print(f"built {LIBRARY}")
