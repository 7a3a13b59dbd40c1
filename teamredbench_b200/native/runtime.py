"""Resolve, build, cache and run native kernel executables.

The boundary contract is the reference's (src/teamredbench/native/runtime.py:
65-291): a native kernel is an executable that receives the benchmark's CLI
flags and prints one JSON object as its last non-empty stdout line,
    {"status": "ok"|"skipped", "raw_metrics": {...}, "metadata": {...}, "error": ...}
Sources are compiled once into a cache keyed by a SHA-256 over the source, its
local #includes (recursively), the benchmark, kernel name, compiler and flags.

B200 changes: the compiler is nvcc (TEAMREDBENCH_NVCC, params.native.compiler,
PATH, /usr/local/cuda/bin/nvcc); definitions may carry a prebuilt binary; and
every run has a timeout (params.native.timeout_s, default 900 s) so that a
stuck process becomes a NativeKernelError instead of hanging the suite.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
import shutil
import subprocess
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from teamredbench_b200.native.registry import get_native_kernel

DEFAULT_TIMEOUT_S = 900.0
B200_ARCH_ARGS = ("-gencode", "arch=compute_100a,code=sm_100a")


class NativeKernelError(RuntimeError):
    pass


@dataclass(frozen=True)
class ResolvedNativeKernel:
    benchmark: str
    name: str
    description: str
    source_path: Path | None = None
    binary_path: Path | None = None
    compiler: str | None = None
    compile_args: tuple[str, ...] = ()
    run_args: tuple[str, ...] = ()
    env: dict[str, str] = field(default_factory=dict)
    cache_dir: Path | None = None
    timeout_s: float = DEFAULT_TIMEOUT_S


@dataclass(frozen=True)
class NativeKernelResult:
    status: str
    raw_metrics: dict[str, Any]
    metadata: dict[str, Any]
    error: str | None = None


def _as_list(value: Any, label: str) -> list[str]:
    if value is None:
        return []
    if not isinstance(value, list):
        raise ValueError(f"{label} must be a list of strings.")
    return [str(v) for v in value]


def _as_mapping(value: Any, label: str) -> dict[str, str]:
    if value is None:
        return {}
    if not isinstance(value, dict):
        raise ValueError(f"{label} must be a mapping.")
    return {str(k): str(v) for k, v in value.items()}


def _user_path(base: Path, target: str) -> Path:
    p = Path(target)
    return p if p.is_absolute() else (base / p).resolve()


def resolve_native_kernel(*, benchmark: str, params: dict[str, Any], suite_path: Path | None,
                          repo_root: Path | None, default_kernel: str | None = None) -> ResolvedNativeKernel:
    native = params.get("native") or {}
    if not isinstance(native, dict):
        raise ValueError("benchmark params.native must be a mapping.")
    base = suite_path.parent if suite_path else (repo_root or Path.cwd())
    name = str(native.get("kernel", default_kernel or "")).strip() or None
    definition = get_native_kernel(name) if name else None
    if definition is not None and definition.benchmark != benchmark:
        raise ValueError(f"Native kernel {definition.name} is registered for {definition.benchmark}, not {benchmark}.")

    source = definition.source_path if definition is not None else None
    binary = definition.binary_path if definition is not None else None
    if native.get("source"):
        source, binary = _user_path(base, str(native["source"])), None
    if native.get("binary"):
        binary = _user_path(base, str(native["binary"]))
    if source is None and binary is None:
        if name is None:
            raise ValueError("No native kernel configured. Set params.native.kernel, params.native.source, "
                             "or params.native.binary.")
        raise ValueError(f"Native kernel {name} does not define a source or binary path.")

    compile_args = list(definition.compile_args if definition is not None else ())
    compile_args += _as_list(native.get("compile_args"), "native.compile_args")
    return ResolvedNativeKernel(
        benchmark=benchmark,
        name=name or (source.stem if source else binary.stem),
        description=definition.description if definition is not None else "external native kernel",
        source_path=source,
        binary_path=binary,
        compiler=str(native["compiler"]) if native.get("compiler") else None,
        compile_args=tuple(compile_args),
        run_args=tuple(_as_list(native.get("run_args"), "native.run_args")),
        env=_as_mapping(native.get("env"), "native.env"),
        cache_dir=_user_path(base, str(native["cache_dir"])) if native.get("cache_dir") else None,
        timeout_s=float(native.get("timeout_s", DEFAULT_TIMEOUT_S)),
    )


def native_cache_dir(explicit: Path | None = None) -> Path:
    if explicit is not None:
        return explicit
    xdg = os.environ.get("XDG_CACHE_HOME")
    root = Path(xdg).expanduser().resolve() if xdg else Path.home().resolve() / ".cache"
    return root / "teamredbench" / "native"


def clear_native_cache(explicit: Path | None = None) -> tuple[Path, int]:
    cache = native_cache_dir(explicit)
    if not cache.exists():
        return cache, 0
    removed = 0
    for entry in cache.iterdir():
        if entry.is_dir():
            shutil.rmtree(entry)
        else:
            entry.unlink()
        removed += 1
    return cache, removed


def _find_cuda_compiler(preferred: str | None = None) -> str:
    for candidate in (preferred, os.environ.get("TEAMREDBENCH_NVCC"), "nvcc", "/usr/local/cuda/bin/nvcc"):
        if not candidate:
            continue
        path = Path(candidate)
        if path.is_absolute():
            if path.exists():
                return str(path)
            continue
        found = shutil.which(candidate)
        if found:
            return found
    raise NativeKernelError("No CUDA compiler found. Set TEAMREDBENCH_NVCC, params.native.compiler, "
                            "or params.native.binary.")


_INCLUDE_RE = re.compile(r'^\s*#\s*include\s*"([^"]+)"', re.MULTILINE)


def _digest_source(digest: "hashlib._Hash", path: Path, seen: set[Path]) -> None:
    path = path.resolve()
    if path in seen:
        return
    seen.add(path)
    digest.update(str(path).encode() + b"\0")
    digest.update(path.read_bytes())
    for include in _INCLUDE_RE.findall(path.read_text(encoding="utf-8", errors="ignore")):
        child = (path.parent / include).resolve()
        if child.exists():
            _digest_source(digest, child, seen)


def prepare_native_kernel_binary(kernel: ResolvedNativeKernel) -> Path:
    if kernel.binary_path is not None:
        if not kernel.binary_path.exists():
            raise NativeKernelError(f"Native kernel binary does not exist: {kernel.binary_path}")
        return kernel.binary_path
    if kernel.source_path is None:
        raise NativeKernelError(f"Native kernel {kernel.name} is missing both source_path and binary_path.")
    if not kernel.source_path.exists():
        raise NativeKernelError(f"Native kernel source does not exist: {kernel.source_path}")

    compiler = _find_cuda_compiler(kernel.compiler)
    cache = native_cache_dir(kernel.cache_dir)
    cache.mkdir(parents=True, exist_ok=True)
    digest = hashlib.sha256()
    _digest_source(digest, kernel.source_path, set())
    for part in (kernel.benchmark, kernel.name, compiler, *kernel.compile_args):
        digest.update(part.encode())
    target = cache / f"{kernel.name}-{digest.hexdigest()[:16]}"
    if target.exists():
        return target
    args = list(kernel.compile_args)
    if Path(compiler).name.startswith("nvcc") and not any("arch=" in a or a.startswith("-arch") for a in args):
        args = [*B200_ARCH_ARGS, *args]
    command = [compiler, "-O3", "-std=c++17", str(kernel.source_path), "-o", str(target), *args]
    completed = subprocess.run(command, check=False, capture_output=True, text=True)
    if completed.returncode != 0:
        error = completed.stderr.strip() or completed.stdout.strip() or "unknown compiler failure"
        raise NativeKernelError(f"Failed to compile native kernel {kernel.name}: {error}")
    target.chmod(0o755)
    return target


def _parse_native_result(stdout: str) -> NativeKernelResult:
    lines = [line.strip() for line in stdout.splitlines() if line.strip()]
    if not lines:
        raise NativeKernelError("Native kernel produced no JSON output.")
    try:
        payload = json.loads(lines[-1])
    except json.JSONDecodeError as exc:
        raise NativeKernelError(f"Native kernel output was not valid JSON: {exc}") from exc
    if not isinstance(payload, dict):
        raise NativeKernelError("Native kernel output JSON must be an object.")
    raw, meta = payload.get("raw_metrics", {}), payload.get("metadata", {})
    if not isinstance(raw, dict):
        raise NativeKernelError("Native kernel raw_metrics must be a JSON object.")
    if not isinstance(meta, dict):
        raise NativeKernelError("Native kernel metadata must be a JSON object.")
    return NativeKernelResult(status=str(payload.get("status", "ok")), raw_metrics=dict(raw), metadata=dict(meta),
                              error=str(payload["error"]) if payload.get("error") is not None else None)


def run_native_kernel(kernel: ResolvedNativeKernel, args: list[str]) -> NativeKernelResult:
    binary = prepare_native_kernel_binary(kernel)
    env = {**os.environ, **kernel.env}
    try:
        completed = subprocess.run([str(binary), *args, *kernel.run_args], check=False, capture_output=True,
                                   text=True, env=env, timeout=kernel.timeout_s)
    except subprocess.TimeoutExpired as exc:
        raise NativeKernelError(f"Native kernel {kernel.name} timed out after {kernel.timeout_s:.0f} s") from exc
    if completed.returncode != 0:
        error = completed.stderr.strip() or completed.stdout.strip() or "native kernel process failed"
        raise NativeKernelError(f"Native kernel {kernel.name} failed: {error}")
    return _parse_native_result(completed.stdout)
