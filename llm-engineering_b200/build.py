"""Build the sm_100a C-ABI library ``libb200paged.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled for ``-gencode arch=compute_100a,code=sm_100a``
into ``_build/`` and linked (static cudart) into ``libb200paged.so`` next to this file,
so the library travels with the source tree and is found without an install step.
Rebuilds are incremental on file modification times (sources and headers).
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_NAME = "libb200paged.so"
LIB_PATH = PKG_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    f"-I{REPO_DIR / 'include'}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libb200paged.so")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((REPO_DIR / "include").glob("*.h"))


def _compile(nvcc: str, src: Path, obj: Path, verbose_ptxas: bool) -> str:
    cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return proc.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    """Compile every CUDA source and link the shared library; return its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    header_mtime = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = []
    objects = []
    for src in sources:
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        stale = (
            force
            or verbose_ptxas
            or not obj.exists()
            or obj.stat().st_mtime < max(src.stat().st_mtime, header_mtime)
        )
        if stale:
            todo.append((src, obj))
    logs: dict[str, str] = {}
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            futures = {pool.submit(_compile, nvcc, s, o, verbose_ptxas): s for s, o in todo}
            for fut in concurrent.futures.as_completed(futures):
                logs[futures[fut].name] = fut.result()
    relink = (
        bool(todo)
        or not LIB_PATH.exists()
        or LIB_PATH.stat().st_mtime < max(o.stat().st_mtime for o in objects)
    )
    if relink:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects), "-lcuda"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            # libcuda.so is only needed for the driver API symbols that are resolved
            # through cudaGetDriverEntryPoint; link without it when the stub is absent.
            cmd = cmd[:-1]
            proc = subprocess.run(cmd, capture_output=True, text=True)
            if proc.returncode != 0:
                raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB_PATH)
    if verbose_ptxas:
        for name, log in sorted(logs.items()):
            print(f"== {name}\n{log}")
    return LIB_PATH


if __name__ == "__main__":
    import sys

    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print(LIB_PATH)
