"""Build the sm_100a C-ABI library ``libria_attention.so`` in-tree with nvcc.

The library is plain CUDA C++ behind ``extern "C"`` entry points (declared in
``include/ria_attention.h``); no torch extension machinery is involved, so the
built ``.so`` travels with the source tree and is loaded with ``ctypes``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_ROOT = PKG_DIR.parent  # router-ia_b200/
REPO_ROOT = SRC_ROOT.parent
CSRC = SRC_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_DIR = PKG_DIR / "lib"
LIB_NAME = "libria_attention.so"
LIB_PATH = LIB_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the router-ia B200 library needs the CUDA 12.9 toolkit to build")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libria_attention.so``."""
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    obj_dir = SRC_ROOT / "_build"
    obj_dir.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    nvcc = nvcc_path()
    objs: list[Path] = []
    procs: list[tuple[subprocess.Popen, Path]] = []
    max_jobs = jobs or max(1, min(8, os.cpu_count() or 1))
    for src in sources():
        obj = obj_dir / (src.stem + ".o")
        objs.append(obj)
        if not force and not _stale(obj, [src, *headers]):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        while len(procs) >= max_jobs:
            _reap(procs)
        procs.append((subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True), src))
    while procs:
        _reap(procs)
    if force or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link of {LIB_NAME} failed:\n{res.stdout}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def _reap(procs: list[tuple[subprocess.Popen, Path]]) -> None:
    proc, src = procs.pop(0)
    out, _ = proc.communicate()
    if proc.returncode != 0:
        for p, _s in procs:
            p.kill()
        raise RuntimeError(f"nvcc failed on {src.name}:\n{out}")
    if out and out.strip():
        sys.stdout.write(out)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB_PATH)
