"""Builds libtpp_b200.so (all CUDA kernels + the C-ABI) in-tree for sm_100a.

Usage: python -m torchplusplus_b200.build [--force] [-j N]

Objects go to ``_build/`` at the repository root; the shared library is
written next to this file under ``_lib/`` so it travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIB_DIR = PKG / "_lib"
LIB = LIB_DIR / "libtpp_b200.so"
OBJ_DIR = ROOT / "_build" / "tpp_b200"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-v", "-I", str(INCLUDE)]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> tuple[Path, str]:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = r.stdout + r.stderr
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{log}")
    (OBJ_DIR / (src.stem + ".ptxas.txt")).write_text(log)
    if verbose:
        print(f"[tpp-build] {src.name}", file=sys.stderr)
    return obj, log


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile every kernel source and link the shared library (incremental)."""
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    hdrs = _headers()
    todo = [s for s in srcs if force or _stale(OBJ_DIR / (s.stem + ".o"), [s, *hdrs])]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda s: _compile(s, verbose), todo))
    objs = [OBJ_DIR / (s.stem + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda"
               if False else "-cudart=static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    print(build(force=a.force, jobs=a.j, verbose=True))


if __name__ == "__main__":
    main()
