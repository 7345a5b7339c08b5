"""Build the sm_100a C-ABI library ``agentserve_b200/lib/libagentserve_b200.so``.

Plain nvcc, no torch extension machinery: every ``csrc/*.cu`` is compiled with
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared library
whose exported symbols are exactly the ``extern "C"`` entry points declared in
``include/agentserve_b200.h``.  The library is built in-tree so that it travels
with the source tree.

Usage: ``python -m agentserve_b200.build [--force] [--verbose-ptxas]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "lib"
OBJ_DIR = PKG_DIR / "_build"
LIB_NAME = "libagentserve_b200.so"
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
    "--expt-relaxed-constexpr",
    "-I",
    str(INCLUDE),
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the agentserve_b200 CUDA library cannot be built")
    return cand


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> Path:
    """Compile (if stale) and return the path of the shared library."""
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = _headers()
    todo = [s for s in _sources()
            if force or verbose_ptxas or _stale(OBJ_DIR / (s.stem + ".o"), [s, *headers])]
    if todo:
        workers = min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            list(ex.map(lambda s: _compile(s, verbose_ptxas), todo))
    objs = [OBJ_DIR / (s.stem + ".o") for s in _sources()]
    if force or todo or _stale(LIB_PATH, objs):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
        if not quiet:
            print(f"built {LIB_PATH}")
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    build(force=args.force, verbose_ptxas=args.verbose_ptxas, quiet=False)


if __name__ == "__main__":
    main()
