"""Build ``theorem_b200/libtheorem_b200.so`` from ``theorem_b200/csrc/*.cu`` for sm_100a.

Each translation unit is compiled with nvcc (``-gencode
arch=compute_100a,code=sm_100a -lineinfo -O3``) into ``theorem_b200/_build/``
in parallel, then linked into one shared library with a plain C ABI
(``include/theorem_b200.h``). cudart is linked statically so the library
depends only on the CUDA driver at run time. Objects are rebuilt when their
source or any header under ``csrc/`` or ``include/`` is newer.

    python -m theorem_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libtheorem_b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", str(INCLUDE), "-I", str(CSRC)]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build theorem_b200)")
    return cand


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, ptxas_v: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link the shared library."""
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    hdr = _headers_mtime()
    todo = []
    for s in srcs:
        obj = BUILD / (s.stem + ".o")
        if force or ptxas_v or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, hdr):
            todo.append(s)
    logs = []
    if todo:
        with ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose, ptxas_v), todo):
                logs.append((obj.name, log))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if todo or force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if ptxas_v:
        for name, log in logs:
            print(f"== {name}\n{log}")
    return LIB


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--force", action="store_true")
    p.add_argument("--verbose", action="store_true")
    p.add_argument("--ptxas-v", action="store_true", help="print registers / spills / smem per kernel")
    a = p.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_v=a.ptxas_v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
