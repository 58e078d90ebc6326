"""Build `lib/libdecodek.so`, the C-ABI library of the sm_100a decode kernels.

    python llm-decode-kernels_b200/build.py [--force] [--debug]

Each `csrc/*.cu` is compiled by nvcc for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`,
`-lineinfo`, IEEE fp32 division and square root, no fast-math) into `_build/`, then linked into one
shared library with the CUDA runtime linked statically. The library lands in-tree, next to the
Python package that loads it, so a copy of the repository carries it to the GPU machine.
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
LIB = PKG / "lib" / "libdecodek.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the decodek library needs the CUDA toolkit to build")


def _flags(debug: bool) -> list[str]:
    f = ARCH + ["-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE), "-I", str(CSRC),
                "--expt-relaxed-constexpr", "-diag-suppress", "177"]
    f += ["-O0", "-G"] if debug else ["-O3"]
    return f


def _stale(obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    flags = _flags(debug)
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, [src, *headers, Path(__file__)]):
            cmd = [cc, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    if force or _stale(LIB, objs):
        tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
        cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.debug, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
