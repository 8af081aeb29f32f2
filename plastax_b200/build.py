"""Build libpxb.so, the sm_100a edge-arena kernels behind the C ABI (include/pxb.h).

Each ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` (``-gencode
arch=compute_100a,code=sm_100a``) into ``_build/``, and the objects are linked
into ``plastax_b200/libpxb.so`` with the CUDA runtime linked statically, so
the library loads beside any PyTorch build. The build is incremental: an
object is rebuilt when its source or a shared header is newer.

Run as ``python -m plastax_b200.build`` (or through ``__graft_entry__.build``).
"""

from __future__ import annotations

import concurrent.futures
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libpxb.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    """The nvcc binary: $CUDA_HOME/bin/nvcc, else the one on PATH."""
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = pathlib.Path(home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _headers() -> list[pathlib.Path]:
    return [*CSRC.glob("*.cuh"), ROOT / "include" / "pxb.h"]


def _stale(target: pathlib.Path, deps: list[pathlib.Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: pathlib.Path) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    if _stale(obj, [src, *_headers()]):
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stderr}")
    return obj


def build(verbose: bool = False) -> pathlib.Path:
    """Compile and link libpxb.so; returns its path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objs = list(pool.map(_compile, sources))
    if _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "--cudart", "static", "-o", str(LIB), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link of libpxb.so failed:\n{proc.stderr}")
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
