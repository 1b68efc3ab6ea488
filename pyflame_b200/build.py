"""Build libpyflame_cuda.so in-tree.

C++ host sources are compiled with g++, CUDA sources with nvcc for sm_100a
(`-gencode arch=compute_100a,code=sm_100a -lineinfo`), and everything is
linked into `pyflame_b200/lib/libpyflame_cuda.so` against the static CUDA
runtime (the library does not need libcuda to load; the driver is reached at
run time) and NVRTC.  Objects are cached under `pyflame_b200/_build/` and
rebuilt when a source or header is newer.

Usage: python -m pyflame_b200.build [--force] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libpyflame_cuda.so"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

CXXFLAGS = ["-O2", "-g", "-fPIC", "-std=c++17", "-Wall", "-Wno-unused-function", "-fvisibility=hidden",
            f"-I{CUDA}/include"]
NVCCFLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
             "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", f"-I{CUDA}/include",
             "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def _sources():
    cpp = sorted(CSRC.glob("*.cpp"))
    cu = sorted((CSRC / "kernels").glob("*.cu"))
    return cpp, cu


def _headers():
    hs = list(CSRC.rglob("*.hpp")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, hdr_time: float):
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "_") + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time):
        return obj, ""
    if src.suffix == ".cu":
        cmd = [str(CUDA / "bin" / "nvcc"), *NVCCFLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = ["g++", *CXXFLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, jobs: int = 8, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    cpp, cu = _sources()
    hdr = _headers()
    with cf.ThreadPoolExecutor(max_workers=jobs) as pool:
        results = list(pool.map(lambda s: _compile(s, force, hdr), cpp + cu))
    objs = [o for o, _ in results]
    if verbose:
        for o, log in results:
            if log:
                print(f"--- {o.name}\n{log}", file=sys.stderr)
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = ["g++", "-shared", "-o", str(LIB), *map(str, objs), f"-L{CUDA}/lib64", "-lcudart_static", "-lnvrtc",
               "-ldl", "-lpthread", "-lrt", f"-Wl,-rpath,{CUDA}/lib64", "-Wl,--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.v))


if __name__ == "__main__":
    main()
