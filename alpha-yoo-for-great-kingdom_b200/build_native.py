"""Build libgk.so (all CUDA kernels + the C ABI) for sm_100a with nvcc.

Objects go to ``_build/`` beside this file and the shared library to
``kingdom_ai/libgk.so`` so it travels with the source tree. Sources are
compiled in parallel; an object is rebuilt only when its source or a header
is newer.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIBRARY = HERE / "kingdom_ai" / "libgk.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def _headers():
    return list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(source: Path, verbose: bool) -> Path:
    obj = BUILD / (source.stem + ".o")
    if _stale(obj, [source, *_headers()]):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=max(1, min(len(sources), os.cpu_count() or 4))) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    if _stale(LIBRARY, objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
