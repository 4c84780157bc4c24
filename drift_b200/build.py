"""Builds libdrift_cuda.so in-tree from drift_b200/csrc/*.cu for sm_100a.

    python -m drift_b200.build [--verbose]

Each source compiles to its own object under drift_b200/_build/ (in parallel,
only when the source or a header changed), then one nvcc link makes
drift_b200/libdrift_cuda.so. The flags are the B200's and nothing else:
-gencode arch=compute_100a,code=sm_100a -lineinfo -O3, IEEE division and
square root (no fast math: the kernels' results are checked against a CPU
oracle).
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PACKAGE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PACKAGE)
SOURCES = os.path.join(PACKAGE, "csrc")
BUILD = os.path.join(PACKAGE, "_build")
LIBRARY = os.path.join(PACKAGE, "libdrift_cuda.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"),
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libdrift_cuda")
    return found


def _headers() -> list[str]:
    return (glob.glob(os.path.join(SOURCES, "*.cuh"))
            + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _compile(source: str, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(source).replace(".cu", ".o"))
    newest = max([os.path.getmtime(source)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj
    cmd = [nvcc(), *FLAGS, "-c", source, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(source)}:\n"
                           f"{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(SOURCES, "*.cu")))
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    newest = max(os.path.getmtime(o) for o in objects)
    if not os.path.exists(LIBRARY) or os.path.getmtime(LIBRARY) < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-o", LIBRARY + ".tmp", *objects]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(LIBRARY + ".tmp", LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv))
