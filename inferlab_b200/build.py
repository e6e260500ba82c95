"""Builds libinferlab_attention_cuda.so in-tree with nvcc for sm_100a.

    python -m inferlab_b200.build [--force] [--jobs N]

Each .cu file under csrc/ compiles to an object in csrc/_build/ (rebuilt when
it or any header is newer), then one shared library is linked into
inferlab_b200/lib/. cudart is linked statically, so the library needs only the
driver at run time. This is the nvcc step a worker/build.rs would run for the
Rust worker.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(CSRC, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIBNAME = "libinferlab_attention_cuda.so"
LIBPATH = os.path.join(LIBDIR, LIBNAME)
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-Wall", "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and os.path.exists(candidate):
            return candidate
    raise RuntimeError("nvcc not found")


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    mtime = os.path.getmtime(target)
    return any(os.path.getmtime(src) > mtime for src in sources)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = _headers()
    compiler = nvcc()
    objects = []
    commands = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objects.append(obj)
        if force or _stale(obj, [src] + headers):
            commands.append([compiler, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-c", src, "-o", obj])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{result.stdout}\n{result.stderr}")
        return result.stderr

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as pool:
        for log in pool.map(run, commands):
            if log and verbose:
                print(log, file=sys.stderr)
    if force or commands or _stale(LIBPATH, objects):
        run([compiler, *ARCH, "-shared", "-o", LIBPATH, *objects, "-lpthread"])
    return LIBPATH


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    parser.add_argument("-v", "--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    main()
