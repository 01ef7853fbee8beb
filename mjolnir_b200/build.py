"""Build libmjolnir_b200.so (sm_100a) in-tree with nvcc.

    python -m mjolnir_b200.build [--force] [-v]

Every CUDA source compiles to its own object in parallel (the decode kernels
are split one translation unit per KV format, inst_<format>.cu), then the
objects link into the shared library. The library is written next to this
file so it travels with the source tree; nothing is installed into
site-packages and there is no JIT cache.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libmjolnir_b200.so")
OBJ_DIR = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

COMPILE = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
    "-I", os.path.join(ROOT, "include"),
]
LINK = ["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _newer(target: str, deps) -> bool:
    """True when `target` is missing or older than any of `deps`."""
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(f) > t for f in deps)


def _obj(src: str) -> str:
    return os.path.join(OBJ_DIR, os.path.basename(src)[:-3] + ".o")


def build(force: bool = False, verbose: bool = False) -> str:
    srcs, hdrs = sources(), headers()
    if not force and not _newer(LIB, srcs + hdrs):
        return LIB
    os.makedirs(OBJ_DIR, exist_ok=True)
    todo = [s for s in srcs if force or _newer(_obj(s), [s] + hdrs)]

    def compile_one(src):
        cmd = [NVCC, *COMPILE, *(["-Xptxas", "-v"] if verbose else []), "-c", src, "-o", _obj(src) + ".tmp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode == 0:
            os.replace(_obj(src) + ".tmp", _obj(src))
        return src, r

    with ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as pool:
        results = list(pool.map(compile_one, todo))
    failed = False
    for src, r in results:
        if verbose or r.returncode:
            sys.stderr.write(r.stdout + r.stderr)
        failed = failed or r.returncode != 0
    if failed:
        raise subprocess.CalledProcessError(1, "nvcc", "compilation failed (see the messages above)")
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, *LINK, *[_obj(s) for s in srcs], "-o", tmp], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
