"""Build libtabbysample.so in-tree with nvcc for sm_100a.

    python -m tabby_b200.build        # -> tabby_b200/lib/libtabbysample.so

The library is a plain C-ABI shared object (include/tabby_sample.h); it does not link
against torch. CUDA's runtime is linked statically so the .so only needs the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libtabbysample.so")
SOURCES = ["sampler_kernels.cu", "capi.cu", "noalloc.cu", "softmax_rows.cu", "lmhead.cu",
           "exchange.cu"]
HEADERS = ["finalize.cuh", "js_math.cuh", "sampler_internal.h", "warp_sort.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-ffp-contract=off,-fvisibility=hidden",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "tabby_sample.h"))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, out: str | None = None,
          defines: tuple = ()) -> str:
    """Compile SOURCES into `out` (default: the in-tree library). `defines` adds -D flags
    (e.g. TABBY_CHECKS=1 for the self-checking debug build)."""
    lib_path = out or LIB
    if out is None and not force and not _stale():
        return LIB
    libdir = os.path.dirname(lib_path)
    os.makedirs(libdir, exist_ok=True)
    objs = []
    for src in SOURCES:
        obj = os.path.join(libdir, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *[f"-D{d}" for d in defines],
               "-I", os.path.join(ROOT, "include"), "-I", CSRC,
               "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose:
            sys.stderr.write(r.stderr)
        objs.append(obj)
    tmp = lib_path + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs,
           "-Xlinker", "--exclude-libs,ALL"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib_path)
    for o in objs:
        os.remove(o)
    return lib_path


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
