"""Build the sm_100a shared library ``turbompc_b200/_lib/libtmpc_b200.so``.

Plain ``nvcc`` (no torch JIT cache): every ``csrc/*.cu`` file is compiled to an
object in ``turbompc_b200/_build/`` (in parallel) and linked into one shared
library exporting the C ABI declared in ``include/tmpc_b200.h``.  The library
is rebuilt when a source or header is newer than it.

    python -m turbompc_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libtmpc_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I" + INCLUDE, "-I" + CSRC]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build turbompc_b200")
    return path


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps_mtime() -> float:
    files = glob.glob(os.path.join(CSRC, "*")) + glob.glob(os.path.join(INCLUDE, "*.h")) + [__file__]
    return max(os.path.getmtime(f) for f in files)


def _obj_deps_mtime(src: str) -> float:
    """An object depends on its own source, every header and this script."""
    files = ([src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
             + [__file__])
    return max(os.path.getmtime(f) for f in files)


def needs_build() -> bool:
    return not os.path.exists(LIB) or os.path.getmtime(LIB) < _deps_mtime()


def _compile(src: str, verbose: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= _obj_deps_mtime(src):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    """Compile and link the library; returns its path."""
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    if force:
        for o in glob.glob(os.path.join(BUILD, "*.o")):
            os.remove(o)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, list(extra)), srcs))
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


FFI_SRC = os.path.join(CSRC, "ffi", "admm_b200_ffi.cc")
FFI_LIB = os.path.join(LIBDIR, "libtmpc_b200_ffi.so")


def build_ffi(xla_include: str) -> str:
    """Compile the XLA FFI handlers (csrc/ffi/admm_b200_ffi.cc) against the
    jaxlib FFI headers in ``xla_include`` (``jax.ffi.include_dir()``) into
    _lib/libtmpc_b200_ffi.so, linked to the main library.  Only where jaxlib
    is installed; the handlers compile to nothing without its headers."""
    if not os.path.exists(os.path.join(xla_include, "xla", "ffi", "api", "ffi.h")):
        raise RuntimeError(f"no XLA FFI headers under {xla_include}")
    build()
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "include")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-I" + xla_include, "-I" + INCLUDE, "-I" + cuda_inc,
           FFI_SRC, "-o", FFI_LIB, "-L" + LIBDIR, "-ltmpc_b200", "-Wl,-rpath,$ORIGIN",
           "-L" + os.path.join(os.path.dirname(cuda_inc), "lib64"), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"FFI build failed:\n{res.stdout}\n{res.stderr}")
    return FFI_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ffi", metavar="XLA_INCLUDE", default="",
                    help="also build the XLA FFI handlers against these jaxlib headers")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    if a.ffi:
        print(build_ffi(a.ffi))
