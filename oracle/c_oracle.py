"""ctypes wrapper of oracle/liboracle_c.so (the C/OpenMP restatement).
TEST INFRASTRUCTURE / CPU BASELINE ONLY (never imported by turbompc_b200)."""
import ctypes as C
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle_c.so")
_lib = None


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            subprocess.run(["make", "-C", HERE], check=True, capture_output=True)
        _lib = C.CDLL(LIB)
    return _lib


def max_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def admm_fixed(qp, rho, admm_iters, pcg_iters, sigma=1e-6, rho_f_factor=1000.0, alpha=1.6, threads=0, x0=None):
    """Fixed-count ADMM from the initial state of admm.py:1051-1088.  qp is an
    oracle.admm_ref.QP (float32 or float64).  pcg_iters < 0 solves each ADMM
    linear system exactly (block Cholesky, the direct backend's semantics).
    Returns dict of final state arrays."""
    lib = load()
    dt = qp.D.dtype
    suf = "f64" if dt == np.float64 else "f32"
    d = qp.dims
    B, T, N, n, nx, n0, m = (d[k] for k in ("B", "T", "N", "n", "nx", "n0", "m"))
    x = np.zeros((B, T, n), dtype=dt) if x0 is None else np.array(x0, dtype=dt)
    z = np.minimum(np.maximum(np.einsum("btkn,btn->btk", qp.G, x), qp.l), qp.u).astype(dt)
    st = dict(x=np.ascontiguousarray(x), y_g=np.zeros((B, T, m), dt), y_f0=np.zeros((B, n0), dt),
              y_fdyn=np.zeros((B, N, nx), dt), z_g=np.ascontiguousarray(z), rho=np.full(B, rho, dt))
    c = lambda a: np.ascontiguousarray(a, dtype=dt).ctypes.data_as(C.c_void_p)
    keep = [np.ascontiguousarray(getattr(qp, k), dtype=dt) for k in ("D", "E", "q", "A0", "Am", "Ap", "c0", "c",
                                                                      "G", "l", "u")]
    fn = getattr(lib, f"tmpc_oracle_admm_{suf}")
    fn.restype = C.c_int
    threads = threads or max_threads()
    bounds = np.linspace(0, B, min(threads, B) + 1).astype(int)

    def run(lo, hi):
        ptr = lambda a: C.c_void_p(a[lo:hi].ctypes.data)  # noqa: E731 (row slices of C-contiguous arrays)
        fn(C.c_int(hi - lo), C.c_int(T), C.c_int(n), C.c_int(nx), C.c_int(n0), C.c_int(m), *[ptr(a) for a in keep],
           *[ptr(st[k]) for k in ("x", "y_g", "y_f0", "y_fdyn", "z_g", "rho")], C.c_int(admm_iters),
           C.c_int(pcg_iters), C.c_double(sigma), C.c_double(rho_f_factor), C.c_double(alpha), C.c_int(1))

    with ThreadPoolExecutor(max_workers=len(bounds) - 1) as ex:
        list(ex.map(lambda i: run(bounds[i], bounds[i + 1]), range(len(bounds) - 1)))
    del c
    return st
