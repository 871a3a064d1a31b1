"""Registration of the b200 XLA FFI handlers under the reference's target
names, for environments with jax / jaxlib (neither is installed where this
package is built and tested, so this module is untested here).

    from turbompc_b200 import jax_ffi
    jax_ffi.register()   # after `python -m turbompc_b200.build --ffi $(python -c
                         #   "import jax; print(jax.ffi.include_dir())")`

After ``register()``, the reference's adapter
(turbompc/solvers/admm/admm_ffi_backend.py:271-430, which calls
``jax.ffi.ffi_call("admm_fused_cuda" / "admm_fused_cuda_f64", ...)``) runs the
b200 fused ADMM kernel with its operands, attributes and results unchanged, and
the cuDSS adapter (admm/admm_cudss_ffi_backend.py, targets "admm_cudss_cuda" /
"admm_cudss_cuda_f64") runs the b200 direct (block-Cholesky) solve.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

TARGETS = {"admm_fused_cuda": "AdmmB200Cuda", "admm_fused_cuda_f64": "AdmmB200CudaF64",
           "admm_cudss_cuda": "AdmmB200DirectCuda", "admm_cudss_cuda_f64": "AdmmB200DirectCudaF64"}


def register(lib_path: str = _build.FFI_LIB) -> None:
    import jax  # noqa: F401  (jax is required here)

    if not os.path.exists(lib_path):
        raise RuntimeError(f"{lib_path} is missing: build it with python -m turbompc_b200.build --ffi <xla include>")
    C.CDLL(_build.LIB, mode=C.RTLD_GLOBAL)
    lib = C.CDLL(lib_path)
    for target, symbol in TARGETS.items():
        jax.ffi.register_ffi_target(target, jax.ffi.pycapsule(getattr(lib, symbol)), platform="CUDA")
