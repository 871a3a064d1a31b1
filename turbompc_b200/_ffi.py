"""ctypes binding of the C ABI in ``include/tmpc_b200.h``.

The shared library is built in-tree (``python -m turbompc_b200.build``) and
loaded from ``turbompc_b200/_lib/libtmpc_b200.so``.  There is no fallback: if
the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

c_int32_p = C.POINTER(C.c_int32)
c_uint32_p = C.POINTER(C.c_uint32)


class TmpcDims(C.Structure):
    _fields_ = [("Nb", C.c_int32), ("T", C.c_int32), ("n", C.c_int32), ("nx", C.c_int32),
                ("n0", C.c_int32), ("m", C.c_int32)]


class TmpcQP(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ("D", "E", "q", "A0", "A_minus", "A_plus", "c0", "c", "G", "l", "u")]


class TmpcAdmmState(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ("x", "y_g", "y_f0", "y_fdyn", "z_g", "xi_g", "rho_bar")]


class TmpcAdmmConfig(C.Structure):
    _fields_ = [("max_iter", C.c_int32), ("pcg_max_iter", C.c_int32), ("check_every", C.c_int32),
                ("adapt_rho_every", C.c_int32), ("eps_abs", C.c_double), ("eps_rel", C.c_double),
                ("sigma", C.c_double), ("rho_f_factor", C.c_double), ("alpha", C.c_double),
                ("pcg_eps", C.c_double), ("adaptive_rho_tolerance", C.c_double), ("rho_min", C.c_double),
                ("rho_max", C.c_double), ("use_slack", C.c_int32), ("linsys", C.c_int32)]


LINSYS_PCG = 0
LINSYS_DIRECT = 1
LINSYS_PCG_PACKED = 2
LAYOUT_REFERENCE = 0
LAYOUT_INTERLEAVED = 1
MODEL_QUADROTOR12 = 1
MODEL_CLOHESSY_WILTSHIRE = 2

# name -> (restype, argtypes)
_P = C.c_void_p
_SIGS = {
    "tmpc_version": (C.c_int32, []),
    "tmpc_error_string": (C.c_char_p, [C.c_int32]),
    "tmpc_set_transfer_poll_limit": (C.c_uint32, [C.c_uint32]),
    "tmpc_admm_iteration_timing": (C.c_int32, [C.c_int32]),
    "tmpc_admm_iteration_timing_read": (C.c_int32, [C.c_void_p, C.c_int32]),
    "tmpc_packed_operator_bytes": (C.c_size_t, [C.POINTER(TmpcDims), C.c_int32]),
    "tmpc_admm_workspace_bytes": (C.c_size_t, [C.POINTER(TmpcDims), C.c_int32, C.POINTER(TmpcAdmmConfig)]),
    "tmpc_admm_solve_fixed_scratch_f64": (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP),
                                                      C.POINTER(TmpcAdmmState), C.POINTER(TmpcAdmmState), C.c_void_p,
                                                      C.POINTER(TmpcAdmmConfig), C.c_void_p, C.c_void_p, C.c_void_p,
                                                      C.c_void_p]),
}
_SIGS["tmpc_riccati_factor_bytes"] = (C.c_size_t, [C.POINTER(TmpcDims), C.c_int32])
_SIGS["tmpc_interleaved_elems"] = (C.c_size_t, [C.c_int32, C.c_int64])
_SIGS["tmpc_riccati_il_elems_per_problem"] = (C.c_int64, [C.POINTER(TmpcDims)])
_SIGS["tmpc_stream_operator_bytes"] = (C.c_size_t, [C.POINTER(TmpcDims), C.c_int32])
_SIGS["tmpc_adjoint_kkt_workspace_bytes"] = (C.c_size_t, [C.POINTER(TmpcDims), C.c_int32])
for _s in ("f32", "f64"):
    _SIGS[f"tmpc_obstacle_rows_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.c_int32, C.c_int32, _P, _P, _P,
                                                     C.c_double, _P, _P, _P, _P])
    _SIGS[f"tmpc_ineq_rows_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P, _P, _P, _P])
    _SIGS[f"tmpc_mlp_cost_blocks_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.c_int32, _P, _P, _P, _P, _P,
                                                       C.c_double, _P, _P, _P])
    _SIGS[f"tmpc_interleave_{_s}"] = (C.c_int32, [C.c_int32, C.c_int64, _P, _P, _P])
    _SIGS[f"tmpc_deinterleave_{_s}"] = (C.c_int32, [C.c_int32, C.c_int64, _P, _P, _P])
    _SIGS[f"tmpc_schur_interleave_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P])
    _SIGS[f"tmpc_riccati_factor_il_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P])
    _SIGS[f"tmpc_riccati_solve_il_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P])
    _SIGS[f"tmpc_riccati_factor_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P])
    _SIGS[f"tmpc_linearize_dynamics_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.c_int32, C.c_int32, C.c_double, _P,
                                                          _P, _P, C.c_int32, _P, _P, _P])
    _SIGS[f"tmpc_schur_assemble_stream_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP), _P,
                                                             C.c_double, C.c_double, _P, _P, _P])
    _SIGS[f"tmpc_pcg_solve_stream_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P, _P, C.c_double,
                                                        C.c_int32, _P])
    _SIGS[f"tmpc_first_order_error_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP)] + [_P] * 6 +
                                                         [C.c_int32] + [_P] * 4 + [_P])
    _SIGS[f"tmpc_riccati_solve_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P])
    _SIGS[f"tmpc_adjoint_kkt_solve_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP), _P, _P, _P, _P,
                                                          C.c_size_t, _P])
    _SIGS[f"tmpc_schur_assemble_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP), _P, C.c_double,
                                                      C.c_double, _P, _P, _P, _P])
    _SIGS[f"tmpc_schur_assemble_packed_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP), _P,
                                                             C.c_double, C.c_double, _P, _P, _P])
    _SIGS[f"tmpc_pcg_solve_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P, _P, _P, C.c_double,
                                                 C.c_int32, _P])
    _SIGS[f"tmpc_pcg_solve_packed_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), _P, _P, _P, _P, _P, C.c_double,
                                                        C.c_int32, _P])
    _SIGS[f"tmpc_admm_solve_{_s}"] = (C.c_int32, [C.POINTER(TmpcDims), C.POINTER(TmpcQP),
                                                  C.POINTER(TmpcAdmmState), C.POINTER(TmpcAdmmState), _P,
                                                  C.POINTER(TmpcAdmmConfig), _P, _P, _P, _P, C.c_size_t, _P])

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    """The in-tree library, or the file named by TMPC_B200_LIB (a variant
    build, e.g. one compiled with phase timers)."""
    return os.environ.get("TMPC_B200_LIB") or _build.LIB


def load(build_if_missing: bool = True):
    """Load (building first if needed and allowed) the shared library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = lib_path()
        if not os.path.exists(path):
            if not build_if_missing:
                raise RuntimeError(f"turbompc_b200 CUDA library not built: {path} is missing "
                                   "(run `python -m turbompc_b200.build`)")
            _build.build()
        lib = C.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def exported_symbols():
    return sorted(_SIGS)


class TmpcError(RuntimeError):
    def __init__(self, fn: str, code: int):
        lib = load()
        msg = lib.tmpc_error_string(code).decode()
        super().__init__(f"{fn} failed with code {code}: {msg}")
        self.code = code


def check(fn: str, code: int) -> None:
    if code != 0:
        raise TmpcError(fn, code)
