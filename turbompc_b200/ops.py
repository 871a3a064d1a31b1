"""Torch-facing wrappers of the CUDA C ABI (one call = one kernel launch on the
current CUDA stream).  All tensors must live on the same CUDA device, share
one dtype (float32 or float64) and be contiguous; wrappers raise otherwise.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import NamedTuple, Optional

import torch

from . import _ffi
from .qp_data import QPData


class ADMMState(NamedTuple):
    """turbompc/solvers/admm/admm.py:27-34, batched."""

    x_blocks: torch.Tensor  # (Nb, T, n)
    y_g: torch.Tensor  # (Nb, T, m)
    y_f_0: torch.Tensor  # (Nb, n0)
    y_f_dyn: torch.Tensor  # (Nb, N, nx)
    z_g: torch.Tensor  # (Nb, T, m)
    xi_g: torch.Tensor  # (Nb, T, m)
    rho_bar: torch.Tensor  # (Nb,)


@dataclass
class AdmmConfig:
    """ADMMConfig of turbompc/solvers/admm/csrc/admm_fused.cuh:6-22."""

    max_iter: int = 100
    pcg_max_iter: int = 10000
    check_every: int = 25
    adapt_rho_every: int = 25
    eps_abs: float = 1e-9
    eps_rel: float = 1e-9
    sigma: float = 1e-6
    rho_f_factor: float = 1000.0
    alpha: float = 1.6
    pcg_eps: float = 1e-20
    adaptive_rho_tolerance: float = 5.0
    rho_min: float = 1e-6
    rho_max: float = 1e6
    use_slack: bool = False
    linsys: int = _ffi.LINSYS_PCG

    def to_c(self) -> _ffi.TmpcAdmmConfig:
        return _ffi.TmpcAdmmConfig(int(self.max_iter), int(self.pcg_max_iter), int(self.check_every),
                                   int(self.adapt_rho_every), float(self.eps_abs), float(self.eps_rel),
                                   float(self.sigma), float(self.rho_f_factor), float(self.alpha),
                                   float(self.pcg_eps), float(self.adaptive_rho_tolerance), float(self.rho_min),
                                   float(self.rho_max), int(bool(self.use_slack)), int(self.linsys))


def _suffix(dtype: torch.dtype) -> str:
    if dtype == torch.float32:
        return "f32"
    if dtype == torch.float64:
        return "f64"
    raise TypeError(f"turbompc_b200 kernels support float32/float64, got {dtype}")


# Every tensor whose pointer goes to the library must stay referenced until the
# call has enqueued its kernel: a temporary such as ``x.contiguous()`` passed
# straight to _ptr is freed as soon as _ptr returns, and the caching allocator
# may hand its block to the next temporary, whose copy kernel (enqueued first)
# then overwrites the data the launch was meant to read.  Wrappers bind such
# temporaries to local names first.
def _ptr(t: Optional[torch.Tensor], dtype=None, device=None) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("turbompc_b200 kernels need CUDA tensors (no CPU fallback)")
    if device is not None and t.device != device:
        raise ValueError(f"tensor on {t.device}, expected {device}")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"tensor dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError("turbompc_b200 kernels need contiguous tensors")
    return t.data_ptr() if t.numel() > 0 else None


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dims_of(qp: QPData) -> _ffi.TmpcDims:
    return _ffi.TmpcDims(qp.Nb, qp.T, qp.n, qp.nx, qp.n0, qp.m)


def _qp_c(qp: QPData) -> _ffi.TmpcQP:
    dt, dev = qp.dtype, qp.device
    t = qp.tensors()
    B, T, n, nx, n0, m = qp.Nb, qp.T, qp.n, qp.nx, qp.n0, qp.m
    N = T - 1
    shapes = dict(D=(B, T, n, n), E=(B, N, n, n), q=(B, T, n), A0=(B, n0, n), A_minus=(B, N, nx, n),
                  A_plus=(B, N, nx, n), c0=(B, n0), c=(B, N, nx), G=(B, T, m, n), l=(B, T, m), u=(B, T, m))
    for k, s in shapes.items():
        if tuple(t[k].shape) != s:
            raise ValueError(f"QP field {k} has shape {tuple(t[k].shape)}, expected {s}")
    return _ffi.TmpcQP(*(_ptr(t[k], dt, dev) for k in ("D", "E", "q", "A0", "A_minus", "A_plus", "c0", "c", "G",
                                                       "l", "u")))


def _rho_vec(rho, qp: QPData) -> torch.Tensor:
    r = torch.as_tensor(rho, dtype=qp.dtype, device=qp.device)
    return r.expand(qp.Nb).contiguous() if r.dim() == 0 else r.contiguous()


def schur_assemble(qp: QPData, rho_bar, sigma: float, rho_f_factor: float):
    """compute_S_Phiinv (admm.py:71-154) for rho_f = rho_bar*rho_f_factor, rho_ineq = rho_bar.
    Returns (S, Phiinv, status), S/Phiinv (Nb, T, n, 3n) in the reference layout."""
    lib = _ffi.load()
    B, T, n = qp.Nb, qp.T, qp.n
    S = torch.empty(B, T, n, 3 * n, dtype=qp.dtype, device=qp.device)
    P = torch.empty_like(S)
    st = torch.zeros(B, dtype=torch.int32, device=qp.device)
    rho = _rho_vec(rho_bar, qp)
    name = f"tmpc_schur_assemble_{_suffix(qp.dtype)}"
    d, q = dims_of(qp), _qp_c(qp)
    _ffi.check(name, getattr(lib, name)(C.byref(d), C.byref(q), _ptr(rho), float(sigma), float(rho_f_factor),
                                        _ptr(S), _ptr(P), _ptr(st), _stream(qp.device)))
    return S, P, st


def schur_assemble_packed(qp: QPData, rho_bar, sigma: float, rho_f_factor: float):
    """Same operators in the packed format; returns (ops uint8 tensor, status)."""
    lib = _ffi.load()
    d, q = dims_of(qp), _qp_c(qp)
    nbytes = lib.tmpc_packed_operator_bytes(C.byref(d), qp.dtype.itemsize)
    if nbytes == 0 and qp.Nb > 0:
        raise ValueError(f"unsupported dimensions for the packed format (n={qp.n})")
    ops = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=qp.device)
    st = torch.zeros(qp.Nb, dtype=torch.int32, device=qp.device)
    rho = _rho_vec(rho_bar, qp)
    name = f"tmpc_schur_assemble_packed_{_suffix(qp.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), C.byref(q), _ptr(rho), float(sigma), float(rho_f_factor),
                                        ops.data_ptr(), _ptr(st), _stream(qp.device)))
    return ops, st


def pcg_solve(S: torch.Tensor, Phiinv: torch.Tensor, rhs: torch.Tensor, x0: torch.Tensor, eps: float,
              max_iters: int):
    """pcg_blktridi_cuda (pcg_ffi.cc:115-147) on reference-layout operators.
    S, Phiinv (Nb, T, n, 3n); rhs, x0 (Nb, T, n).  Returns (x, iters uint32->int64)."""
    lib = _ffi.load()
    if S.dim() != 4 or S.shape[-1] != 3 * S.shape[-2]:
        raise ValueError("S must be (Nb, T, n, 3n)")
    B, T, n = S.shape[:3]
    for name_, t in (("Phiinv", Phiinv), ("rhs", rhs), ("x0", x0)):
        want = S.shape if name_ == "Phiinv" else (B, T, n)
        if tuple(t.shape) != tuple(want):
            raise ValueError(f"{name_} has shape {tuple(t.shape)}, expected {tuple(want)}")
    x = torch.empty_like(rhs)
    it = torch.empty(B, dtype=torch.int32, device=S.device)
    d = _ffi.TmpcDims(B, T, n, n, 0, 0)
    name = f"tmpc_pcg_solve_{_suffix(S.dtype)}"
    dt = S.dtype
    _ffi.check(name, getattr(lib, name)(C.byref(d), _ptr(S, dt), _ptr(Phiinv, dt), _ptr(rhs, dt), _ptr(x0, dt),
                                        _ptr(x), _ptr(it), float(eps), int(max_iters), _stream(S.device)))
    return x, it.to(torch.int64) & 0xFFFFFFFF


def pcg_solve_packed(ops: torch.Tensor, dims: _ffi.TmpcDims, rhs: torch.Tensor, x0: torch.Tensor, eps: float,
                     max_iters: int):
    """PCG on packed operators (from schur_assemble_packed)."""
    lib = _ffi.load()
    x = torch.empty_like(rhs)
    it = torch.empty(rhs.shape[0], dtype=torch.int32, device=rhs.device)
    name = f"tmpc_pcg_solve_packed_{_suffix(rhs.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(dims), ops.data_ptr(), _ptr(rhs), _ptr(x0, rhs.dtype), _ptr(x),
                                        _ptr(it), float(eps), int(max_iters), _stream(rhs.device)))
    return x, it.to(torch.int64) & 0xFFFFFFFF


def schur_assemble_stream(qp: QPData, rho_bar, sigma: float, rho_f_factor: float):
    """S and Phiinv in the stream layout (full blocks, for the HBM-streaming
    PCG); returns (ops tensor of the QP's dtype, flat, status)."""
    lib = _ffi.load()
    d, q = dims_of(qp), _qp_c(qp)
    nbytes = lib.tmpc_stream_operator_bytes(C.byref(d), qp.dtype.itemsize)
    if nbytes == 0 and qp.Nb > 0:
        raise ValueError(f"unsupported dimensions for the stream layout (n={qp.n})")
    ops = torch.empty(max(nbytes // qp.dtype.itemsize, 4), dtype=qp.dtype, device=qp.device)
    st = torch.zeros(qp.Nb, dtype=torch.int32, device=qp.device)
    rho = _rho_vec(rho_bar, qp)
    name = f"tmpc_schur_assemble_stream_{_suffix(qp.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), C.byref(q), _ptr(rho), float(sigma), float(rho_f_factor),
                                        ops.data_ptr(), _ptr(st), _stream(qp.device)))
    return ops, st


def pcg_solve_stream(ops: torch.Tensor, dims: _ffi.TmpcDims, rhs: torch.Tensor, x0: torch.Tensor, eps: float,
                     max_iters: int, x_out: Optional[torch.Tensor] = None):
    """HBM-streaming PCG on stream-layout operators (schur_assemble_stream)."""
    lib = _ffi.load()
    x = torch.empty_like(rhs) if x_out is None else x_out
    it = torch.empty(rhs.shape[0], dtype=torch.int32, device=rhs.device)
    name = f"tmpc_pcg_solve_stream_{_suffix(rhs.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(dims), _ptr(ops, rhs.dtype), _ptr(rhs), _ptr(x0, rhs.dtype),
                                        _ptr(x), _ptr(it), float(eps), int(max_iters), _stream(rhs.device)))
    return x, it.to(torch.int64) & 0xFFFFFFFF


def admm_workspace_bytes(qp: QPData, cfg: AdmmConfig) -> int:
    lib = _ffi.load()
    d = dims_of(qp)
    c = cfg.to_c()
    return int(lib.tmpc_admm_workspace_bytes(C.byref(d), qp.dtype.itemsize, C.byref(c)))


def _state_c(s: ADMMState, dt, dev) -> _ffi.TmpcAdmmState:
    return _ffi.TmpcAdmmState(_ptr(s.x_blocks, dt, dev), _ptr(s.y_g, dt, dev), _ptr(s.y_f_0, dt, dev),
                              _ptr(s.y_f_dyn, dt, dev), _ptr(s.z_g, dt, dev), _ptr(s.xi_g, dt, dev),
                              _ptr(s.rho_bar, dt, dev))


def empty_state_like(s: ADMMState) -> ADMMState:
    return ADMMState(*(torch.empty_like(t) for t in s))


def admm_solve(qp: QPData, state0: ADMMState, cfg: AdmmConfig, slack_weight=None, out: Optional[ADMMState] = None,
               workspace: Optional[torch.Tensor] = None):
    """Fused ADMM solve (admm_fused_cuda).  Returns (state, iters, status)."""
    lib = _ffi.load()
    dt, dev = qp.dtype, qp.device
    if out is None:
        out = empty_state_like(state0)
    it = torch.empty(qp.Nb, dtype=torch.int32, device=dev)
    st = torch.empty(qp.Nb, dtype=torch.int32, device=dev)
    sw = None if slack_weight is None else _rho_vec(slack_weight, qp)
    ws_need = admm_workspace_bytes(qp, cfg)
    if ws_need > 0 and (workspace is None or workspace.numel() < ws_need):
        workspace = torch.empty(ws_need, dtype=torch.uint8, device=dev)
    ws_ptr = workspace.data_ptr() if (workspace is not None and ws_need > 0) else None
    d, q, c = dims_of(qp), _qp_c(qp), cfg.to_c()
    si, so = _state_c(state0, dt, dev), _state_c(out, dt, dev)
    name = f"tmpc_admm_solve_{_suffix(dt)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), C.byref(q), C.byref(si), C.byref(so), _ptr(sw), C.byref(c),
                                        None, _ptr(it), _ptr(st), ws_ptr, ws_need, _stream(dev)))
    return out, it.to(torch.int64) & 0xFFFFFFFF, st


def admm_initial_state(qp: QPData, rho_bar, x0: Optional[torch.Tensor] = None) -> ADMMState:
    """admm.py:1051-1088: x = 0 (or x0), z_g = clamp(G x, l, u), duals zero."""
    B, T, n, m = qp.Nb, qp.T, qp.n, qp.m
    x = torch.zeros(B, T, n, dtype=qp.dtype, device=qp.device) if x0 is None else x0.clone().contiguous()
    if x0 is None:  # G 0 = 0
        z = torch.minimum(torch.maximum(torch.zeros_like(qp.ineq.l), qp.ineq.l), qp.ineq.u)
    elif x.is_cuda:
        z = ineq_rows(qp.ineq.G, x, lo=qp.ineq.l, hi=qp.ineq.u)
    else:
        z = torch.minimum(torch.maximum(torch.einsum("btmn,btn->btm", qp.ineq.G, x), qp.ineq.l), qp.ineq.u)
    return ADMMState(x, torch.zeros_like(z), torch.zeros_like(qp.eq.c0), torch.zeros_like(qp.eq.c),
                     z.contiguous(), torch.zeros_like(z), _rho_vec(rho_bar, qp).clone())


def riccati_factor(S: torch.Tensor, factor: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None):
    """Block Cholesky of reference-layout S (Nb, T, n, 3n).  Returns
    (factor uint8 tensor, status int32 (Nb,)); ``factor`` / ``status`` reuse
    caller buffers (uint8 of at least the factor size, int32 (Nb,))."""
    lib = _ffi.load()
    B, T, n = S.shape[:3]
    d = _ffi.TmpcDims(B, T, n, n, 0, 0)
    nbytes = lib.tmpc_riccati_factor_bytes(C.byref(d), S.dtype.itemsize)
    if nbytes == 0 and B > 0:
        raise ValueError(f"unsupported dimensions for the block Cholesky (n={n})")
    if factor is not None:
        if factor.dtype != torch.uint8 or factor.numel() < nbytes or not factor.is_contiguous():
            raise ValueError(f"factor buffer must be contiguous uint8 with at least {nbytes} bytes")
        fac = factor
    else:
        fac = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=S.device)
    if status is not None:
        if status.dtype != torch.int32 or status.numel() != B:
            raise ValueError("status buffer must be int32 with one entry per problem")
        st = status
    else:
        st = torch.zeros(B, dtype=torch.int32, device=S.device)
    name = f"tmpc_riccati_factor_{_suffix(S.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), _ptr(S), fac.data_ptr(), _ptr(st), _stream(S.device)))
    return fac, st


def riccati_solve(factor: torch.Tensor, rhs: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Solve S x = rhs (rhs (Nb, T, n)) with a factor from riccati_factor
    (into ``out`` when given: same shape / dtype as rhs, contiguous)."""
    lib = _ffi.load()
    B, T, n = rhs.shape
    d = _ffi.TmpcDims(B, T, n, n, 0, 0)
    if out is not None and (out.shape != rhs.shape or out.dtype != rhs.dtype or not out.is_contiguous()):
        raise ValueError("out must be a contiguous tensor shaped like rhs")
    x = torch.empty_like(rhs) if out is None else out
    name = f"tmpc_riccati_solve_{_suffix(rhs.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), factor.data_ptr(), _ptr(rhs), _ptr(x), _stream(rhs.device)))
    return x


def adjoint_kkt_solve(qp: QPData, workspace: Optional[torch.Tensor] = None):
    """Adjoint KKT solve (backward_kkt_jax.py:177-211) on the GPU.  qp.ineq.G
    holds the active rows (sign * G, zero rows inactive).  Returns
    (dz (Nb, T, n), multipliers (Nb, n0 + N*nx + T*m), status)."""
    lib = _ffi.load()
    d, q = dims_of(qp), _qp_c(qp)
    B, T, n, nx, n0, m = qp.Nb, qp.T, qp.n, qp.nx, qp.n0, qp.m
    dz = torch.empty(B, T, n, dtype=qp.dtype, device=qp.device)
    mult = torch.empty(B, n0 + (T - 1) * nx + T * m, dtype=qp.dtype, device=qp.device)
    st = torch.zeros(B, dtype=torch.int32, device=qp.device)
    need = int(lib.tmpc_adjoint_kkt_workspace_bytes(C.byref(d), qp.dtype.itemsize))
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=qp.device)
    name = f"tmpc_adjoint_kkt_solve_{_suffix(qp.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), C.byref(q), _ptr(dz), _ptr(mult), _ptr(st), workspace.data_ptr(),
                                        need, _stream(qp.device)))
    return dz, mult, st


def linearize_dynamics(model: int, params, scheme: int, dt: float, states: torch.Tensor, controls: torch.Tensor):
    """Dynamics rows of the QP for a built-in model (tmpc_linearize_dynamics_*):
    returns (A_minus (Nb, N, nx, n), c (Nb, N, nx)) at the stages t < N."""
    lib = _ffi.load()
    states, controls = states.contiguous(), controls.contiguous()
    Nb, T, nx = states.shape
    nu = controls.shape[-1]
    N = T - 1
    Am = torch.empty(Nb, N, nx, nx + nu, dtype=states.dtype, device=states.device)
    c = torch.empty(Nb, N, nx, dtype=states.dtype, device=states.device)
    d = _ffi.TmpcDims(Nb, T, nx + nu, nx, 0, 0)
    pa = (C.c_double * max(1, len(params)))(*[float(v) for v in params])
    name = f"tmpc_linearize_dynamics_{_suffix(states.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), int(model), int(scheme), float(dt), _ptr(states),
                                        _ptr(controls, states.dtype, states.device), pa, len(params), _ptr(Am),
                                        _ptr(c), _stream(states.device)))
    return Am, c


def first_order_error(qp: QPData, z: torch.Tensor, state: ADMMState, slacks: Optional[torch.Tensor] = None):
    """First-order (KKT) error of SQP iterates (tmpc_first_order_error_*):
    returns (conv, eq, ineq, g) with g = G z (+ slacks), shapes (Nb,), (Nb,),
    (Nb,), (Nb, T, m)."""
    lib = _ffi.load()
    dt, dev = qp.dtype, qp.device
    z = z.contiguous()
    conv = torch.empty(qp.Nb, dtype=dt, device=dev)
    eq = torch.empty_like(conv)
    ineq = torch.empty_like(conv)
    g = torch.empty(qp.Nb, qp.T, qp.m, dtype=dt, device=dev)
    use_slack = bool(qp.ineq.use_slack_variables) and qp.m > 0
    sw = qp.ineq.slack_penalization_weight if use_slack else None
    yf0, yfd, yg = state.y_f_0.contiguous(), state.y_f_dyn.contiguous(), state.y_g.contiguous()
    sl = slacks.contiguous() if use_slack else None
    swv = _rho_vec(sw, qp) if sw is not None else None
    name = f"tmpc_first_order_error_{_suffix(dt)}"
    _ffi.check(name, getattr(lib, name)(C.byref(dims_of(qp)), C.byref(_qp_c(qp)), _ptr(z, dt, dev),
                                        _ptr(yf0, dt, dev), _ptr(yfd, dt, dev), _ptr(yg, dt, dev), _ptr(sl, dt, dev),
                                        _ptr(swv, dt, dev), int(use_slack), _ptr(conv), _ptr(eq), _ptr(ineq),
                                        _ptr(g), _stream(dev)))
    return conv, eq, ineq, g


# ---------------------------------------------------------------------------
# Batch-interleaved layout (TMPC_LAYOUT_INTERLEAVED): groups of 32 problems,
# element-major and problem-minor inside a group.
# ---------------------------------------------------------------------------
def interleaved_numel(nb: int, elems_per_problem: int) -> int:
    return int(_ffi.load().tmpc_interleaved_elems(int(nb), int(elems_per_problem)))


def interleave(x: torch.Tensor) -> torch.Tensor:
    """Problem-major (Nb, ...) -> flat interleaved tensor."""
    lib = _ffi.load()
    nb = x.shape[0]
    e = x[0].numel() if nb > 0 else 0
    out = torch.empty(max(interleaved_numel(nb, e), 1), dtype=x.dtype, device=x.device)
    xc = x.contiguous()
    name = f"tmpc_interleave_{_suffix(x.dtype)}"
    _ffi.check(name, getattr(lib, name)(nb, e, _ptr(xc), out.data_ptr(), _stream(x.device)))
    return out


def deinterleave(flat: torch.Tensor, shape) -> torch.Tensor:
    """Flat interleaved tensor -> problem-major tensor of ``shape`` (Nb, ...)."""
    lib = _ffi.load()
    out = torch.empty(shape, dtype=flat.dtype, device=flat.device)
    nb = shape[0]
    e = out[0].numel() if nb > 0 else 0
    name = f"tmpc_deinterleave_{_suffix(flat.dtype)}"
    _ffi.check(name, getattr(lib, name)(nb, e, flat.data_ptr(), _ptr(out), _stream(flat.device)))
    return out


def schur_interleave(S: torch.Tensor) -> torch.Tensor:
    """Reference-layout S (Nb, T, n, 3n) -> the interleaved operator (Theta
    lower-packed and Phi blocks) that riccati_factor_il takes."""
    lib = _ffi.load()
    B, T, n = S.shape[:3]
    d = _ffi.TmpcDims(B, T, n, n, 0, 0)
    e = int(lib.tmpc_riccati_il_elems_per_problem(C.byref(d)))
    ops_il = torch.empty(max(interleaved_numel(B, e), 1), dtype=S.dtype, device=S.device)
    name = f"tmpc_schur_interleave_{_suffix(S.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), _ptr(S), ops_il.data_ptr(), _stream(S.device)))
    return ops_il


def riccati_factor_il(ops_il: torch.Tensor, dims: _ffi.TmpcDims, factor: Optional[torch.Tensor] = None,
                      status: Optional[torch.Tensor] = None):
    """Block Cholesky on the interleaved operator; returns (factor, status)."""
    lib = _ffi.load()
    fac = torch.empty_like(ops_il) if factor is None else factor
    st = torch.zeros(dims.Nb, dtype=torch.int32, device=ops_il.device) if status is None else status
    name = f"tmpc_riccati_factor_il_{_suffix(ops_il.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(dims), ops_il.data_ptr(), fac.data_ptr(), _ptr(st),
                                        _stream(ops_il.device)))
    return fac, st


def riccati_solve_il(factor: torch.Tensor, dims: _ffi.TmpcDims, rhs_il: torch.Tensor,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Solve S x = rhs on interleaved vectors (flat, from interleave)."""
    lib = _ffi.load()
    x = torch.empty_like(rhs_il) if out is None else out
    name = f"tmpc_riccati_solve_il_{_suffix(factor.dtype)}"
    _ffi.check(name, getattr(lib, name)(C.byref(dims), factor.data_ptr(), rhs_il.data_ptr(), x.data_ptr(),
                                        _stream(factor.device)))
    return x


# ---------------------------------------------------------------------------
# QP producers beyond the dynamics rows
# ---------------------------------------------------------------------------
def obstacle_rows(states: torch.Tensor, centers: torch.Tensor, radii: torch.Tensor, dim: int, n: int,
                  row_scale: float = 1.0):
    """Linearised spherical obstacle rows (tmpc_obstacle_rows_*): returns
    (G (Nb, T, K, n), l, u (Nb, T, K))."""
    lib = _ffi.load()
    states = states.contiguous()
    Nb, T, nx = states.shape
    K = centers.shape[1]
    dt, dev = states.dtype, states.device
    G = torch.empty(Nb, T, K, n, dtype=dt, device=dev)
    lo = torch.empty(Nb, T, K, dtype=dt, device=dev)
    hi = torch.empty_like(lo)
    d = _ffi.TmpcDims(Nb, T, n, nx, 0, 0)
    cc, rr = centers.contiguous(), radii.contiguous()
    name = f"tmpc_obstacle_rows_{_suffix(dt)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), int(dim), int(K), _ptr(states), _ptr(cc, dt, dev),
                                        _ptr(rr, dt, dev), float(row_scale), _ptr(G), _ptr(lo), _ptr(hi),
                                        _stream(dev)))
    return G, lo, hi


def ineq_rows(G: torch.Tensor, z: torch.Tensor, slack: Optional[torch.Tensor] = None,
              lo: Optional[torch.Tensor] = None, hi: Optional[torch.Tensor] = None) -> torch.Tensor:
    """g = G_t z_t (+ slack), clamped to [lo, hi] when given
    (tmpc_ineq_rows_*); G (Nb, T, m, n), z (Nb, T, n) -> (Nb, T, m)."""
    lib = _ffi.load()
    Nb, T, m, n = G.shape
    dt, dev = G.dtype, G.device
    out = torch.empty(Nb, T, m, dtype=dt, device=dev)
    d = _ffi.TmpcDims(Nb, T, n, 0, 0, m)
    Gc, zc = G.contiguous(), z.contiguous()
    sl = slack.contiguous() if slack is not None else None
    lc = lo.contiguous() if lo is not None else None
    hc = hi.contiguous() if hi is not None else None
    name = f"tmpc_ineq_rows_{_suffix(dt)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), _ptr(Gc, dt, dev), _ptr(zc, dt, dev), _ptr(sl, dt, dev),
                                        _ptr(lc, dt, dev), _ptr(hc, dt, dev), _ptr(out), _stream(dev)))
    return out


def mlp_cost_blocks_(D: torch.Tensor, q: torch.Tensor, states: torch.Tensor, controls: torch.Tensor,
                     W1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor, scale: float):
    """Adds the exact quadratisation of s * w2 . tanh(W1 z + b1) to D and q in
    place (tmpc_mlp_cost_blocks_*); D (Nb, T, n, n), q (Nb, T, n) contiguous."""
    lib = _ffi.load()
    Nb, T, nx = states.shape
    nu = controls.shape[-1]
    dt, dev = D.dtype, D.device
    d = _ffi.TmpcDims(Nb, T, nx + nu, nx, 0, 0)
    xs, us = states.contiguous(), controls.contiguous()
    w1c, b1c, w2c = W1.contiguous(), b1.contiguous(), w2.contiguous()
    name = f"tmpc_mlp_cost_blocks_{_suffix(dt)}"
    _ffi.check(name, getattr(lib, name)(C.byref(d), int(W1.shape[0]), _ptr(xs, dt, dev), _ptr(us, dt, dev),
                                        _ptr(w1c, dt, dev), _ptr(b1c, dt, dev), _ptr(w2c, dt, dev), float(scale),
                                        _ptr(D, dt, dev), _ptr(q, dt, dev), _stream(dev)))
    return D, q
