"""CPU restatement (NumPy) of TurboMPC's batched ADMM / Schur / PCG inner solve.

TEST INFRASTRUCTURE ONLY.  Nothing in ``turbompc_b200`` imports this module;
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use it, and only as the checker.

Every function restates one reference function (paths are relative to the
reference project root) and works on a leading batch axis ``B``:

    x       (B, T, n)      z_g / y_g / xi_g (B, T, m)
    y_f0    (B, n0)        y_fdyn           (B, N, nx)
    rho     (B,)           S / Phiinv       (B, T, n, 3n)

Parity pins: the algebra is pinned by the known-answer checks restated in
``tests/test_oracle.py`` (reference tests
``tests/cuda/backends/test_admm_math_cuda_vs_python.py:135-158`` and
``tests/python/solvers/test_solver_pcg.py:92-110``, dense-solve agreement as in
``tests/cuda/backends/test_pcg_ffi_backend.py:29-51``) and by the golden
vectors in ``tests/golden/`` produced by the reference's own CUDA kernels
(``admmFusedKernel`` / ``pcgBlkTridiSingleBlock``) compiled from source by
``oracle/build_ref.sh`` and run on a B200.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import numpy as np

PCG_ABS_TOL = 1e-12  # turbompc/solvers/linear_systems_solvers/pcg_primal.py:113


@dataclass
class QP:
    """Batched stage-blocked QP (turbompc/solvers/qp_data.py:13-97)."""

    D: np.ndarray  # (B, T, n, n)
    E: np.ndarray  # (B, N, n, n)   P[t+1, t] = E[t]
    q: np.ndarray  # (B, T, n)
    A0: np.ndarray  # (B, n0, n)
    Am: np.ndarray  # (B, N, nx, n)
    Ap: np.ndarray  # (B, N, nx, n)
    c0: np.ndarray  # (B, n0)
    c: np.ndarray  # (B, N, nx)
    G: np.ndarray  # (B, T, m, n)
    l: np.ndarray  # (B, T, m)
    u: np.ndarray  # (B, T, m)
    slack_weight: Optional[np.ndarray] = None  # (B,)
    use_slack: bool = False

    @property
    def dims(self):
        B, T, n, _ = self.D.shape
        return dict(B=B, T=T, N=T - 1, n=n, nx=self.Am.shape[2], n0=self.A0.shape[1], m=self.G.shape[2])

    def astype(self, dtype) -> "QP":
        kw = {k: (getattr(self, k).astype(dtype) if isinstance(getattr(self, k), np.ndarray) else getattr(self, k))
              for k in ("D", "E", "q", "A0", "Am", "Ap", "c0", "c", "G", "l", "u", "slack_weight")}
        return QP(**kw, use_slack=self.use_slack)


@dataclass
class ADMMState:
    """turbompc/solvers/admm/admm.py:27-34 (batched)."""

    x: np.ndarray
    y_g: np.ndarray
    y_f0: np.ndarray
    y_fdyn: np.ndarray
    z_g: np.ndarray
    xi_g: np.ndarray
    rho: np.ndarray

    def copy(self) -> "ADMMState":
        return ADMMState(*(np.array(a, copy=True) for a in
                           (self.x, self.y_g, self.y_f0, self.y_fdyn, self.z_g, self.xi_g, self.rho)))


@dataclass
class ADMMConfig:
    """Fields of ADMMConfig (turbompc/solvers/admm/csrc/admm_fused.cuh:6-22)."""

    max_iter: int = 100
    pcg_max_iter: int = 200
    check_every: int = 25
    eps_abs: float = 1e-9
    eps_rel: float = 1e-9
    sigma: float = 1e-6
    rho_f_factor: float = 1000.0
    alpha: float = 1.6
    pcg_eps: float = 1e-20
    use_slack: bool = False
    adapt_rho_every: int = 25
    adaptive_rho_tolerance: float = 5.0
    rho_min: float = 1e-6
    rho_max: float = 1e6


def _bmv(M, v):
    return np.einsum("...ij,...j->...i", M, v)


def _bmtv(M, v):
    return np.einsum("...ji,...j->...i", M, v)


# ---------------------------------------------------------------------------
# Schur complement and preconditioner: turbompc/solvers/admm/admm.py:71-154
# ---------------------------------------------------------------------------
def theta_phi(qp: QP, rho_f, sigma, rho_ineq):
    """Θ_t and Φ_t (admm.py:86-101).  rho_f / rho_ineq are (B,) or scalars."""
    d = qp.dims
    B, N, n = d["B"], d["N"], d["n"]
    rho_f = np.broadcast_to(np.asarray(rho_f, dtype=qp.D.dtype), (B,))[:, None, None]
    rho_i = np.broadcast_to(np.asarray(rho_ineq, dtype=qp.D.dtype), (B,))[:, None, None]
    GtG = np.einsum("btki,btkj->btij", qp.G, qp.G)
    theta = qp.D + sigma * np.eye(n, dtype=qp.D.dtype) + rho_i[:, None] * GtG
    AmtAm = np.einsum("btki,btkj->btij", qp.Am, qp.Am)
    AptAp = np.einsum("btki,btkj->btij", qp.Ap, qp.Ap)
    A0tA0 = np.einsum("bki,bkj->bij", qp.A0, qp.A0)
    theta = theta.copy()
    theta[:, 0] += rho_f * (A0tA0 + AmtAm[:, 0])
    if N > 1:
        theta[:, 1:N] += rho_f[:, None] * (AptAp[:, :-1] + AmtAm[:, 1:])
    theta[:, N] += rho_f * AptAp[:, -1]
    phi = qp.E + rho_f[:, None] * np.einsum("btki,btkj->btij", qp.Ap, qp.Am)
    return theta, phi


def compute_S_Phiinv(qp: QP, rho_f, sigma, rho_ineq):
    """Reference-layout S and Φ⁻¹, each (B, T, n, 3n) (admm.py:103-153)."""
    theta, phi = theta_phi(qp, rho_f, sigma, rho_ineq)
    B, T, n, _ = theta.shape
    dt = theta.dtype
    tinv = np.linalg.inv(theta)
    z = np.zeros((B, 1, n, n), dtype=dt)
    phis = np.concatenate([z, phi, z], axis=1)  # phis[t+1] = Φ_t
    S = np.concatenate([phis[:, :-1], theta, np.swapaxes(phis[:, 1:], -1, -2)], axis=-1)
    tinv_p = np.concatenate([z, tinv, z], axis=1)
    prev = tinv_p[:, 1:-1] @ phis[:, :-1] @ tinv_p[:, :-2]
    nxt = tinv_p[:, 1:-1] @ np.swapaxes(phis[:, 1:], -1, -2) @ tinv_p[:, 2:]
    Phiinv = np.concatenate([prev, -tinv, nxt], axis=-1)
    return S, Phiinv


def block_tridi_apply(M, v):
    """y_t = M[t,:, :n] v_{t-1} + M[t,:,n:2n] v_t + M[t,:,2n:] v_{t+1}
    (turbompc/solvers/linear_systems_solvers/linear_solve.py:18-47)."""
    n = v.shape[-1]
    z = np.zeros_like(v[:, :1])
    vp = np.concatenate([z, v[:, :-1]], axis=1)
    vn = np.concatenate([v[:, 1:], z], axis=1)
    return _bmv(M[..., :n], vp) + _bmv(M[..., n:2 * n], v) + _bmv(M[..., 2 * n:], vn)


def block_tridi_to_dense(M):
    """linear_solve.py:50-82, batched."""
    B, T, n, _ = M.shape
    A = np.zeros((B, T * n, T * n), dtype=M.dtype)
    for t in range(T):
        r = slice(t * n, (t + 1) * n)
        A[:, r, r] = M[:, t, :, n:2 * n]
        if t > 0:
            A[:, r, (t - 1) * n:t * n] = M[:, t, :, :n]
        if t < T - 1:
            A[:, r, (t + 1) * n:(t + 2) * n] = M[:, t, :, 2 * n:]
    return A


def solve_block_tridi_dense(M, rhs):
    """linear_solve.py:85-112 (dense LU solve), batched."""
    B, T, n, _ = M.shape
    A = block_tridi_to_dense(M)
    return np.linalg.solve(A, rhs.reshape(B, T * n, 1))[..., 0].reshape(B, T, n)


# ---------------------------------------------------------------------------
# Operators: admm.py:177-256
# ---------------------------------------------------------------------------
def apply_C_parts(qp: QP, x):
    Cx0 = _bmv(qp.A0, x[:, 0])
    Cx = _bmv(qp.Am, x[:, :-1]) + _bmv(qp.Ap, x[:, 1:])
    return Cx0, Cx


def apply_Ct(qp: QP, y0, ydyn):
    N = ydyn.shape[1]
    first = _bmtv(qp.A0, y0) + _bmtv(qp.Am[:, 0], ydyn[:, 0])
    last = _bmtv(qp.Ap[:, N - 1], ydyn[:, N - 1])
    if N == 1:
        return np.stack([first, last], axis=1)
    mid = _bmtv(qp.Ap[:, :-1], ydyn[:, :-1]) + _bmtv(qp.Am[:, 1:], ydyn[:, 1:])
    return np.concatenate([first[:, None], mid, last[:, None]], axis=1)


def apply_G(qp: QP, x):
    return _bmv(qp.G, x)


def apply_Gt(qp: QP, y):
    return _bmtv(qp.G, y)


def apply_P(qp: QP, x):
    """admm.py:177-206: P[t,t]=D_t, P[t+1,t]=E_t, P[t,t+1]=E_tᵀ."""
    out = _bmv(qp.D, x)
    out[:, 1:] += _bmv(qp.E, x[:, :-1])
    out[:, :-1] += _bmtv(qp.E, x[:, 1:])
    return out


def compute_gamma(qp: QP, x, z_g, y_g, y_f0, y_fdyn, rho_f, rho_ineq, sigma):
    """admm.py:157-174."""
    rf = np.asarray(rho_f, dtype=x.dtype).reshape(-1, 1)
    ri = np.asarray(rho_ineq, dtype=x.dtype).reshape(-1, 1, 1)
    c0t = rf * qp.c0 - y_f0
    ct = rf[:, :, None] * qp.c - y_fdyn
    eq = apply_Ct(qp, c0t, ct)
    ineq = apply_Gt(qp, ri * z_g - y_g)
    return sigma * x - qp.q + eq + ineq


# ---------------------------------------------------------------------------
# PCG: turbompc/solvers/linear_systems_solvers/pcg_primal.py:70-175 (semantics="jax")
# and admm/csrc/admm_fused.cu:54-161 / pcg_blktridi.cu:96-229 (semantics="cuda")
# ---------------------------------------------------------------------------
def pcg(S, Phiinv, gamma, x0, max_iter, eps, semantics="cuda"):
    """Batched PCG with per-problem stopping.  Returns (x, iters[int64])."""
    x = np.array(x0, copy=True)
    dt = x.dtype
    B = x.shape[0]
    r = gamma - block_tridi_apply(S, x)
    z = block_tridi_apply(Phiinv, r)
    p = z.copy()
    eta = np.einsum("btn,btn->b", r, z)
    eta0 = np.abs(eta)
    iters = np.full(B, max_iter, dtype=np.int64)
    done = np.zeros(B, dtype=bool)
    if semantics == "jax":
        # lax.cond(eta_init_abs <= 1e-12, _already_converged, ...) (pcg_primal.py:158-175)
        short = eta0 <= PCG_ABS_TOL
        iters[short] = 0
        done |= short
    for k in range(max_iter):
        conv = np.abs(eta) < dt.type(PCG_ABS_TOL) + dt.type(eps) * eta0
        if semantics == "jax" and k == 0:
            conv = np.zeros_like(conv)  # `it < 1` forces the first iteration
        newly = conv & ~done
        iters[newly] = k
        done |= conv
        if done.all():
            break
        act = ~done
        Sp = block_tridi_apply(S, p)
        d = np.einsum("btn,btn->b", p, Sp)
        if semantics == "cuda":
            d = np.where(np.abs(d) < dt.type(1e-30), dt.type(1e-30), d)
        with np.errstate(divide="ignore", invalid="ignore"):
            a = np.where(act, eta / d, 0).astype(dt)
        x = x + a[:, None, None] * p
        r = r - a[:, None, None] * Sp
        z = block_tridi_apply(Phiinv, r)
        eta_new = np.einsum("btn,btn->b", r, z)
        with np.errstate(divide="ignore", invalid="ignore"):
            beta = np.where(act, eta_new / eta, 0).astype(dt)
        p = np.where(act[:, None, None], z + beta[:, None, None] * p, p)
        eta = np.where(act, eta_new, eta)
    return x, iters


# ---------------------------------------------------------------------------
# Residuals: admm.py:266-331
# ---------------------------------------------------------------------------
def _inf(a):
    if a.size == 0:
        return np.zeros(a.shape[0], dtype=a.dtype)
    return np.abs(a.reshape(a.shape[0], -1)).max(axis=1)


def residuals(qp: QP, st: ADMMState):
    Cx0, Cx = apply_C_parts(qp, st.x)
    Gx = apply_G(qp, st.x)
    cs = np.concatenate([qp.c0, qp.c.reshape(qp.c.shape[0], -1)], axis=1)
    Cxs = np.concatenate([Cx0, Cx.reshape(Cx.shape[0], -1)], axis=1)
    prim = _inf(Cxs - cs)
    m = qp.G.shape[2]
    gx_n = z_n = np.zeros_like(prim)
    if m > 0:
        prim = np.maximum(prim, _inf(Gx - st.z_g))
        gx_n, z_n = _inf(Gx), _inf(st.z_g)
    prim_term = np.maximum(np.maximum(_inf(Cxs), gx_n), np.maximum(_inf(cs), z_n))
    Px = apply_P(qp, st.x)
    Ct = apply_Ct(qp, st.y_f0, st.y_fdyn)
    Gt = apply_Gt(qp, st.y_g)
    dual = _inf(Px + qp.q + Ct + Gt)
    sw = qp.slack_weight if qp.slack_weight is not None else np.zeros_like(prim)
    if qp.use_slack and m > 0:
        dual = np.maximum(dual, _inf(sw[:, None, None] * st.xi_g + st.y_g))
    dual_term = np.maximum(np.maximum(_inf(Px), _inf(Ct + Gt)), _inf(qp.q))
    if qp.use_slack and m > 0:
        dual_term = np.maximum(dual_term, np.maximum(sw * _inf(st.xi_g), _inf(st.y_g)))
    return prim, dual, prim / (1e-10 + prim_term), dual / (1e-10 + dual_term), prim_term, dual_term


def initial_state(qp: QP, rho, x0=None) -> ADMMState:
    """admm.py:1051-1088: x=0 (or given), z_g=Π(Gx), all duals zero."""
    d = qp.dims
    dt = qp.D.dtype
    x = np.zeros((d["B"], d["T"], d["n"]), dtype=dt) if x0 is None else np.array(x0, dtype=dt)
    z = np.minimum(np.maximum(apply_G(qp, x), qp.l), qp.u)
    return ADMMState(
        x=x, y_g=np.zeros_like(z), y_f0=np.zeros_like(qp.c0), y_fdyn=np.zeros_like(qp.c),
        z_g=z, xi_g=np.zeros_like(z), rho=np.broadcast_to(np.asarray(rho, dtype=dt), (d["B"],)).copy())


# ---------------------------------------------------------------------------
# ADMM loop: fused-kernel order (admm/csrc/admm_fused.cu:701-925).
# ---------------------------------------------------------------------------
def admm_solve(qp: QP, st0: ADMMState, cfg: ADMMConfig, pcg_semantics="cuda", linsys="pcg"):
    """Returns (state, iters).  linsys="pcg" or "dense" (exact Schur solve)."""
    st = st0.copy()
    dt = st.x.dtype
    B = st.x.shape[0]
    m = qp.G.shape[2]
    al = dt.type(cfg.alpha)
    sw = qp.slack_weight if qp.slack_weight is not None else np.zeros(B, dtype=dt)
    S, Pinv = compute_S_Phiinv(qp, st.rho * cfg.rho_f_factor, cfg.sigma, st.rho)
    iters = np.full(B, cfg.max_iter, dtype=np.int64)
    active = np.ones(B, dtype=bool)
    for it in range(cfg.max_iter):
        a3 = active[:, None, None]
        a2 = active[:, None]
        rho = st.rho
        rho_f = rho * dt.type(cfg.rho_f_factor)
        gam = compute_gamma(qp, st.x, st.z_g, st.y_g, st.y_f0, st.y_fdyn, rho_f, rho, cfg.sigma)
        if linsys == "pcg":
            xn, _ = pcg(S, Pinv, gam, st.x, cfg.pcg_max_iter, cfg.pcg_eps, semantics=pcg_semantics)
        else:
            xn = solve_block_tridi_dense(S, gam)
        Cx0, Cx = apply_C_parts(qp, xn)
        Gx = apply_G(qp, xn)
        x_relax = al * xn + (1 - al) * st.x
        z_old = st.z_g
        if m > 0:
            zt = al * Gx + (1 - al) * z_old + st.y_g / rho[:, None, None]
            proj = np.minimum(np.maximum(zt, qp.l), qp.u)
            if cfg.use_slack:
                f = (sw / (sw + rho))[:, None, None]
                z_new = (1 - f) * zt + f * proj
                xi_new = (rho / (sw + rho))[:, None, None] * (proj - zt)
            else:
                z_new, xi_new = proj, st.xi_g
            yg_new = st.y_g + rho[:, None, None] * (al * Gx + (1 - al) * z_old - z_new)
        else:
            z_new, xi_new, yg_new = st.z_g, st.xi_g, st.y_g
        yf0_new = st.y_f0 + (rho_f * al)[:, None] * (Cx0 - qp.c0)
        yfd_new = st.y_fdyn + (rho_f * al)[:, None, None] * (Cx - qp.c)
        st.x = np.where(a3, x_relax, st.x)
        st.z_g = np.where(a3, z_new, st.z_g)
        st.xi_g = np.where(a3, xi_new, st.xi_g)
        st.y_g = np.where(a3, yg_new, st.y_g)
        st.y_f0 = np.where(a2, yf0_new, st.y_f0)
        st.y_fdyn = np.where(a3, yfd_new, st.y_fdyn)
        if cfg.check_every > 0 and it % cfg.check_every == 0:
            pr, du, prn, dun, pt, dtm = residuals(qp, st)
            conv = (pr < cfg.eps_abs + cfg.eps_rel * pt) & (du < cfg.eps_abs + cfg.eps_rel * dtm)
            newly = conv & active
            iters[newly] = it + 1
            active &= ~conv
            if cfg.adapt_rho_every > 0 and it >= 2 and it % cfg.adapt_rho_every == 0:
                with np.errstate(divide="ignore", invalid="ignore"):
                    ratio = np.sqrt(prn / (dun + 1e-30))
                cand = np.clip(st.rho * ratio, cfg.rho_min, cfg.rho_max).astype(dt)
                rr = np.maximum(cand / st.rho, st.rho / cand)
                upd = active & (rr >= cfg.adaptive_rho_tolerance)
                if upd.any():
                    st.rho = np.where(upd, cand, st.rho)
                    S2, P2 = compute_S_Phiinv(qp, st.rho * cfg.rho_f_factor, cfg.sigma, st.rho)
                    S = np.where(upd[:, None, None, None], S2, S)
                    Pinv = np.where(upd[:, None, None, None], P2, Pinv)
        if not active.any():
            break
    return st, iters


# ---------------------------------------------------------------------------
# Adjoint (backward) KKT: turbompc/solvers/backward/backward_kkt_jax.py:10-211
# ---------------------------------------------------------------------------
def assemble_backward_kkt(qp: QP, eps_reg=1e-12):
    """Dense [P Cᵀ; C R] with C = [A0 rows; dynamics rows; G rows] and
    R = -eps_reg on the diagonal of all-zero G rows.  Returns (K, rhs)."""
    d = qp.dims
    B, T, N, n, nx, n0, m = (d[k] for k in ("B", "T", "N", "n", "nx", "n0", "m"))
    nt = T * n
    meq = n0 + N * nx
    mi = T * m
    K = np.zeros((B, nt + meq + mi, nt + meq + mi), dtype=qp.D.dtype)
    for t in range(T):
        r = slice(t * n, (t + 1) * n)
        K[:, r, r] = qp.D[:, t]
        if t < N:
            K[:, (t + 1) * n:(t + 2) * n, r] = qp.E[:, t]
            K[:, r, (t + 1) * n:(t + 2) * n] = np.swapaxes(qp.E[:, t], -1, -2)
    C = np.zeros((B, meq + mi, nt), dtype=qp.D.dtype)
    C[:, :n0, :n] = qp.A0
    for t in range(N):
        rows = slice(n0 + t * nx, n0 + (t + 1) * nx)
        C[:, rows, t * n:(t + 1) * n] = qp.Am[:, t]
        C[:, rows, (t + 1) * n:(t + 2) * n] = qp.Ap[:, t]
    for t in range(T):
        rows = slice(meq + t * m, meq + (t + 1) * m)
        C[:, rows, t * n:(t + 1) * n] = qp.G[:, t]
    K[:, nt:, :nt] = C
    K[:, :nt, nt:] = np.swapaxes(C, -1, -2)
    if mi > 0:
        inactive = (qp.G.reshape(B, mi, n) ** 2).sum(-1) == 0
        idx = np.arange(mi) + nt + meq
        K[:, idx, idx] = np.where(inactive, -eps_reg, 0.0)
    rhs = np.concatenate([-qp.q.reshape(B, nt), np.zeros((B, meq + mi), dtype=qp.D.dtype)], axis=1)
    return K, rhs


def solve_backward_kkt(qp: QP):
    """Returns (dz (B,T,n), multipliers (B, n0+N*nx+T*m))."""
    d = qp.dims
    K, rhs = assemble_backward_kkt(qp)
    sol = np.linalg.solve(K, rhs[..., None])[..., 0]
    nt = d["T"] * d["n"]
    return sol[:, :nt].reshape(d["B"], d["T"], d["n"]), sol[:, nt:]
