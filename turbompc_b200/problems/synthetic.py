"""Seeded synthetic QPs for the benchmark configurations that are linear.

The QPs are what TurboMPC's OptimalControlProblem linearisation
(turbompc/problems/optimal_control_problem.py:1068-1332) produces for linear
dynamics written with the reference's "dt = 1 Euler" trick
(benchmarking/linear-system/benchmark_turbompc_constrained.py:87-95):
A_minus = [A B], A_plus = [-I 0], c = 0, A0 = [I 0], c0 = x0.  The cost
convention is sum w (z - ref)^2 without a 1/2 (optimal_control_problem.py:
1003-1008), so the Hessian blocks are 2 diag(w); with a zero reference q = 0.

Generators return a dict of NumPy arrays with a leading batch axis, keys
D, E, q, A0, Am, Ap, c0, c, G, l, u (reference layout).
"""
from __future__ import annotations

import numpy as np


def _assemble(A, B, Qd, Rd, Qf, Rf, x0, G, lo, hi, N):
    """A (Nb,nx,nx), B (Nb,nx,nu), diagonal weights (Nb,nx)/(Nb,nu)."""
    Nb, nx, nu = B.shape
    n = nx + nu
    T = N + 1
    D = np.zeros((Nb, T, n, n))
    for t in range(T):
        w = np.concatenate([Qf if t == N else Qd, Rf if t == N else Rd], axis=1)
        D[:, t, np.arange(n), np.arange(n)] = 2.0 * w
    E = np.zeros((Nb, N, n, n))
    q = np.zeros((Nb, T, n))
    A0 = np.broadcast_to(np.concatenate([np.eye(nx), np.zeros((nx, nu))], 1), (Nb, nx, n)).copy()
    Am = np.broadcast_to(np.concatenate([A, B], axis=2)[:, None], (Nb, N, nx, n)).copy()
    Ap = np.broadcast_to(np.concatenate([-np.eye(nx), np.zeros((nx, nu))], 1), (Nb, N, nx, n)).copy()
    c = np.zeros((Nb, N, nx))
    m = G.shape[0]
    Gb = np.broadcast_to(G, (Nb, T, m, n)).copy()
    l = np.broadcast_to(lo, (Nb, T, m)).copy()
    u = np.broadcast_to(hi, (Nb, T, m)).copy()
    return dict(D=D, E=E, q=q, A0=A0, Am=Am, Ap=Ap, c0=x0.copy(), c=c, G=Gb, l=l, u=u)


def double_integrator(batch=64, N=20, dt=0.1, seed=0):
    """Config 1: nx=4, nu=2, Q=I, R=0.1 I, Qf=10 I, |u|<=1, |x|<=10, x0 ~ U(-2,2)."""
    rng = np.random.default_rng(seed)
    I2 = np.eye(2)
    A = np.block([[I2, dt * I2], [np.zeros((2, 2)), I2]])
    B = np.concatenate([0.5 * dt * dt * I2, dt * I2], axis=0)
    A = np.broadcast_to(A, (batch, 4, 4))
    B = np.broadcast_to(B, (batch, 4, 2))
    Qd = np.ones((batch, 4))
    Rd = 0.1 * np.ones((batch, 2))
    Qf = 10.0 * np.ones((batch, 4))
    x0 = rng.uniform(-2.0, 2.0, size=(batch, 4))
    G = np.eye(6)
    lo = np.array([-10.0] * 4 + [-1.0] * 2)
    hi = -lo
    return _assemble(A, B, Qd, Rd, Qf, Rd, x0, G, lo, hi, N)


def random_lti(batch, nx, nu, N, seed=0, u_bound=1.0):
    """Config 2: A = I + 0.1 G, G ~ N(0, 1/nx); B ~ N(0, 1/nu); Q, R diagonal
    ~ U(0.5, 2); x0 ~ N(0, I); box |u| <= u_bound (m = nu)."""
    rng = np.random.default_rng(seed)
    A = np.eye(nx) + 0.1 * rng.normal(0.0, 1.0 / np.sqrt(nx), size=(batch, nx, nx))
    B = rng.normal(0.0, 1.0 / np.sqrt(nu), size=(batch, nx, nu))
    Qd = rng.uniform(0.5, 2.0, size=(batch, nx))
    Rd = rng.uniform(0.5, 2.0, size=(batch, nu))
    x0 = rng.normal(size=(batch, nx))
    G = np.concatenate([np.zeros((nu, nx)), np.eye(nu)], axis=1)
    lo = -u_bound * np.ones(nu)
    return _assemble(A, B, Qd, Rd, Qd, Rd, x0, G, lo, -lo, N)


def random_dense(batch, nx, nu, N, m, seed=0):
    """General dense blocks (non-zero E, q, c, affine A_plus, random G) for
    parity tests that must exercise every term of the algorithm."""
    rng = np.random.default_rng(seed)
    n = nx + nu
    T = N + 1
    L = rng.normal(size=(batch, T, n, n)) / np.sqrt(n)
    D = np.einsum("btij,btkj->btik", L, L) + 0.5 * np.eye(n)
    E = 0.1 * rng.normal(size=(batch, N, n, n))
    q = rng.normal(size=(batch, T, n))
    A0 = np.concatenate([np.eye(nx), np.zeros((nx, nu))], 1)[None].repeat(batch, 0)
    Am = np.concatenate([np.eye(nx) + 0.1 * rng.normal(size=(batch, N, nx, nx)),
                         rng.normal(size=(batch, N, nx, nu)) / np.sqrt(nu)], axis=3)
    Ap = np.concatenate([-np.eye(nx) + 0.05 * rng.normal(size=(batch, N, nx, nx)),
                         0.05 * rng.normal(size=(batch, N, nx, nu))], axis=3)
    c0 = rng.normal(size=(batch, nx))
    c = 0.1 * rng.normal(size=(batch, N, nx))
    G = rng.normal(size=(batch, T, m, n)) / np.sqrt(n)
    l = -0.5 - rng.uniform(size=(batch, T, m))
    u = 0.5 + rng.uniform(size=(batch, T, m))
    return dict(D=D, E=E, q=q, A0=A0, Am=Am, Ap=Ap, c0=c0, c=c, G=G, l=l, u=u)


def to_qpdata(blocks, dtype=None, device=None, slack_weight=None, use_slack=False):
    """Dict of NumPy arrays -> turbompc_b200.qp_data.QPData (torch tensors)."""
    import torch

    from ..qp_data import QPCostBlocks, QPData, QPEqualityBlocks, QPInequalityBlocks

    dtype = dtype or torch.float64
    t = {k: torch.as_tensor(np.ascontiguousarray(v), dtype=dtype, device=device) for k, v in blocks.items()}
    sw = None if slack_weight is None else torch.as_tensor(slack_weight, dtype=dtype, device=device)
    return QPData(QPCostBlocks(t["D"], t["E"], t["q"]),
                  QPEqualityBlocks(t["A0"], t["Am"], t["Ap"], t["c0"], t["c"]),
                  QPInequalityBlocks(t["G"], t["l"], t["u"], sw, use_slack))
