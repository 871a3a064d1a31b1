"""GPU parity of the HBM-streaming PCG (tmpc_pcg_solve_stream_*) and its
operator assembly (tmpc_schur_assemble_stream_*) against the NumPy oracle.
Tolerances (relative, ||a-b||_inf / ||b||_inf): assembly 1e-10 fp64 / 1e-4
fp32; PCG solution 1e-6 fp64 / 1e-3 fp32 at fixed iteration counts."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200 import _ffi, ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu
DT = {"f64": (torch.float64, np.float64, 1e-6, 1e-10), "f32": (torch.float32, np.float32, 1e-3, 1e-4)}
NBS = [8, 12, 16, 24, 32]


def _nb(n):
    return next(b for b in NBS if b >= n)


def _unpack(opsf, B, T, n):
    """Stream layout -> reference layout (B, T, n, 3n) for S and Phiinv."""
    NB = _nb(n)
    a = opsf.detach().cpu().numpy().reshape(B, 2, 2 * T - 1, NB, NB)
    out = []
    for k in range(2):
        M = np.zeros((B, T, n, 3 * n))
        D = a[:, k, :T, :n, :n]
        L = a[:, k, T:, :n, :n]
        M[:, :, :, n:2 * n] = D
        M[:, 1:, :, :n] = L
        M[:, :-1, :, 2 * n:] = np.swapaxes(L, -1, -2)
        out.append(M)
    return out


@pytest.mark.parametrize("prec", ["f64", "f32"])
@pytest.mark.parametrize("nx,nu,N,m", [(6, 3, 12, 3), (12, 4, 20, 4), (24, 8, 6, 5), (3, 2, 2, 0)])
def test_stream_assembly_matches_oracle(prec, nx, nu, N, m):
    tdt, _, _, tol = DT[prec]
    b = dense_blocks(4, nx, nu, N, m, seed=nx + N)
    rho = np.linspace(0.05, 0.4, 4)
    qd = synthetic.to_qpdata(b, dtype=tdt, device="cuda")
    o, st = ops.schur_assemble_stream(qd, torch.tensor(rho, dtype=tdt, device="cuda"), 1e-6, 100.0)
    S, P = _unpack(o, 4, N + 1, nx + nu)
    So, Po = ref.compute_S_Phiinv(oracle_qp(b), rho * 100.0, 1e-6, rho)
    assert (st.cpu().numpy() == 0).all()
    assert rel_err(S, So) < tol
    assert rel_err(P, Po) < (tol if prec == "f64" else 1e-3)


@pytest.mark.parametrize("prec", ["f64", "f32"])
@pytest.mark.parametrize("nx,nu,N", [(6, 3, 32), (12, 4, 64), (24, 8, 128), (4, 2, 1)])
def test_stream_pcg_matches_oracle(prec, nx, nu, N):
    tdt, ndt, tol, _ = DT[prec]
    B, T, n = 5, N + 1, nx + nu
    blk = synthetic.random_lti(B, nx, nu, N, seed=N)
    qd = synthetic.to_qpdata(blk, dtype=tdt, device="cuda")
    o, st = ops.schur_assemble_stream(qd, 0.1, 1e-6, 100.0)
    S, P = ref.compute_S_Phiinv(oracle_qp(blk), np.full(B, 10.0), 1e-6, np.full(B, 0.1))
    rng = np.random.default_rng(2)
    rhs = rng.normal(size=(B, T, n))
    x0 = 0.1 * rng.normal(size=rhs.shape)
    xo, ito = ref.pcg(S.astype(ndt), P.astype(ndt), rhs.astype(ndt), x0.astype(ndt), 30, 0.0)
    c = lambda a: torch.tensor(a, dtype=tdt, device="cuda")
    x, it = ops.pcg_solve_stream(o, _ffi.TmpcDims(B, T, n, nx, 0, 0), c(rhs), c(x0), 0.0, 30)
    assert rel_err(x.cpu().numpy(), xo) < tol
    assert (it.cpu().numpy() == ito).all()


def test_stream_pcg_early_stop_and_empty_batch():
    blk = synthetic.random_lti(4, 12, 4, 20, seed=3)
    qd = synthetic.to_qpdata(blk, dtype=torch.float64, device="cuda")
    o, _ = ops.schur_assemble_stream(qd, 0.1, 1e-6, 100.0)
    S, P = ref.compute_S_Phiinv(oracle_qp(blk), np.full(4, 10.0), 1e-6, np.full(4, 0.1))
    rhs = np.random.default_rng(3).normal(size=(4, 21, 16))
    xo, ito = ref.pcg(S, P, rhs, np.zeros_like(rhs), 200, 1e-8)
    c = lambda a: torch.tensor(a, dtype=torch.float64, device="cuda")
    x, it = ops.pcg_solve_stream(o, _ffi.TmpcDims(4, 21, 16, 12, 0, 0), c(rhs), c(np.zeros_like(rhs)), 1e-8, 200)
    assert (it.cpu().numpy() == ito).all() and (ito < 200).all()
    assert rel_err(x.cpu().numpy(), xo) < 1e-6
    e = torch.zeros(0, 21, 16, dtype=torch.float64, device="cuda")
    x, it = ops.pcg_solve_stream(o, _ffi.TmpcDims(0, 21, 16, 12, 0, 0), e, e, 0.0, 30)
    assert x.shape[0] == 0
