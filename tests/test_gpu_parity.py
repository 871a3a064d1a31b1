"""GPU parity: CUDA kernels (through the C ABI) vs the NumPy oracle on the same
seeded inputs.  Tolerances (relative, ||a-b||_inf / ||b||_inf): 1e-6 in fp64
and 1e-3 in fp32 for solver outputs at fixed iteration counts; assembly is
checked tighter (1e-10 fp64 / 1e-4 fp32)."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200 import ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu

DT = {"f64": (torch.float64, np.float64, 1e-6, 1e-10), "f32": (torch.float32, np.float32, 1e-3, 1e-4)}


def _qp(blocks, dt, **kw):
    return synthetic.to_qpdata(blocks, dtype=dt, device="cuda", **kw)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("prec", ["f64", "f32"])
@pytest.mark.parametrize("nx,nu,N,m", [(4, 2, 6, 3), (6, 3, 12, 3), (12, 4, 10, 4), (13, 4, 5, 2), (24, 8, 4, 5),
                                       (2, 1, 1, 0)])
def test_schur_assemble_matches_oracle(prec, nx, nu, N, m):
    tdt, ndt, _, tol = DT[prec]
    b = dense_blocks(5, nx, nu, N, m, seed=nx * 100 + N)
    rho = np.linspace(0.05, 0.5, 5)
    S, P, st = ops.schur_assemble(_qp(b, tdt), torch.tensor(rho, dtype=tdt, device="cuda"), 1e-6, 100.0)
    So, Po = ref.compute_S_Phiinv(oracle_qp(b), rho * 100.0, 1e-6, rho)
    assert (_np(st) == 0).all()
    assert rel_err(_np(S), So) < tol
    assert rel_err(_np(P), Po) < (tol if prec == "f64" else 1e-3)


@pytest.mark.parametrize("prec", ["f64", "f32"])
@pytest.mark.parametrize("nx,nu,N", [(6, 3, 32), (12, 4, 50), (24, 8, 20), (4, 2, 1)])
def test_pcg_reference_layout_matches_oracle(prec, nx, nu, N):
    tdt, ndt, tol, _ = DT[prec]
    b = synthetic.random_lti(6, nx, nu, N, seed=N)
    qp = oracle_qp(b)
    S, P = ref.compute_S_Phiinv(qp, np.full(6, 100.0), 1e-6, np.full(6, 0.1))
    rng = np.random.default_rng(1)
    rhs = rng.normal(size=(6, N + 1, nx + nu))
    x0 = 0.1 * rng.normal(size=rhs.shape)
    xo, ito = ref.pcg(S.astype(ndt), P.astype(ndt), rhs.astype(ndt), x0.astype(ndt), 30, 0.0)
    c = lambda a: torch.tensor(a, dtype=tdt, device="cuda")
    x, it = ops.pcg_solve(c(S), c(P), c(rhs), c(x0), 0.0, 30)
    assert rel_err(_np(x), xo) < tol
    if prec == "f64":
        assert (_np(it) == ito).all()


@pytest.mark.parametrize("prec", ["f64", "f32"])
@pytest.mark.parametrize("nx,nu,N", [(6, 3, 32), (12, 4, 50), (24, 8, 40), (3, 2, 2)])
def test_pcg_packed_matches_oracle(prec, nx, nu, N):
    tdt, ndt, tol, _ = DT[prec]
    Nb = 6
    b = synthetic.random_lti(Nb, nx, nu, N, seed=N + 7)
    qd = _qp(b, tdt)
    ops_buf, st = ops.schur_assemble_packed(qd, 0.1, 1e-6, 1000.0)
    assert (_np(st) == 0).all()
    S, P = ref.compute_S_Phiinv(oracle_qp(b), np.full(Nb, 100.0), 1e-6, np.full(Nb, 0.1))
    rng = np.random.default_rng(2)
    rhs = rng.normal(size=(Nb, N + 1, nx + nu))
    x0 = np.zeros_like(rhs)
    xo, _ = ref.pcg(S, P, rhs, x0, 30, 0.0)
    c = lambda a: torch.tensor(a, dtype=tdt, device="cuda")
    x, it = ops.pcg_solve_packed(ops_buf, ops.dims_of(qd), c(rhs), c(x0), 0.0, 30)
    assert rel_err(_np(x), xo) < tol


def _run_admm(blocks, prec, cfg_kw, slack=None, rho=0.1):
    tdt, ndt, tol, _ = DT[prec]
    use_slack = slack is not None
    Nb = blocks["D"].shape[0]
    sw = None if slack is None else np.full(Nb, slack)
    qd = _qp(blocks, tdt, slack_weight=sw, use_slack=use_slack)
    cfg = ops.AdmmConfig(**cfg_kw, use_slack=use_slack)
    st0 = ops.admm_initial_state(qd, rho)
    out, iters, status = ops.admm_solve(qd, st0, cfg, slack_weight=sw)
    qo = oracle_qp(blocks, slack_weight=sw, use_slack=use_slack)
    rcfg = ref.ADMMConfig(**{k: v for k, v in cfg_kw.items()}, use_slack=use_slack)
    so, io = ref.admm_solve(qo, ref.initial_state(qo, rho), rcfg)
    return out, iters, status, so, io, tol


FIXED = dict(max_iter=50, pcg_max_iter=20, check_every=0, adapt_rho_every=0, eps_abs=0.0, eps_rel=0.0,
             pcg_eps=0.0, rho_f_factor=1000.0, alpha=1.6, sigma=1e-6)


@pytest.mark.parametrize("prec", ["f64", "f32"])
def test_admm_config1_double_integrator(prec):
    """Benchmark configuration 1: nx=4, nu=2, N=20, batch 64, 1 x 50 ADMM x 20 PCG."""
    b = synthetic.double_integrator(batch=64, N=20)
    out, iters, status, so, io, tol = _run_admm(b, prec, FIXED)
    assert (_np(status) == 0).all()
    assert (_np(iters) == 50).all()
    for got, want in ((out.x_blocks, so.x), (out.y_g, so.y_g), (out.z_g, so.z_g), (out.y_f_0, so.y_f0),
                      (out.y_f_dyn, so.y_fdyn)):
        assert rel_err(_np(got), want) < tol


@pytest.mark.parametrize("prec", ["f64", "f32"])
@pytest.mark.parametrize("nx,nu,N,m", [(12, 4, 50, 4), (6, 3, 30, 3), (3, 2, 3, 0), (20, 6, 8, 6)])
def test_admm_dense_problems(prec, nx, nu, N, m):
    b = dense_blocks(8, nx, nu, N, m, seed=11 + N)
    kw = dict(FIXED, max_iter=15, pcg_max_iter=30)
    out, iters, status, so, io, tol = _run_admm(b, prec, kw)
    assert (_np(status) == 0).all()
    assert rel_err(_np(out.x_blocks), so.x) < tol
    assert rel_err(_np(out.y_f_dyn), so.y_fdyn) < tol
    if m:
        assert rel_err(_np(out.z_g), so.z_g) < tol


@pytest.mark.parametrize("prec", ["f64"])
def test_admm_slack_and_residual_checks(prec):
    """Soft constraints (slack update, admm_math.cuh:168-200), residual checks
    and adaptive rho; early termination per problem."""
    b = dense_blocks(6, 4, 2, 10, 3, seed=3)
    # Few PCG iterations (no PCG early stop) keep the residuals far from
    # convergence, where the rho candidate sqrt(p/d) is well conditioned.
    kw = dict(max_iter=60, pcg_max_iter=6, check_every=5, adapt_rho_every=10, eps_abs=1e-3, eps_rel=1e-3,
              pcg_eps=0.0, rho_f_factor=100.0, alpha=1.6, sigma=1e-6)
    out, iters, status, so, io, tol = _run_admm(b, prec, kw, slack=10.0)
    assert (_np(iters) == io).all()
    assert rel_err(_np(out.rho_bar), so.rho) < 1e-9
    assert rel_err(_np(out.x_blocks), so.x) < 1e-6
    assert rel_err(_np(out.xi_g), so.xi_g) < 1e-6


def test_admm_warm_start_chain_matches_single_solve():
    """Two chained solves of 10 iterations == one of 20 (state is the resume unit)."""
    b = synthetic.double_integrator(batch=8, N=12)
    qd = _qp(b, torch.float64)
    cfg10 = ops.AdmmConfig(**dict(FIXED, max_iter=10))
    cfg20 = ops.AdmmConfig(**dict(FIXED, max_iter=20))
    s0 = ops.admm_initial_state(qd, 0.1)
    a, _, _ = ops.admm_solve(qd, s0, cfg10)
    a, _, _ = ops.admm_solve(qd, a, cfg10)
    c, _, _ = ops.admm_solve(qd, s0, cfg20)
    assert rel_err(_np(a.x_blocks), _np(c.x_blocks)) < 1e-12


def test_admm_empty_batch_and_in_place():
    b = synthetic.double_integrator(batch=3, N=5)
    qd = _qp(b, torch.float64)
    s0 = ops.admm_initial_state(qd, 0.1)
    cfg = ops.AdmmConfig(**FIXED)
    ref_out, _, _ = ops.admm_solve(qd, s0, cfg)
    inplace, _, _ = ops.admm_solve(qd, s0, cfg, out=s0)  # state_out aliases state_in
    assert rel_err(_np(inplace.x_blocks), _np(ref_out.x_blocks)) == 0.0
    q0 = qd.slice(0, 0)
    e, it, st = ops.admm_solve(q0, ops.admm_initial_state(q0, 0.1), cfg)
    assert e.x_blocks.shape[0] == 0


def test_singular_theta_sets_status_without_fault():
    """A singular Theta block is reported per problem (status bit), not trapped."""
    b = dense_blocks(3, 2, 1, 3, 0, seed=4)
    b["D"][1] = 0.0
    b["Am"][1] = 0.0
    b["Ap"][1] = 0.0
    b["A0"][1] = 0.0
    qd = _qp(b, torch.float64)
    _, _, st = ops.schur_assemble(qd, 0.1, 0.0, 10.0)
    st = _np(st)
    assert st[1] & 1 and st[0] == 0 and st[2] == 0
