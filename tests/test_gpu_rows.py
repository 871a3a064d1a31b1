"""GPU parity of the register-resident fused ADMM kernel (fp32, 8 < n <= 16,
T <= 64; chosen automatically for TMPC_LINSYS_PCG) against the NumPy oracle,
and against the shared-memory packed kernel (TMPC_LINSYS_PCG_PACKED).
Tolerance: 1e-3 relative (||a-b||_inf / ||b||_inf), the fp32 bar."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200 import _ffi, ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu

FIXED = dict(max_iter=30, pcg_max_iter=30, check_every=0, adapt_rho_every=0, eps_abs=0.0, eps_rel=0.0,
             pcg_eps=0.0, rho_f_factor=1000.0, alpha=1.6, sigma=1e-6)


def _np(t):
    return t.detach().cpu().numpy()


def _solve(blocks, cfg_kw, linsys=_ffi.LINSYS_PCG, slack=None, rho=0.1):
    Nb = blocks["D"].shape[0]
    sw = None if slack is None else np.full(Nb, slack)
    qd = synthetic.to_qpdata(blocks, dtype=torch.float32, device="cuda", slack_weight=sw,
                             use_slack=slack is not None)
    cfg = ops.AdmmConfig(**cfg_kw, use_slack=slack is not None, linsys=linsys)
    return ops.admm_solve(qd, ops.admm_initial_state(qd, rho), cfg, slack_weight=sw)


def _oracle(blocks, cfg_kw, slack=None, rho=0.1):
    Nb = blocks["D"].shape[0]
    sw = None if slack is None else np.full(Nb, slack)
    qo = oracle_qp(blocks, slack_weight=sw, use_slack=slack is not None)
    return ref.admm_solve(qo, ref.initial_state(qo, rho), ref.ADMMConfig(**cfg_kw, use_slack=slack is not None))


@pytest.mark.parametrize("nx,nu,N,m", [(12, 4, 50, 4),   # quadrotor shape (n = 16, T = 51)
                                       (12, 4, 51, 4),   # T = 52: every thread owns a stage
                                       (6, 3, 30, 3),    # n = 9: padded rows
                                       (10, 2, 1, 2),    # T = 2
                                       (8, 5, 17, 0),    # no inequalities
                                       (11, 5, 40, 7)])
def test_rows_kernel_matches_oracle(nx, nu, N, m):
    b = dense_blocks(6, nx, nu, N, m, seed=100 + N + m)
    out, iters, status = _solve(b, FIXED)
    so, _ = _oracle(b, FIXED)
    assert (_np(status) == 0).all()
    assert (_np(iters) == FIXED["max_iter"]).all()
    assert rel_err(_np(out.x_blocks), so.x) < 1e-3
    assert rel_err(_np(out.y_f_dyn), so.y_fdyn) < 1e-3
    assert rel_err(_np(out.y_f_0), so.y_f0) < 1e-3
    if m:
        assert rel_err(_np(out.z_g), so.z_g) < 1e-3
        assert rel_err(_np(out.y_g), so.y_g) < 1e-3


@pytest.mark.parametrize("nx,nu,N,m", [(6, 3, 60, 3),    # T = 61, n = 9: the config-5 shape
                                       (10, 2, 58, 2),   # T = 59, n = 12
                                       (10, 2, 52, 2),   # T = 53: the first horizon of this instance
                                       (6, 3, 63, 3)])   # T = 64: the largest
def test_rows_kernel_64_stage_instance(nx, nu, N, m):
    """Horizons with 52 < T <= 64 run the 64-stage instance (512 threads).
    It must match the oracle, and it must be the kernel that ran: its
    rounding differs from the packed kernel's on the same problems."""
    b = dense_blocks(4, nx, nu, N, m, seed=7 + N)
    out, iters, status = _solve(b, FIXED)
    packed, _, _ = _solve(b, FIXED, linsys=_ffi.LINSYS_PCG_PACKED)
    so, _ = _oracle(b, FIXED)
    assert (_np(status) == 0).all()
    assert (_np(iters) == FIXED["max_iter"]).all()
    assert rel_err(_np(out.x_blocks), so.x) < 1e-3
    assert rel_err(_np(out.y_f_dyn), so.y_fdyn) < 1e-3
    assert rel_err(_np(out.z_g), so.z_g) < 1e-3
    assert not torch.equal(out.x_blocks, packed.x_blocks)


def test_rows_kernel_lti_config_matches_packed_kernel():
    """Quadrotor-sized LTI batch: register-resident and packed kernels agree to
    fp32 rounding (and are different code paths: not bit-identical)."""
    b = synthetic.random_lti(64, 12, 4, 50, seed=5)
    a, _, sa = _solve(b, FIXED)
    p, _, sp = _solve(b, FIXED, linsys=_ffi.LINSYS_PCG_PACKED)
    so, _ = _oracle(b, FIXED)
    assert (_np(sa) == 0).all() and (_np(sp) == 0).all()
    assert rel_err(_np(a.x_blocks), _np(p.x_blocks)) < 1e-3
    assert rel_err(_np(a.x_blocks), so.x) < 1e-3
    assert not torch.equal(a.x_blocks, p.x_blocks)


def test_rows_kernel_slack_residual_checks_and_rho_adaptation():
    """Soft constraints, residual checks every 5 iterations and an OSQP rho
    update at iteration 10 with the on-chip rebuild of the operators, followed
    by two iterations on the rebuilt operators.  Tolerance 1.0 makes every
    problem take the update (no borderline accept/reject decision); stopping
    after one update keeps the rho rule rho * sqrt(p / d) well conditioned
    (later updates, near convergence, amplify fp32 rounding of the residual
    norms by orders of magnitude, in the fp32 oracle as much as here)."""
    b = dense_blocks(6, 10, 4, 12, 3, seed=3)
    kw = dict(max_iter=12, pcg_max_iter=6, check_every=5, adapt_rho_every=10, eps_abs=1e-9, eps_rel=1e-9,
              pcg_eps=0.0, rho_f_factor=100.0, alpha=1.6, sigma=1e-6, adaptive_rho_tolerance=1.0)
    out, iters, status = _solve(b, kw, slack=10.0)
    so, io = _oracle(b, kw, slack=10.0)
    assert (_np(status) == 0).all()
    assert (io == 12).all() and (_np(iters) == 12).all()
    assert (np.abs(so.rho - 0.1) > 1e-2).all(), "every problem must take the rho update"
    assert rel_err(_np(out.rho_bar), so.rho) < 1e-3
    assert rel_err(_np(out.x_blocks), so.x) < 1e-3
    assert rel_err(_np(out.xi_g), so.xi_g) < 1e-3
    assert rel_err(_np(out.y_g), so.y_g) < 1e-3


def test_rows_kernel_convergence_stop():
    """Per-problem early termination at a residual check: the stop iteration
    is within one check period of the fp64 oracle's (fp32 residual norms can
    move a borderline check), and equal for most problems."""
    b = synthetic.random_lti(8, 10, 4, 12, seed=3)
    kw = dict(max_iter=200, pcg_max_iter=20, check_every=5, adapt_rho_every=0, eps_abs=1e-2, eps_rel=1e-2,
              pcg_eps=0.0, rho_f_factor=100.0, alpha=1.6, sigma=1e-6)
    out, iters, status = _solve(b, kw)
    so, io = _oracle(b, kw)
    it = _np(iters)
    assert (_np(status) == 0).all()
    assert (io < 200).all(), "every problem must stop early in the oracle"
    assert (np.abs(it - io) <= 5).all()
    same = it == io
    assert same.sum() >= 6
    assert rel_err(_np(out.x_blocks)[same], so.x[same]) < 1e-2


def test_rows_kernel_pcg_early_stop():
    """PCG tolerance > 0: the per-solve stop test |eta| < 1e-12 + eps |eta0|.
    eta = r.z is a squared norm, so eps = 1e-4 stops at about 1e-2 of the
    initial residual, and an fp32 stop decision near the threshold can fall
    one iteration from the fp64 oracle's.  The early stops move the oracle's
    solution by `shift` (5e-3 relative here) away from the full-count one; the
    kernel must follow the stopped iterates: within shift / 2 of the oracle's
    stopped solution (measured 1.1e-3) and farther from the full-count one."""
    b = dense_blocks(4, 12, 4, 20, 4, seed=9)
    kw = dict(FIXED, max_iter=10, pcg_max_iter=50, pcg_eps=1e-4)
    out, _, status = _solve(b, kw)
    so, _ = _oracle(b, kw)
    so_full, _ = _oracle(b, dict(kw, pcg_eps=0.0))
    assert (_np(status) == 0).all()
    shift = rel_err(so.x, so_full.x)
    assert shift > 1e-3, "the stop test must change the result for this check to mean anything"
    x = _np(out.x_blocks)
    assert rel_err(x, so.x) < 0.5 * shift
    assert rel_err(x, so_full.x) > rel_err(x, so.x)


@pytest.mark.parametrize("linsys", [_ffi.LINSYS_PCG, _ffi.LINSYS_PCG_PACKED])
def test_initial_control_constraint_rows(linsys):
    """n0 = n (constrain_initial_control: A0 = I over states and controls):
    both fp32 kernels against the oracle."""
    b = dense_blocks(4, 10, 4, 20, 3, seed=21)
    n = 14
    b = dict(b)
    b["A0"] = np.repeat(np.eye(n)[None], 4, 0)
    b["c0"] = np.random.default_rng(0).normal(size=(4, n))
    out, iters, status = _solve(b, FIXED, linsys=linsys)
    so, _ = _oracle(b, FIXED)
    assert (_np(status) == 0).all()
    assert rel_err(_np(out.x_blocks), so.x) < 1e-3
    assert rel_err(_np(out.y_f_0), so.y_f0) < 1e-3
