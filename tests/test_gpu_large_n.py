"""Stage blocks wider than 32 (32 < n <= 96; the reference's dimension sweep
reaches (nx, nu) = (64, 32), benchmarking/linear-system/
run_sweeps_oat_turbompc.sh:122): the reference-layout assembly
(compute_S_Phiinv, admm.py:71-154), the standalone PCG and the fused ADMM
solve against the NumPy oracle, fp64 at 1e-6 relative (assembly 1e-10) and
fp32 at 1e-3, including residual checks and rho adaptation (per-problem
iteration counts equal to the oracle's)."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err, wide_problem
from turbompc_b200 import _ffi, ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu
KEYS = ("x_blocks", "y_g", "y_f_0", "y_f_dyn", "z_g", "xi_g", "rho_bar")
OKEYS = ("x", "y_g", "y_f0", "y_fdyn", "z_g", "xi_g", "rho")


@pytest.mark.parametrize("nx,nu", [(32, 16), (45, 25), (64, 32)])
def test_schur_assembly_wide_blocks_matches_oracle(nx, nu):
    b = dense_blocks(3, nx, nu, 5, 4, seed=nx)
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    rho = torch.tensor([0.1, 0.3, 1.0], dtype=torch.float64, device="cuda")
    S, P, st = ops.schur_assemble(qd, rho, 1e-6, 100.0)
    assert int(st.abs().sum()) == 0
    q = oracle_qp(b)
    So, Po = ref.compute_S_Phiinv(q, rho.cpu().numpy() * 100.0, 1e-6, rho.cpu().numpy())
    assert rel_err(S.cpu().numpy(), So) < 1e-10
    assert rel_err(P.cpu().numpy(), Po) < 1e-9


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_pcg_wide_blocks_matches_oracle(dtype):
    b = wide_problem(4, 32, 16, 8, 4, seed=3)
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    S, P, _ = ops.schur_assemble(qd, 0.1, 1e-6, 100.0)
    g = torch.Generator(device="cuda").manual_seed(1)
    rhs = torch.randn(4, 9, 48, generator=g, device="cuda", dtype=torch.float64)
    x0 = torch.zeros_like(rhs)
    x, it = ops.pcg_solve(S.to(dtype), P.to(dtype), rhs.to(dtype), x0.to(dtype), 0.0, 25)
    xr, itr = ref.pcg(S.cpu().numpy(), P.cpu().numpy(), rhs.cpu().numpy(), x0.cpu().numpy(), 25, 0.0)
    if dtype == torch.float64:
        assert (it.cpu().numpy() == itr).all()
    assert rel_err(x.cpu().numpy(), xr) < (1e-6 if dtype == torch.float64 else 1e-3)


def _run(b, dtype, cfg, slack=None):
    qd = synthetic.to_qpdata(b, dtype=dtype, device="cuda")
    Nb = b["D"].shape[0]
    c = ops.AdmmConfig(**cfg, use_slack=slack is not None)
    assert ops.admm_workspace_bytes(qd, c) > 0
    out, it, st = ops.admm_solve(qd, ops.admm_initial_state(qd, 0.1), c,
                                 slack_weight=None if slack is None else np.full(Nb, slack))
    assert int(st.abs().sum()) == 0
    q = oracle_qp(b, slack_weight=None if slack is None else np.full(Nb, slack), use_slack=slack is not None)
    oc = ref.ADMMConfig(**{k: cfg[k] for k in ("max_iter", "pcg_max_iter", "check_every", "eps_abs", "eps_rel",
                                               "sigma", "rho_f_factor", "alpha", "pcg_eps", "adapt_rho_every",
                                               "adaptive_rho_tolerance", "rho_min", "rho_max")},
                        use_slack=slack is not None)
    so, ito = ref.admm_solve(q, ref.initial_state(q, 0.1), oc)
    return out, it, so, ito


FIXED = dict(max_iter=12, pcg_max_iter=20, check_every=0, adapt_rho_every=0, eps_abs=0.0, eps_rel=0.0, pcg_eps=0.0,
             sigma=1e-6, rho_f_factor=100.0, alpha=1.6, adaptive_rho_tolerance=5.0, rho_min=1e-6, rho_max=1e6)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("nx,nu,N", [(32, 16, 10), (40, 20, 6), (64, 32, 5)])
def test_fused_admm_wide_blocks_matches_oracle(dtype, nx, nu, N):
    b = wide_problem(3, nx, nu, N, 6, seed=nx + N)
    out, it, so, ito = _run(b, dtype, FIXED)
    tol = 1e-6 if dtype == torch.float64 else 1e-3
    assert (it.cpu().numpy() == ito).all()
    for k, ok in zip(KEYS, OKEYS):
        assert rel_err(getattr(out, k).cpu().numpy(), getattr(so, ok)) < tol, k


def test_fused_admm_wide_blocks_checks_slack_and_rho_adaptation_fp64():
    b = wide_problem(4, 32, 16, 6, 4, seed=9)
    cfg = dict(FIXED, max_iter=60, pcg_max_iter=8, check_every=5, adapt_rho_every=10, eps_abs=1e-4, eps_rel=1e-4)
    out, it, so, ito = _run(b, torch.float64, cfg, slack=10.0)
    assert (it.cpu().numpy() == ito).all(), (it, ito)
    for k, ok in zip(KEYS, OKEYS):
        assert rel_err(getattr(out, k).cpu().numpy(), getattr(so, ok)) < 1e-6, k


def test_wide_blocks_limits():
    lib = _ffi.load()
    d = _ffi.TmpcDims(2, 4, 97, 60, 60, 0)
    c = ops.AdmmConfig().to_c()
    import ctypes as C
    assert lib.tmpc_admm_workspace_bytes(C.byref(d), 8, C.byref(c)) == 0  # beyond 96: no path
