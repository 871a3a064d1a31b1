"""GPU parity of the direct (block Cholesky / Riccati) path, which replaces
the reference's cuDSS solves.  The reference pins cuDSS only against dense
solves (tests/cuda/backends/test_cudss_ffi_backend.py:19-40,
test_admm_math_cuda_vs_python.py:221-253), so the oracle here is the dense LU
solve of the same Schur system.  Tolerances as in test_gpu_parity.py."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200 import ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu
TOL = {torch.float64: 1e-6, torch.float32: 1e-3}


@pytest.mark.parametrize("dt", [torch.float64, torch.float32])
@pytest.mark.parametrize("nx,nu,N", [(6, 3, 32), (12, 4, 50), (24, 8, 20), (4, 2, 1), (3, 1, 7)])
def test_riccati_solve_matches_dense(dt, nx, nu, N):
    Nb = 5
    b = synthetic.random_lti(Nb, nx, nu, N, seed=N + nx)
    S, _ = ref.compute_S_Phiinv(oracle_qp(b), np.full(Nb, 100.0), 1e-6, np.full(Nb, 0.1))
    rng = np.random.default_rng(3)
    rhs = rng.normal(size=(Nb, N + 1, nx + nu))
    xd = ref.solve_block_tridi_dense(S, rhs)
    c = lambda a: torch.tensor(a, dtype=dt, device="cuda")
    fac, st = ops.riccati_factor(c(S))
    x = ops.riccati_solve(fac, c(rhs))
    assert int(st.abs().sum()) == 0
    assert rel_err(x.cpu().numpy(), xd) < TOL[dt]


def test_riccati_reuses_caller_buffers():
    """Factor / solve into caller-provided buffers, twice with different
    systems: the second result does not depend on the first one's contents."""
    Nb, nx, nu, N = 4, 12, 4, 30
    c = lambda a: torch.tensor(a, dtype=torch.float64, device="cuda")
    rng = np.random.default_rng(11)
    fac = st = x = None
    for seed in (5, 6):
        b = synthetic.random_lti(Nb, nx, nu, N, seed=seed)
        S, _ = ref.compute_S_Phiinv(oracle_qp(b), np.full(Nb, 50.0), 1e-6, np.full(Nb, 0.1))
        rhs = rng.normal(size=(Nb, N + 1, nx + nu))
        if fac is None:
            fac, st = ops.riccati_factor(c(S))
            x = torch.empty(Nb, N + 1, nx + nu, dtype=torch.float64, device="cuda")
        else:
            f2, s2 = ops.riccati_factor(c(S), fac, st)
            assert f2.data_ptr() == fac.data_ptr() and s2.data_ptr() == st.data_ptr()
        out = ops.riccati_solve(fac, c(rhs), x)
        assert out.data_ptr() == x.data_ptr()
        assert int(st.abs().sum()) == 0
        assert rel_err(x.cpu().numpy(), ref.solve_block_tridi_dense(S, rhs)) < TOL[torch.float64]


def test_riccati_reports_indefinite():
    b = synthetic.random_lti(3, 4, 2, 5, seed=1)
    S, _ = ref.compute_S_Phiinv(oracle_qp(b), np.full(3, 10.0), 1e-6, np.full(3, 0.1))
    S[1, 2, :, 6:12] *= -1.0  # make a diagonal block negative definite
    fac, st = ops.riccati_factor(torch.tensor(S, device="cuda"))
    st = st.cpu().numpy()
    assert st[1] & 1 and st[0] == 0 and st[2] == 0


FIXED = dict(max_iter=40, pcg_max_iter=1, check_every=0, adapt_rho_every=0, eps_abs=0.0, eps_rel=0.0, pcg_eps=0.0,
             rho_f_factor=1000.0, alpha=1.6, sigma=1e-6)


@pytest.mark.parametrize("dt", [torch.float64, torch.float32])
@pytest.mark.parametrize("case", ["dbl_int", "dense16", "dense_m0"])
def test_admm_direct_matches_dense_schur_oracle(dt, case):
    if case == "dbl_int":
        b = synthetic.double_integrator(batch=16, N=20)
    elif case == "dense16":
        b = dense_blocks(6, 12, 4, 12, 4, seed=9)
    else:
        b = dense_blocks(4, 3, 2, 6, 0, seed=10)
    qd = synthetic.to_qpdata(b, dtype=dt, device="cuda")
    cfg = ops.AdmmConfig(**FIXED, linsys=ops._ffi.LINSYS_DIRECT)
    out, it, st = ops.admm_solve(qd, ops.admm_initial_state(qd, 0.1), cfg)
    qo = oracle_qp(b)
    so, _ = ref.admm_solve(qo, ref.initial_state(qo, 0.1), ref.ADMMConfig(**FIXED), linsys="dense")
    assert int(st.abs().sum()) == 0
    for g, w in ((out.x_blocks, so.x), (out.y_f_dyn, so.y_fdyn), (out.z_g, so.z_g)):
        assert rel_err(g.cpu().numpy(), w) < TOL[dt]


def test_admm_direct_adaptive_rho_refactors():
    b = dense_blocks(6, 4, 2, 10, 3, seed=3)
    kw = dict(max_iter=60, pcg_max_iter=1, check_every=5, adapt_rho_every=10, eps_abs=1e-3, eps_rel=1e-3,
              pcg_eps=0.0, rho_f_factor=100.0, alpha=1.6, sigma=1e-6)
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    out, it, st = ops.admm_solve(qd, ops.admm_initial_state(qd, 0.1),
                                 ops.AdmmConfig(**kw, linsys=ops._ffi.LINSYS_DIRECT))
    qo = oracle_qp(b)
    so, io = ref.admm_solve(qo, ref.initial_state(qo, 0.1), ref.ADMMConfig(**kw), linsys="dense")
    assert (it.cpu().numpy() == io).all()
    assert rel_err(out.rho_bar.cpu().numpy(), so.rho) < 1e-9
    assert rel_err(out.x_blocks.cpu().numpy(), so.x) < 1e-6


@pytest.mark.parametrize("dt", [torch.float64, torch.float32])
def test_admm_direct_structured_and_general_groups_in_one_batch(dt):
    """The interleaved direct path checks per group of 32 problems whether
    A+_t = [-I 0] and whether every inequality row is a unit vector on the
    same columns, and then stops streaming those matrices.  A batch of 70
    problems (three groups, the last ragged) with one perturbed A+ in group 1
    and one perturbed G row in group 2 runs group 0 on the structured form and
    the others on the general one; all match the dense oracle."""
    b = synthetic.random_lti(70, 6, 3, 12, seed=4)
    b["Ap"][40, 2, 0, 1] = 0.01
    b["G"][65, 3, 1, 0] = 0.2
    qd = synthetic.to_qpdata(b, dtype=dt, device="cuda")
    cfg = ops.AdmmConfig(**FIXED, linsys=ops._ffi.LINSYS_DIRECT)
    out, it, st = ops.admm_solve(qd, ops.admm_initial_state(qd, 0.1), cfg)
    qo = oracle_qp(b)
    so, _ = ref.admm_solve(qo, ref.initial_state(qo, 0.1), ref.ADMMConfig(**FIXED), linsys="dense")
    assert int(st.abs().sum()) == 0
    for g, w in ((out.x_blocks, so.x), (out.y_f_dyn, so.y_fdyn), (out.z_g, so.z_g), (out.y_g, so.y_g)):
        assert rel_err(g.cpu().numpy(), w) < TOL[dt]
