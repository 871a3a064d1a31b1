"""CPU checks of the NumPy oracle against the reference's own known-answer
tests (restated: the JAX reference cannot run here) and dense solves."""
import numpy as np
import pytest

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200.problems import synthetic


@pytest.mark.parametrize("T", [2, 5])
@pytest.mark.parametrize("nx", [1, 5])
@pytest.mark.parametrize("nu", [1, 5])
def test_compute_S_Phiinv_identity_dynamics(T, nx, nu):
    """tests/python/solvers/test_solver_pcg.py:92-110 restated: identity
    dynamics, unit weights -> finite S / Phiinv of shape (T+1, n, 3n)."""
    n = nx + nu
    B = 1
    blocks = dict(
        D=np.broadcast_to(np.eye(n), (B, T + 1, n, n)).copy(), E=np.zeros((B, T, n, n)),
        q=np.zeros((B, T + 1, n)), A0=np.concatenate([np.eye(nx), np.zeros((nx, nu))], 1)[None],
        Am=np.concatenate([np.eye(nx), np.ones((nx, nu))], 1)[None, None].repeat(T, 1),
        Ap=np.concatenate([-np.eye(nx), np.zeros((nx, nu))], 1)[None, None].repeat(T, 1),
        c0=np.ones((B, nx)), c=np.ones((B, T, nx)), G=np.zeros((B, T + 1, 0, n)),
        l=np.zeros((B, T + 1, 0)), u=np.zeros((B, T + 1, 0)))
    S, P = ref.compute_S_Phiinv(oracle_qp(blocks), 1.0, 1e-6, 0.1)
    assert S.shape == (B, T + 1, n, 3 * n) and P.shape == S.shape
    assert np.isfinite(S).all() and np.isfinite(P).all()


def test_compute_gamma_matches_manual():
    """tests/cuda/backends/test_admm_math_cuda_vs_python.py:135-158 restated:
    gamma = sigma x - q + C^T(rho_f c - y_f) + G^T(rho z - y_g) with explicit
    dense C and G, to 1e-12."""
    b = dense_blocks(3, 4, 2, 6, 3, seed=1)
    qp = oracle_qp(b)
    d = qp.dims
    rng = np.random.default_rng(2)
    B, T, N, n, nx, n0, m = (d[k] for k in ("B", "T", "N", "n", "nx", "n0", "m"))
    x = rng.normal(size=(B, T, n))
    z = rng.normal(size=(B, T, m))
    yg = rng.normal(size=(B, T, m))
    y0 = rng.normal(size=(B, n0))
    yd = rng.normal(size=(B, N, nx))
    rf, ri, sig = 3.0, 0.7, 1e-3
    g = ref.compute_gamma(qp, x, z, yg, y0, yd, np.full(B, rf), np.full(B, ri), sig)
    K, _ = ref.assemble_backward_kkt(qp)
    nt = T * n
    C = K[:, nt:nt + n0 + N * nx, :nt]
    Gd = K[:, nt + n0 + N * nx:, :nt]
    c = np.concatenate([qp.c0, qp.c.reshape(B, -1)], 1)
    y = np.concatenate([y0, yd.reshape(B, -1)], 1)
    man = (sig * x.reshape(B, -1) - qp.q.reshape(B, -1) + np.einsum("bij,bi->bj", C, rf * c - y)
           + np.einsum("bij,bi->bj", Gd, ri * z.reshape(B, -1) - yg.reshape(B, -1)))
    assert rel_err(g.reshape(B, -1), man) < 1e-12


def test_schur_is_the_admm_system_matrix():
    """S = P + sigma I + rho_f C^T C + rho G^T G (the x-update normal matrix of
    admm.py) and Phiinv is symmetric."""
    b = dense_blocks(2, 3, 2, 5, 2, seed=3)
    qp = oracle_qp(b)
    d = qp.dims
    B, T, n = d["B"], d["T"], d["n"]
    S, P = ref.compute_S_Phiinv(qp, np.full(B, 5.0), 1e-4, np.full(B, 0.3))
    K, _ = ref.assemble_backward_kkt(qp)
    nt = T * n
    Pd = K[:, :nt, :nt]
    meq = d["n0"] + d["N"] * d["nx"]
    C = K[:, nt:nt + meq, :nt]
    Gd = K[:, nt + meq:, :nt]
    want = Pd + 1e-4 * np.eye(nt) + 5.0 * np.swapaxes(C, 1, 2) @ C + 0.3 * np.swapaxes(Gd, 1, 2) @ Gd
    assert rel_err(ref.block_tridi_to_dense(S), want) < 1e-12
    Pdn = ref.block_tridi_to_dense(P)
    assert rel_err(Pdn, np.swapaxes(Pdn, 1, 2)) < 1e-10


@pytest.mark.parametrize("semantics", ["cuda", "jax"])
def test_pcg_matches_dense_solve(semantics):
    """tests/cuda/backends/test_pcg_ffi_backend.py:29-51: PCG vs dense <= 5e-6."""
    b = synthetic.random_lti(4, 6, 3, 16, seed=4)
    qp = oracle_qp(b)
    S, P = ref.compute_S_Phiinv(qp, np.full(4, 100.0), 1e-6, np.full(4, 0.1))
    rng = np.random.default_rng(5)
    rhs = rng.normal(size=(4, 17, 9))
    x, it = ref.pcg(S, P, rhs, np.zeros_like(rhs), 500, 1e-24, semantics=semantics)
    xd = ref.solve_block_tridi_dense(S, rhs)
    assert rel_err(x, xd) < 5e-6
    assert (it > 0).all()


def test_pcg_zero_rhs_shortcut():
    """pcg_primal.py:158-175: r = 0 at the warm start -> zero iterations, no NaN."""
    b = synthetic.random_lti(2, 4, 2, 5, seed=6)
    qp = oracle_qp(b)
    S, P = ref.compute_S_Phiinv(qp, np.full(2, 10.0), 1e-6, np.full(2, 0.1))
    z = np.zeros((2, 6, 6))
    for sem in ("cuda", "jax"):
        x, it = ref.pcg(S, P, z, z, 20, 0.0, semantics=sem)
        assert (it == 0).all() and np.all(x == 0)


def test_admm_dense_and_pcg_agree_and_converge():
    """ADMM with PCG and with an exact Schur solve converge to the same point,
    which satisfies the QP's KKT conditions."""
    b = synthetic.double_integrator(batch=4, N=10)
    qp = oracle_qp(b)
    cfg = ref.ADMMConfig(max_iter=400, pcg_max_iter=200, check_every=0, adapt_rho_every=0, pcg_eps=1e-28,
                         rho_f_factor=1000.0)
    st0 = ref.initial_state(qp, 0.1)
    s1, _ = ref.admm_solve(qp, st0, cfg, linsys="pcg")
    s2, _ = ref.admm_solve(qp, st0, cfg, linsys="dense")
    assert rel_err(s1.x, s2.x) < 1e-6
    pr, du, *_ = ref.residuals(qp, s2)
    assert pr.max() < 1e-6 and du.max() < 1e-5


def test_backward_kkt_solution_satisfies_system():
    b = dense_blocks(2, 3, 2, 4, 2, seed=7)
    b["G"][:, ::2] = 0.0  # inactive rows -> regularised
    qp = oracle_qp(b)
    K, rhs = ref.assemble_backward_kkt(qp)
    dz, mu = ref.solve_backward_kkt(qp)
    sol = np.concatenate([dz.reshape(2, -1), mu], 1)
    assert rel_err(np.einsum("bij,bj->bi", K, sol), rhs) < 1e-10
