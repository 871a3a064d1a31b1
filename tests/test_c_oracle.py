"""The C/OpenMP restatement (CPU baseline) agrees with the NumPy oracle."""
import numpy as np

from oracle import admm_ref as ref
from oracle import c_oracle
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200.problems import synthetic


def _cmp(blocks, dt, tol, iters=(20, 15)):
    qp = oracle_qp(blocks, dtype=dt)
    st = c_oracle.admm_fixed(qp, 0.1, iters[0], iters[1], threads=2)
    cfg = ref.ADMMConfig(max_iter=iters[0], pcg_max_iter=iters[1], check_every=0, adapt_rho_every=0, eps_abs=0,
                         eps_rel=0, pcg_eps=0.0)
    so, _ = ref.admm_solve(qp, ref.initial_state(qp, 0.1), cfg)
    for k, o in (("x", so.x), ("y_fdyn", so.y_fdyn), ("z_g", so.z_g), ("y_g", so.y_g)):
        assert rel_err(st[k], o) < tol, k


def test_c_oracle_matches_numpy_f64():
    _cmp(synthetic.double_integrator(batch=8, N=20), np.float64, 1e-9)
    _cmp(dense_blocks(4, 6, 3, 8, 3, seed=2), np.float64, 1e-9)


def test_c_oracle_matches_numpy_f32():
    _cmp(synthetic.double_integrator(batch=8, N=20), np.float32, 1e-3)


def test_c_oracle_direct_solve_matches_numpy_dense():
    """pcg_iters < 0: block-Cholesky solve of every ADMM linear system (the
    CPU baseline of the direct backend) against the NumPy oracle's dense
    solves."""
    for blocks in (synthetic.double_integrator(batch=6, N=20), dense_blocks(4, 6, 3, 8, 3, seed=2)):
        qp = oracle_qp(blocks, dtype=np.float64)
        st = c_oracle.admm_fixed(qp, 0.1, 25, -1, threads=2)
        cfg = ref.ADMMConfig(max_iter=25, pcg_max_iter=1, check_every=0, adapt_rho_every=0, eps_abs=0, eps_rel=0,
                             pcg_eps=0.0)
        so, _ = ref.admm_solve(qp, ref.initial_state(qp, 0.1), cfg, linsys="dense")
        for k, o in (("x", so.x), ("y_fdyn", so.y_fdyn), ("z_g", so.z_g), ("y_g", so.y_g)):
            assert rel_err(st[k], o) < 1e-9, k
