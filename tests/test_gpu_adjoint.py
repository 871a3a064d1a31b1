"""GPU parity of the adjoint KKT solve vs the dense oracle (a restatement of
turbompc/solvers/backward/backward_kkt_jax.py:10-211)."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, oracle_qp, rel_err
from turbompc_b200 import ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu
TOL = {torch.float64: 1e-6, torch.float32: 1e-3}


def _backward_blocks(nx, nu, N, m, seed, active_frac=0.4):
    b = dense_blocks(4, nx, nu, N, m, seed=seed)
    rng = np.random.default_rng(seed)
    if m:
        sign = rng.choice([-1.0, 0.0, 1.0], size=b["G"].shape[:3], p=[active_frac / 2, 1 - active_frac, active_frac / 2])
        b["G"] = b["G"] * sign[..., None]
        # x0 is fixed by the A0 rows; active rows at t = 0 on top of them would
        # violate LICQ (singular KKT, non-unique multipliers).
        b["G"][:, 0] = 0.0
    return b


@pytest.mark.parametrize("dt", [torch.float64, torch.float32])
@pytest.mark.parametrize("nx,nu,N,m", [(4, 2, 10, 3), (12, 4, 20, 4), (6, 3, 30, 3), (3, 2, 1, 0), (5, 5, 6, 6)])
def test_adjoint_kkt_matches_dense(dt, nx, nu, N, m):
    b = _backward_blocks(nx, nu, N, m, seed=N + m)
    dzo, muo = ref.solve_backward_kkt(oracle_qp(b))
    qd = synthetic.to_qpdata(b, dtype=dt, device="cuda")
    dz, mu, st = ops.adjoint_kkt_solve(qd)
    assert int(st.abs().sum()) == 0
    assert rel_err(dz.cpu().numpy(), dzo) < TOL[dt]
    n_eq = b["A0"].shape[1] + N * nx
    assert rel_err(mu.cpu().numpy()[:, :n_eq], muo[:, :n_eq]) < TOL[dt]
    if m:
        assert rel_err(mu.cpu().numpy()[:, n_eq:], muo[:, n_eq:]) < TOL[dt] * 10
