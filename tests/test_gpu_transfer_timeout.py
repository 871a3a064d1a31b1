"""Failure detection without a GPU fault: the bounded wait on the TMA bulk
copies that stage a problem's operators into shared memory.  With the poll
limit set to 0 (tmpc_set_transfer_poll_limit) every wait reports a time-out
on copies that do complete; the kernel must drain them, mark the problem
(iters_out = 0xffffffff) and return, leaving the context usable: the next
launch with the default limit solves the same systems correctly."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import rel_err
from turbompc_b200 import _ffi, ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu


def test_transfer_timeout_sets_status_and_context_stays_usable():
    b = synthetic.random_lti(8, 6, 3, 16, seed=9)
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    o, st = ops.schur_assemble_packed(qd, 0.1, 1e-6, 100.0)
    rng = np.random.default_rng(2)
    rhs = torch.as_tensor(rng.normal(size=(8, 17, 9)), device="cuda")
    x0 = torch.zeros_like(rhs)
    lib = _ffi.load()
    prev = lib.tmpc_set_transfer_poll_limit(0)
    try:
        _, it = ops.pcg_solve_packed(o, ops.dims_of(qd), rhs, x0, 0.0, 20)
        torch.cuda.synchronize()
    finally:
        assert lib.tmpc_set_transfer_poll_limit(prev) == 0
    assert (it.cpu().numpy() == 0xFFFFFFFF).all()
    x, it2 = ops.pcg_solve_packed(o, ops.dims_of(qd), rhs, x0, 0.0, 20)
    q = ref.QP(**{k: np.asarray(v) for k, v in b.items()})
    S, P = ref.compute_S_Phiinv(q, np.full(8, 10.0), 1e-6, np.full(8, 0.1))
    xr, itr = ref.pcg(S, P, rhs.cpu().numpy(), x0.cpu().numpy(), 20, 0.0)
    assert (it2.cpu().numpy() == itr).all()  # the 1e-12 floor may stop some problems early
    assert rel_err(x.cpu().numpy(), xr) < 1e-6
