"""tmpc_admm_solve_fixed_scratch_f64: the fused ADMM entry point for callers
that cannot allocate device memory (a runtime that owns every allocation, a
handler restricted to the buffers it is handed, an embedded controller with a
fixed memory plan).  Its scratch is a fixed 64 MiB device buffer inside the
library.  This file is collected last on purpose: it runs after every other
test in a full run, and must also pass alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

from tests.helpers import dense_blocks, rel_err
from turbompc_b200 import _ffi, ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu

CFG = dict(max_iter=15, pcg_max_iter=30, check_every=0, adapt_rho_every=0, eps_abs=0.0, eps_rel=0.0, pcg_eps=0.0,
           rho_f_factor=1000.0, alpha=1.6, sigma=1e-6)


def _call_fixed(qd, s0, cfg):
    lib = _ffi.load()
    out = ops.empty_state_like(s0)
    it = torch.empty(qd.Nb, dtype=torch.int32, device=qd.device)
    st = torch.empty(qd.Nb, dtype=torch.int32, device=qd.device)
    d, q, c = ops.dims_of(qd), ops._qp_c(qd), cfg.to_c()
    si, so = ops._state_c(s0, qd.dtype, qd.device), ops._state_c(out, qd.dtype, qd.device)
    rc = lib.tmpc_admm_solve_fixed_scratch_f64(C.byref(d), C.byref(q), C.byref(si), C.byref(so), None, C.byref(c),
                                               None, it.data_ptr(), st.data_ptr(),
                                               torch.cuda.current_stream().cuda_stream)
    return rc, out, it, st


def test_fixed_scratch_matches_workspace_entry_point_twice():
    # n = 26 -> block size 32; in fp64 these operators exceed one CTA's shared
    # memory, so both entry points run from scratch in HBM.
    b = dense_blocks(16, 20, 6, 8, 6, seed=5)
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    assert ops.admm_workspace_bytes(qd, ops.AdmmConfig(**CFG)) > 0
    cfg = ops.AdmmConfig(**CFG)
    s0 = ops.admm_initial_state(qd, 0.1)
    want, want_it, _ = ops.admm_solve(qd, s0, cfg)
    for _ in range(2):  # the buffer keeps the previous call's contents; results must not depend on them
        rc, got, it, st = _call_fixed(qd, s0, cfg)
        torch.cuda.synchronize()
        assert rc == 0, _ffi.load().tmpc_error_string(rc)
        assert int(st.abs().sum()) == 0
        assert (it.cpu().numpy() == want_it.cpu().numpy()).all()
        for g, w in zip(got, want):
            assert rel_err(g.cpu().numpy(), w.cpu().numpy()) < 1e-6


def test_fixed_scratch_direct_linsys_matches_workspace_entry_point_twice():
    # The direct (block-Cholesky) solve keeps its whole factor in the scratch
    # buffer; compared with the same solve given a caller workspace.
    b = dense_blocks(16, 20, 6, 8, 6, seed=7)
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    cfg = ops.AdmmConfig(**CFG, linsys=_ffi.LINSYS_DIRECT)
    assert ops.admm_workspace_bytes(qd, cfg) > 0
    s0 = ops.admm_initial_state(qd, 0.1)
    want, want_it, _ = ops.admm_solve(qd, s0, cfg)
    for _ in range(2):
        rc, got, it, st = _call_fixed(qd, s0, cfg)
        torch.cuda.synchronize()
        assert rc == 0, _ffi.load().tmpc_error_string(rc)
        assert int(st.abs().sum()) == 0
        assert (it.cpu().numpy() == want_it.cpu().numpy()).all()
        for g, w in zip(got, want):
            assert rel_err(g.cpu().numpy(), w.cpu().numpy()) < 1e-6


def test_fixed_scratch_rejects_batches_beyond_its_buffer():
    b = dense_blocks(400, 20, 6, 8, 6, seed=6)  # ~400 x 207 KB of operators > 64 MiB
    qd = synthetic.to_qpdata(b, dtype=torch.float64, device="cuda")
    rc, *_ = _call_fixed(qd, ops.admm_initial_state(qd, 0.1), ops.AdmmConfig(**CFG))
    assert rc == -6
    assert b"fixed device buffer" in _ffi.load().tmpc_error_string(rc)
