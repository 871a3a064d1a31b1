"""The direct (block-Cholesky) solve on the batch-interleaved layout
(tmpc_riccati_factor_il_* / tmpc_riccati_solve_il_*) against the dense oracle
solve (the reference pins its cuDSS direct solve against dense solves,
tests/cuda/backends/test_cudss_ffi_backend.py:19-40) and against the
reference-layout factor; layout conversion round trips; ragged batches (not a
multiple of 32), an empty batch, the smallest horizon and a singular block.
Tolerances: 1e-9 relative in fp64; in fp32 1e-3 against the fp64 dense solve
and 1e-4 against the reference-layout fp32 factor."""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import dense_blocks, rel_err
from turbompc_b200 import _ffi, ops
from turbompc_b200.problems import synthetic

pytestmark = pytest.mark.gpu


def _schur(nb, nx, nu, N, dtype, seed):
    b = dense_blocks(nb, nx, nu, N, 2, seed=seed)
    qd = synthetic.to_qpdata(b, dtype=dtype, device="cuda")
    S, _, st = ops.schur_assemble(qd, 0.1, 1e-6, 100.0)
    assert int(st.abs().sum()) == 0
    return S


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("nb,nx,nu,N", [(37, 6, 3, 16), (64, 3, 1, 1), (33, 12, 4, 10), (5, 8, 4, 7), (1, 2, 2, 3)])
def test_interleaved_factor_solve_matches_dense_oracle(dtype, nb, nx, nu, N):
    n = nx + nu
    if dtype == torch.float64 and n > 12:
        pytest.skip("fp64 interleaved instances cover n <= 12")
    S = _schur(nb, nx, nu, N, dtype, seed=nb + n)
    T = N + 1
    g = torch.Generator(device="cuda").manual_seed(3)
    rhs = torch.randn(nb, T, n, generator=g, device="cuda", dtype=dtype)
    d = _ffi.TmpcDims(nb, T, n, n, 0, 0)
    ops_il = ops.schur_interleave(S)
    fac, st = ops.riccati_factor_il(ops_il, d)
    x = ops.deinterleave(ops.riccati_solve_il(fac, d, ops.interleave(rhs)), (nb, T, n))
    torch.cuda.synchronize()
    assert int(st.abs().sum()) == 0
    want = ref.solve_block_tridi_dense(S.double().cpu().numpy(), rhs.double().cpu().numpy())
    assert rel_err(x.cpu().numpy(), want) < (1e-9 if dtype == torch.float64 else 1e-3)
    # the reference-layout factor of the same S
    f2, _ = ops.riccati_factor(S)
    x2 = ops.riccati_solve(f2, rhs)
    assert rel_err(x.cpu().numpy(), x2.cpu().numpy()) < (1e-11 if dtype == torch.float64 else 1e-4)


def test_interleave_round_trip_and_index_formula():
    nb, E = 45, 37
    x = torch.randn(nb, E, dtype=torch.float64, device="cuda")
    il = ops.interleave(x)
    assert il.numel() == ops.interleaved_numel(nb, E) == 64 * E
    xi = il.cpu().numpy()
    xs = x.cpu().numpy()
    for b in (0, 31, 32, 44):
        for e in (0, 5, 36):
            assert xi[((b // 32) * E + e) * 32 + b % 32] == xs[b, e]
    back = ops.deinterleave(il, (nb, E))
    assert torch.equal(back, x)


def test_schur_interleave_holds_theta_lower_and_phi():
    nb, nx, nu, N = 3, 3, 2, 4
    n, T = nx + nu, N + 1
    S = _schur(nb, nx, nu, N, torch.float64, seed=1)
    il = ops.schur_interleave(S).cpu().numpy()
    Sn = S.cpu().numpy()
    E = T * n * (n + 1) // 2 + N * n * n
    at = lambda b, e: il[((b // 32) * E + e) * 32 + b % 32]
    tri = n * (n + 1) // 2
    for b in range(nb):
        for t in (0, N):
            for i in range(n):
                for j in range(i + 1):
                    assert at(b, t * tri + i * (i + 1) // 2 + j) == Sn[b, t, i, n + j]
        for t in (0, N - 1):
            for i in range(n):
                for k in range(n):
                    assert at(b, T * tri + (t * n + i) * n + k) == Sn[b, t + 1, i, k]


def test_interleaved_singular_block_sets_status_and_others_solve():
    nb, nx, nu, N = 40, 4, 2, 6
    S = _schur(nb, nx, nu, N, torch.float64, seed=2)
    S[7, 3, :, 6:12] = -torch.eye(6, dtype=torch.float64, device="cuda")  # Theta_3 of problem 7 negative definite
    d = _ffi.TmpcDims(nb, N + 1, 6, 6, 0, 0)
    fac, st = ops.riccati_factor_il(ops.schur_interleave(S), d)
    s = st.cpu().numpy()
    assert s[7] == 1  # TMPC_STATUS_SINGULAR_BLOCK
    assert (np.delete(s, 7) == 0).all()


def test_interleaved_empty_batch_and_unsupported_sizes():
    lib = _ffi.load()
    d = _ffi.TmpcDims(0, 5, 6, 6, 0, 0)
    assert lib.tmpc_riccati_factor_il_f32(d, None, None, None, None) == 0
    d = _ffi.TmpcDims(4, 5, 13, 13, 0, 0)
    assert lib.tmpc_riccati_factor_il_f64(d, 1, 1, None, None) == -3  # fp64 instances stop at n = 12
    d = _ffi.TmpcDims(4, 5, 17, 17, 0, 0)
    assert lib.tmpc_riccati_factor_il_f32(d, 1, 1, None, None) == -3


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("nb,nx,nu,N", [(70, 6, 3, 12), (33, 12, 4, 9)])
def test_interleaved_staged_and_global_memory_kernels_agree(dtype, nb, nx, nu, N):
    """16-byte aligned arrays run the kernels that stage each stage's blocks in
    shared memory with cp.async; arrays offset by one element (not 16-byte
    aligned) run the kernels that read global memory directly.  Same
    arithmetic in the same order: the results agree to rounding."""
    n = nx + nu
    if dtype == torch.float64 and n > 12:
        pytest.skip("fp64 interleaved instances cover n <= 12")
    S = _schur(nb, nx, nu, N, dtype, seed=7)
    T = N + 1
    d = _ffi.TmpcDims(nb, T, n, n, 0, 0)
    g = torch.Generator(device="cuda").manual_seed(5)
    rhs = torch.randn(nb, T, n, generator=g, device="cuda", dtype=dtype)
    ops_il = ops.schur_interleave(S)
    rhs_il = ops.interleave(rhs)
    fac, st = ops.riccati_factor_il(ops_il, d)
    x = ops.riccati_solve_il(fac, d, rhs_il)

    def shifted(t):  # same values at an address 1 element past a 16-byte boundary
        buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
        v = buf[1:]
        v.copy_(t.reshape(-1))
        assert v.data_ptr() % 16 != 0
        return v

    ops_u, rhs_u = shifted(ops_il), shifted(rhs_il)
    fac_u, x_u = shifted(torch.zeros_like(fac)), shifted(torch.zeros_like(x))
    _, st_u = ops.riccati_factor_il(ops_u, d, factor=fac_u)
    ops.riccati_solve_il(fac_u, d, rhs_u, out=x_u)
    torch.cuda.synchronize()
    assert int(st.abs().sum()) == 0 and int(st_u.abs().sum()) == 0
    tol = 1e-12 if dtype == torch.float64 else 1e-6
    assert rel_err(fac_u.cpu().numpy(), fac.reshape(-1).cpu().numpy()) < tol
    # the solution slots of the padding problems (past nb) are never written
    xa = ops.deinterleave(x, (nb, T, n)).cpu().numpy()
    xb = ops.deinterleave(x_u.clone(), (nb, T, n)).cpu().numpy()
    assert rel_err(xb, xa) < tol
