"""The CUDA producers of the obstacle rows (tmpc_obstacle_rows_*) and of the
learned stage cost's quadratisation (tmpc_mlp_cost_blocks_*) against their
PyTorch forms, which tests/test_sqp_oracle.py pins to the oracle's autodiff QP
(fp64 1e-12, fp32 1e-5 relative); the whole solves of configurations 4 and 5
in tests/test_gpu_sqp_oracle.py run these kernels too."""
import pytest
import torch

from tests.helpers import rel_err
from turbompc_b200 import ops

pytestmark = pytest.mark.gpu
TOL = {torch.float64: 1e-12, torch.float32: 1e-5}


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_obstacle_rows_kernel_matches_torch(dtype):
    from turbompc_b200.problems.quadrotor import make_obstacle_problem
    prog, p = make_obstacle_problem(37, N=9, n_obstacles=8, seed=3, dtype=dtype, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(2)
    X = torch.randn(37, 10, 12, generator=g, device="cuda", dtype=dtype)
    U = torch.rand(37, 10, 4, generator=g, device="cuda", dtype=dtype)
    c, r = p["obstacles_centers"], p["obstacles_radii"]
    G, lo, hi = ops.obstacle_rows(X, c, r, 3, 16)
    G2, lo2, hi2 = prog._obstacle_rows_torch(X.cpu(), U.cpu(), c.cpu(), r.cpu(), 3)
    assert rel_err(G.cpu().numpy(), G2.numpy()) < TOL[dtype]
    assert rel_err(hi.cpu().numpy(), hi2.numpy()) < TOL[dtype]
    assert rel_err(lo.cpu().numpy(), lo2.numpy()) < TOL[dtype]
    # scaled rows
    Gs, los, his = ops.obstacle_rows(X, c, r, 3, 16, row_scale=0.25)
    assert rel_err(Gs.cpu().numpy(), 0.25 * G2.numpy()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
@pytest.mark.parametrize("hidden", [16, 64])
def test_mlp_cost_blocks_kernel_matches_torch(dtype, hidden):
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    prog, p = make_learned_cost_problem(21, N=12, hidden=hidden, seed=4, dtype=dtype, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(5)
    X = torch.randn(21, 13, 6, generator=gen, device="cuda", dtype=dtype)
    U = 0.1 * torch.randn(21, 13, 3, generator=gen, device="cuda", dtype=dtype)
    D, E, q = prog.get_cost_linearized_blocks(X, U, p)  # CUDA kernel path
    pc = {k: (v.cpu() if isinstance(v, torch.Tensor) else v) for k, v in p.items()}
    pc["dynamics_state_dot_params"] = {k: v.cpu() for k, v in p["dynamics_state_dot_params"].items()}
    D2, E2, q2 = prog.get_cost_linearized_blocks(X.cpu(), U.cpu(), pc)  # PyTorch path
    assert rel_err(D.cpu().numpy(), D2.numpy()) < TOL[dtype]
    assert rel_err(q.cpu().numpy(), q2.numpy()) < TOL[dtype] * 10
    assert torch.equal(E.cpu(), E2)


def test_repeated_learned_cost_solves_are_identical():
    """From the second SQP iteration on the linearisation points are views of
    the ADMM iterate; the producer wrappers must keep their contiguous copies
    alive until the launch (a freed copy's block was handed to the next
    temporary and overwritten before the kernel read it)."""
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    from turbompc_b200.solver import TurboMPCSolver
    prog, p = make_learned_cost_problem(3, N=10, hidden=16, seed=2, dtype=torch.float64, device="cuda")
    sp = {"num_sqp_iteration_max": 3, "tol_convergence": 0.0,
          "admm": {"max_iter": 30, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": 0.0,
                   "eps_rel": 0.0, "pcg": {"max_iter": 10, "tol_epsilon": 0.0}}}
    s = TurboMPCSolver(prog, sp)
    g = s.initial_guess(p)
    first = s.solve(g, p)
    for _ in range(3):
        again = s.solve(g, p)
        assert torch.equal(again.controls, first.controls) and torch.equal(again.states, first.states)


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_ineq_rows_kernel_matches_torch(dtype):
    """tmpc_ineq_rows_*: G z, G z + slack and clamp(G z, l, u) against the
    PyTorch products (the solver's active-set g and ADMM's initial z_g)."""
    gen = torch.Generator(device="cuda").manual_seed(7)
    Nb, T, m, n = 45, 11, 5, 13
    G = torch.randn(Nb, T, m, n, generator=gen, device="cuda", dtype=dtype)
    z = torch.randn(Nb, T, n, generator=gen, device="cuda", dtype=dtype)
    s = torch.randn(Nb, T, m, generator=gen, device="cuda", dtype=dtype)
    lo = -torch.rand(Nb, T, m, generator=gen, device="cuda", dtype=dtype)
    hi = torch.rand(Nb, T, m, generator=gen, device="cuda", dtype=dtype)
    ref = torch.einsum("btki,bti->btk", G.double(), z.double())
    assert rel_err(ops.ineq_rows(G, z).cpu().numpy(), ref.cpu().numpy()) < TOL[dtype]
    assert rel_err(ops.ineq_rows(G, z, s).cpu().numpy(), (ref + s.double()).cpu().numpy()) < TOL[dtype]
    cl = torch.minimum(torch.maximum(ref, lo.double()), hi.double())
    assert rel_err(ops.ineq_rows(G, z, lo=lo, hi=hi).cpu().numpy(), cl.cpu().numpy()) < TOL[dtype]
