"""GPU: the CUDA linearisation of the built-in dynamics (tmpc_linearize_dynamics_*)
against the PyTorch forward-mode path of the same integrator
(OptimalControlProblem.get_dynamics_linearized_matrices), and the SQP solve
with it against the solve on the PyTorch path.  Tolerances (relative,
||a-b||_inf / ||b||_inf): 1e-5 fp32 / 1e-12 fp64 for the rows, 1e-3 fp32 for
solver outputs."""
import numpy as np
import pytest
import torch

from tests.helpers import rel_err
from turbompc_b200 import ops
from turbompc_b200.dynamics import ClohessyWiltshireDynamics, Quadrotor12Dynamics
from turbompc_b200.problems.quadrotor import make_quadrotor_problem
from turbompc_b200.solver import TurboMPCSolver

pytestmark = pytest.mark.gpu
TOL = {torch.float32: 1e-5, torch.float64: 1e-12}


def _torch_rows(prog, states, controls, params):
    _, _, As, Bs, Cs = prog.get_dynamics_linearized_matrices(states, controls, params)
    return torch.cat([As, Bs], -1), Cs[:, 1:]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("scheme", [0, 1, 2])
def test_quadrotor_rows_match_torch_path(dtype, scheme):
    prog, params = make_quadrotor_problem(64, N=20, seed=3, dtype=dtype, device="cuda")
    params = dict(params, discretization_scheme=scheme)
    prog._scheme = type(prog._scheme)(scheme)
    g = torch.Generator(device="cuda").manual_seed(0)
    states = 0.4 * torch.randn(64, 21, 12, generator=g, device="cuda", dtype=dtype)
    controls = 2.0 + torch.randn(64, 21, 4, generator=g, device="cuda", dtype=dtype)
    Am, c = ops.linearize_dynamics(1, Quadrotor12Dynamics().cuda_model()[1], scheme, 0.02, states, controls)
    Am_t, c_t = _torch_rows(prog, states, controls, params)
    assert rel_err(Am.cpu().numpy(), Am_t.cpu().numpy()) < TOL[dtype]
    assert rel_err(c.cpu().numpy(), c_t.cpu().numpy()) < TOL[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_clohessy_wiltshire_rows_match_torch_path(dtype):
    dyn = ClohessyWiltshireDynamics()
    from turbompc_b200.dynamics.integrators import predict_next_state
    Nb, T = 32, 11
    g = torch.Generator(device="cuda").manual_seed(1)
    xs = 100.0 * torch.randn(Nb, T, 6, generator=g, device="cuda", dtype=dtype)
    us = 0.01 * torch.randn(Nb, T, 3, generator=g, device="cuda", dtype=dtype)
    Am, c = ops.linearize_dynamics(2, [0.0011], 2, 10.0, xs, us)
    xu = torch.cat([xs[:, :-1], us[:, :-1]], -1)
    f = lambda z: predict_next_state(dyn, 10.0, 2, {}, z[..., :6], z[..., 6:])
    J = torch.func.vmap(torch.func.jacfwd(f))(xu.reshape(-1, 9)).reshape(Nb, T - 1, 6, 9).to(dtype)
    Fz = f(xu)
    c_t = -Fz + torch.einsum("btij,btj->bti", J, xu)
    assert rel_err(Am.cpu().numpy(), J.cpu().numpy()) < TOL[dtype]
    # c = -F + J z is a cancellation (exactly 0 for this linear model): compare
    # against the scale of F.
    scale = Fz.abs().max().item()
    assert (c - c_t).abs().max().item() < 10 * TOL[dtype] * scale


def test_rows_for_empty_batch():
    z = torch.zeros(0, 5, 12, device="cuda")
    Am, c = ops.linearize_dynamics(1, Quadrotor12Dynamics().cuda_model()[1], 2, 0.02, z, torch.zeros(0, 5, 4,
                                                                                                        device="cuda"))
    assert Am.shape == (0, 4, 12, 16) and c.shape == (0, 4, 12)


def test_quadrotor_sqp_solve_matches_torch_linearisation(monkeypatch):
    """The full SQP solve (5 x 30 x 30, fp32) with the CUDA rows and reused
    constant blocks equals the solve on the PyTorch linearisation path."""
    prog, params = make_quadrotor_problem(128, N=50, seed=7, dtype=torch.float32, device="cuda")
    cfg = {"num_sqp_iteration_max": 5, "tol_convergence": 0.0,
           "admm": {"max_iter": 30, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": 0.0,
                    "eps_rel": 0.0, "pcg": {"max_iter": 30, "tol_epsilon": 0.0}}}
    s = TurboMPCSolver(prog, cfg)
    a = s.solve(s.initial_guess(params), params)
    monkeypatch.setattr(Quadrotor12Dynamics, "cuda_model", lambda self, p=None: None)
    s2 = TurboMPCSolver(prog, cfg)
    b = s2.solve(s2.initial_guess(params), params)
    assert rel_err(a.controls.cpu().numpy(), b.controls.cpu().numpy()) < 1e-3
    assert rel_err(a.states.cpu().numpy(), b.states.cpu().numpy()) < 1e-3


def test_qp_reuse_equals_full_build():
    prog, params = make_quadrotor_problem(16, N=30, seed=2, dtype=torch.float64, device="cuda")
    s = TurboMPCSolver(prog, {"num_sqp_iteration_max": 2})
    g = s.initial_guess(params)
    q0 = s._build_qp_data(g.states, g.controls, params)
    st = g.states + 0.01
    full = s._build_qp_data(st, g.controls, params)
    reuse = s._build_qp_data(st, g.controls, params, prev=q0)
    for f, r in zip(full.tensors().values(), reuse.tensors().values()):
        assert torch.equal(f, r)


@pytest.mark.parametrize("slack", [False, True])
@pytest.mark.parametrize("nx,nu,dtype", [(6, 3, torch.float64), (12, 4, torch.float64), (12, 4, torch.float32),
                                         (6, 2, torch.float32), (5, 3, torch.float32)])
def test_first_order_error_kernel_matches_torch(slack, nx, nu, dtype):
    """tmpc_first_order_error_* against the PyTorch form of the SQP first-order
    check (dense QP blocks incl. E coupling, n0 rows, slack variables) in fp64
    and fp32 at block sizes 8, 9 and 16 (the fp32 results against the fp64
    PyTorch form)."""
    from tests.helpers import dense_blocks
    from turbompc_b200.problems import synthetic
    Nb, n = 5, nx + nu
    b = dense_blocks(Nb, nx, nu, 9, 4, seed=4)
    sw = np.full(Nb, 3.0) if slack else None
    qd = synthetic.to_qpdata(b, dtype=dtype, device="cuda", slack_weight=sw, use_slack=slack)
    g = torch.Generator(device="cuda").manual_seed(5)
    r = lambda *s: torch.randn(*s, generator=g, device="cuda", dtype=dtype)
    st = ops.ADMMState(r(Nb, 10, n), r(Nb, 10, 4), r(Nb, nx), r(Nb, 9, nx), r(Nb, 10, 4), r(Nb, 10, 4), r(Nb).abs())
    states, controls, slacks = r(Nb, 10, nx), r(Nb, 10, nu), r(Nb, 10, 4)
    s = TurboMPCSolver.__new__(TurboMPCSolver)
    a = s._first_order_error(qd, states, controls, slacks, st)
    d64 = lambda t: t.double()
    qd64 = qd.map(d64) if dtype != torch.float64 else qd
    c = s._first_order_error_torch(qd64, d64(states), d64(controls), d64(slacks), ops.ADMMState(*(d64(t) for t in st)))
    tol = 1e-12 if dtype == torch.float64 else 1e-5
    for x, y in zip(a, c):
        assert rel_err(x.double().cpu().numpy(), y.cpu().numpy()) < tol
