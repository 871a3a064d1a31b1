"""Gradients through the solve (the custom_vjp path) against central finite
differences, as the reference does (tests/cuda/solvers/test_differentiable.py:
27-140 with turbompc/utils/gradient_finitediff.py; atol/rtol 1e-3), in fp64 on
converged solves."""
import numpy as np
import pytest
import torch

from turbompc_b200.dynamics import LinearDynamics
from turbompc_b200.problems.ocp import OptimalControlProblem
from turbompc_b200.problems.quadrotor import make_quadrotor_problem
from turbompc_b200.solver import TurboMPCSolver

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _double_integrator(batch=3, N=10, umax=0.6):
    dt = 0.1
    I2 = torch.eye(2, dtype=torch.float64)
    Ad = torch.cat([torch.cat([I2, dt * I2], 1), torch.cat([torch.zeros(2, 2, dtype=torch.float64), I2], 1)], 0)
    Bd = torch.cat([0.5 * dt * dt * I2, dt * I2], 0)
    rng = np.random.default_rng(0)
    x0 = torch.tensor(rng.uniform(-2, 2, size=(batch, 4)), device=DEV)
    t = lambda a: torch.as_tensor(a, dtype=torch.float64, device=DEV)
    params = {
        "horizon": N, "discretization_resolution": 1.0, "discretization_scheme": 0, "initial_state": x0,
        "reference_state_trajectory": t(np.zeros(4)), "reference_control_trajectory": t(np.zeros(2)),
        "penalize_control_reference": False,
        "weights_penalization_reference_state_trajectory": t(np.ones(4)),
        "weights_penalization_final_state": t(np.full(4, 9.0)),
        "weights_penalization_control_squared": t(np.full(2, 0.1)),
        "weights_penalization_control_rate": t(np.zeros(2)),
        "state_min_bounds": t(np.full(4, -10.0)), "state_max_bounds": t(np.full(4, 10.0)),
        "control_min_bounds": t(np.full(2, -umax)), "control_max_bounds": t(np.full(2, umax)),
        "dynamics_state_dot_params": {"A": t(Ad - torch.eye(4, dtype=torch.float64)), "B": t(Bd)},
    }
    return OptimalControlProblem(LinearDynamics(4, 2), params), params


SOLVER = {"num_sqp_iteration_max": 1, "tol_convergence": 0.0,
          "admm": {"max_iter": 4000, "check_termination_every": 10, "adapt_rho_every": 50, "eps_abs": 1e-12,
                   "eps_rel": 1e-12, "rho": 0.1, "pcg": {"max_iter": 1, "tol_epsilon": 0.0}}}


def _loss(sol):
    return (sol.states ** 2).sum() + 3.0 * (sol.controls ** 2).sum()


def _fd(f, w, idx, h=1e-6):
    wp, wm = w.clone(), w.clone()
    wp.view(-1)[idx] += h
    wm.view(-1)[idx] -= h
    return (f(wp) - f(wm)) / (2 * h)


@pytest.mark.parametrize("which", ["weights_penalization_reference_state_trajectory",
                                   "weights_penalization_control_squared", "initial_state"])
def test_linear_mpc_gradients_match_finite_differences(which):
    ocp, params = _double_integrator()
    solver = TurboMPCSolver(ocp, SOLVER, forward_backend="b200_direct", use_full_hessian=True)
    guess = solver.initial_guess(params)
    w0 = params[which].clone()

    def run(w):
        with torch.no_grad():
            return _loss(solver.solve(guess, params, {which: w})).item()

    w = w0.clone().requires_grad_(True)
    sol = solver.solve(guess, params, {which: w})
    assert (sol.kkt_state.ineq_active_lower_idx | sol.kkt_state.ineq_active_upper_idx).any()
    g, = torch.autograd.grad(_loss(sol), w)
    for idx in range(min(w0.numel(), 6)):
        fd = _fd(run, w0, idx)
        gv = g.view(-1)[idx].item()
        assert abs(gv - fd) <= 1e-3 + 1e-3 * abs(fd), (idx, gv, fd)


def test_quadrotor_gradient_wrt_weights_fp64():
    """Nonlinear RK4 quadrotor, 5 SQP iterations, exact-Hessian backward."""
    ocp, params = make_quadrotor_problem(2, N=10, dtype=torch.float64, device=DEV)
    sp = {"num_sqp_iteration_max": 8, "tol_convergence": 0.0,
          "admm": {"max_iter": 2000, "check_termination_every": 10, "adapt_rho_every": 50, "eps_abs": 1e-11,
                   "eps_rel": 1e-11, "pcg": {"max_iter": 1, "tol_epsilon": 0.0}}}
    solver = TurboMPCSolver(ocp, sp, forward_backend="b200_direct", use_full_hessian=True)
    guess = solver.initial_guess(params)
    key = "weights_penalization_reference_state_trajectory"
    w0 = params[key].clone()

    def run(w):
        with torch.no_grad():
            return _loss(solver.solve(guess, params, {key: w})).item()

    w = w0.clone().requires_grad_(True)
    g, = torch.autograd.grad(_loss(solver.solve(guess, params, {key: w})), w)
    for idx in (0, 3, 6, 9):
        fd = _fd(run, w0, idx, h=1e-5)
        gv = g.view(-1)[idx].item()
        assert abs(gv - fd) <= 1e-3 + 1e-2 * abs(fd), (idx, gv, fd)
