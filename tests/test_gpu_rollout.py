"""Closed-loop rollout harness (turbompc/utils/timing.py:69-122) on the GPU:
batched MPC steps with warm start, and the gradient of the rollout cost
with respect to a cost weight against central finite differences (the
reference's gradient-accuracy check; cold-start rollout, fp64, converged
solves; atol 1e-3, rtol 1e-2)."""
import numpy as np
import pytest
import torch

from tests.test_gpu_grad import SOLVER, _double_integrator
from turbompc_b200.problems.quadrotor import make_quadrotor_problem
from turbompc_b200.rollout import closed_loop_rollout
from turbompc_b200.solver import TurboMPCSolver

pytestmark = pytest.mark.gpu


def test_quadrotor_closed_loop_rollout_tracks_setpoint():
    prog, params = make_quadrotor_problem(64, N=20, seed=11, dtype=torch.float32, device="cuda")
    cfg = {"num_sqp_iteration_max": 3, "tol_convergence": 0.0,
           "admm": {"max_iter": 30, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": 0.0,
                    "eps_rel": 0.0, "pcg": {"max_iter": 30, "tol_epsilon": 0.0}}}
    s = TurboMPCSolver(prog, cfg)
    x0 = params["initial_state"]
    with torch.no_grad():
        cost, iters, xs = closed_loop_rollout(s, params, x0, 25, warm_start=True)
    target = params["reference_state_trajectory"][:, 0, :3]
    e0 = (xs[0][:, :3] - target).norm(dim=-1)
    e1 = (xs[-1][:, :3] - target).norm(dim=-1)
    assert torch.isfinite(cost).all()
    assert iters.shape[:2] == (25, 64)
    assert (e1 < e0).float().mean() > 0.9, "the closed loop must move (almost) every vehicle towards its set-point"


def test_rollout_gradient_matches_finite_differences():
    ocp, params = _double_integrator(batch=3, N=10)
    solver = TurboMPCSolver(ocp, SOLVER, forward_backend="b200_direct", use_full_hessian=True)
    key = "weights_penalization_control_squared"
    w0 = params[key].clone()
    x0 = params["initial_state"]

    def total(w):
        c, _, _ = closed_loop_rollout(solver, params, x0, 3, weights={key: w}, warm_start=False)
        return c.sum()

    w = w0.clone().requires_grad_(True)
    g, = torch.autograd.grad(total(w), w)
    for idx in range(w0.numel()):
        h = 1e-6
        wp, wm = w0.clone(), w0.clone()
        wp[idx] += h
        wm[idx] -= h
        with torch.no_grad():
            fd = (total(wp) - total(wm)).item() / (2 * h)
        assert abs(g[idx].item() - fd) <= 1e-3 + 1e-2 * abs(fd), (idx, g[idx].item(), fd)
