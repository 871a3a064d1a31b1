"""Whole SQP solves of benchmark configurations 4 (quadrotor with spherical obstacles,
warm-started re-solve) and 5 (Clohessy-Wiltshire with a learned MLP stage
cost, forward + VJP) on the GPU, against the same SQP loop whose ADMM solves
run in the NumPy oracle (fp64, fixed SQP/ADMM/PCG counts; tolerance 1e-6
relative), at reduced batch and horizon."""
import numpy as np
import pytest
import torch

from tests.helpers import oracle_admm_solve, rel_err
from turbompc_b200 import ops
from turbompc_b200.problems.quadrotor import make_obstacle_problem
from turbompc_b200.solver import TurboMPCSolver

pytestmark = pytest.mark.gpu


def _fixed(sqp, admm, pcg):
    return {"num_sqp_iteration_max": sqp, "tol_convergence": 0.0,
            "admm": {"max_iter": admm, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": 0.0,
                     "eps_rel": 0.0, "rho": 0.1, "pcg": {"max_iter": pcg, "tol_epsilon": 0.0}}}


def _both(monkeypatch, solver, guess, params):
    a = solver.solve(guess, params)
    with monkeypatch.context() as mp:
        mp.setattr(ops, "admm_solve", oracle_admm_solve)
        b = solver.solve(guess, params)
    return a, b


def test_config4_obstacles_with_warm_start_matches_oracle(monkeypatch):
    prog, params = make_obstacle_problem(4, N=12, n_obstacles=8, seed=5, dtype=torch.float64, device="cuda")
    assert prog.num_inequality_constraints == 12  # 4 thrust rows + 8 spheres
    s = TurboMPCSolver(prog, _fixed(3, 25, 10))
    g0 = s.initial_guess(params)
    a, b = _both(monkeypatch, s, g0, params)
    for x, y in ((a.states, b.states), (a.controls, b.controls), (a.admm_state.y_g, b.admm_state.y_g),
                 (a.admm_state.y_f_dyn, b.admm_state.y_f_dyn)):
        assert rel_err(x.cpu().numpy(), y.cpu().numpy()) < 1e-6
    # Warm start (config 4: the previous solution and its ADMM state).
    g1 = a._replace(states=a.states.detach(), controls=a.controls.detach())
    a2, b2 = _both(monkeypatch, s, g1, params)
    assert rel_err(a2.states.cpu().numpy(), b2.states.cpu().numpy()) < 1e-6
    assert rel_err(a2.controls.cpu().numpy(), b2.controls.cpu().numpy()) < 1e-6


def test_config5_learned_cost_forward_matches_oracle(monkeypatch):
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    prog, params = make_learned_cost_problem(3, N=10, hidden=16, seed=2, dtype=torch.float64, device="cuda")
    s = TurboMPCSolver(prog, _fixed(3, 30, 10))
    a, b = _both(monkeypatch, s, s.initial_guess(params), params)
    assert rel_err(a.states.cpu().numpy(), b.states.cpu().numpy()) < 1e-6
    assert rel_err(a.controls.cpu().numpy(), b.controls.cpu().numpy()) < 1e-6
    assert rel_err(a.admm_state.y_f_dyn.cpu().numpy(), b.admm_state.y_f_dyn.cpu().numpy()) < 1e-6


def _fd(f, w, idx, h):
    wp, wm = w.clone(), w.clone()
    wp.view(-1)[idx] += h
    wm.view(-1)[idx] -= h
    return (f(wp) - f(wm)) / (2 * h)


@pytest.mark.parametrize("path,idxs,h", [(("initial_state",), (0, 4, 8), 1e-6),
                                         (("mlp_W1",), (0, 17, 40), 1e-5),
                                         (("mlp_w2",), (1, 5), 1e-5),
                                         (("dynamics_state_dot_params", "A"), (3, 22), 1e-7),
                                         (("dynamics_state_dot_params", "B"), (9, 14), 1e-5)])
def test_config5_vjp_matches_finite_differences(path, idxs, h):
    """VJP w.r.t. x0, the MLP cost parameters and the A, B blocks (fp64,
    converged solves, exact-Hessian backward) against central differences
    (atol 1e-3, rtol 1e-2 as the quadrotor gradient test)."""
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    prog, params = make_learned_cost_problem(2, N=8, hidden=16, seed=3, dtype=torch.float64, device="cuda")
    sp = {"num_sqp_iteration_max": 8, "tol_convergence": 0.0,
          "admm": {"max_iter": 3000, "check_termination_every": 10, "adapt_rho_every": 50, "eps_abs": 1e-11,
                   "eps_rel": 1e-11, "pcg": {"max_iter": 1, "tol_epsilon": 0.0}}}
    solver = TurboMPCSolver(prog, sp, forward_backend="b200_direct", use_full_hessian=True)
    guess = solver.initial_guess(params)

    def put(w):
        if len(path) == 1:
            return {path[0]: w}
        return {path[0]: dict(params[path[0]], **{path[1]: w})}

    w0 = (params[path[0]] if len(path) == 1 else params[path[0]][path[1]]).clone()
    loss = lambda sol: (sol.states ** 2).sum() + 3.0 * (sol.controls ** 2).sum()

    def run(w):
        with torch.no_grad():
            return loss(solver.solve(guess, params, put(w))).item()

    w = w0.clone().requires_grad_(True)
    g, = torch.autograd.grad(loss(solver.solve(guess, params, put(w))), w)
    for idx in idxs:
        fd = _fd(run, w0, idx, h)
        gv = g.reshape(-1)[idx].item()
        assert abs(gv - fd) <= 1e-3 + 1e-2 * abs(fd), (idx, gv, fd)
