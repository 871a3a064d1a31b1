"""Pins of the whole-solve oracle (oracle/sqp_ref.py) on the CPU, and of the
b200 QP builder against it.

* Closed-form fixtures derived by hand from the reference's cost convention
  (turbompc/problems/optimal_control_problem.py:982-1030: sum w (z - r)^2 with
  no 1/2, terminal weight w_ref + w_final, 0.5 du^T Rd du on the control rate)
  pin the oracle's autodiff cost blocks and the b200 closed-form blocks.
* The b200 QP builder (CPU PyTorch path) equals the oracle's QP at perturbed
  linearisation points of the benchmark problems.
* The oracle's VJP (backward QP, dense adjoint KKT, mixed derivatives by
  jacfwd over the weights) equals central finite differences of the oracle's
  own converged solve, for hard constraints and for soft (slack) constraints.
"""
import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from oracle import sqp_ref as sr
from turbompc_b200.dynamics import LinearDynamics
from turbompc_b200.problems.ocp import OptimalControlProblem

F64 = torch.float64


def _di_params(batch=2, N=5, rate=(0.0, 0.0), umax=0.6, seed=0, slack=None):
    """Benchmark configuration 1 (double integrator, dt = 0.1) through the
    reference's dt = 1 Euler trick: A_c = A_d - I, B_c = B_d."""
    dt = 0.1
    I2 = np.eye(2)
    Ad = np.block([[I2, dt * I2], [np.zeros((2, 2)), I2]])
    Bd = np.concatenate([0.5 * dt * dt * I2, dt * I2], 0)
    rng = np.random.default_rng(seed)
    t = lambda a: torch.as_tensor(np.asarray(a, dtype=np.float64))
    p = {
        "horizon": N, "discretization_resolution": 1.0, "discretization_scheme": 0,
        "initial_state": t(rng.uniform(-2, 2, size=(batch, 4))),
        "reference_state_trajectory": t(np.zeros(4)), "reference_control_trajectory": t(np.zeros(2)),
        "penalize_control_reference": False,
        "weights_penalization_reference_state_trajectory": t(np.ones(4)),
        "weights_penalization_final_state": t(np.full(4, 9.0)),
        "weights_penalization_control_squared": t(np.full(2, 0.1)),
        "weights_penalization_control_rate": t(np.asarray(rate)),
        "state_min_bounds": t(np.full(4, -10.0)), "state_max_bounds": t(np.full(4, 10.0)),
        "control_min_bounds": t(np.full(2, -umax)), "control_max_bounds": t(np.full(2, umax)),
        "dynamics_state_dot_params": {"A": t(Ad - np.eye(4)), "B": t(Bd)},
    }
    if slack is not None:
        p["use_slack_variables"] = True
        p["slack_penalization_weight"] = t(slack)
    return p


def _closed_form_blocks(N, w_x, w_u, w_f, rd):
    """D, E, q of sum_t w (z_t)^2 + 0.5 du^T Rd du with zero references."""
    nx, nu = len(w_x), len(w_u)
    n = nx + nu
    D = np.zeros((N + 1, n, n))
    for t in range(N + 1):
        wx = np.asarray(w_x) + (np.asarray(w_f) if t == N else 0.0)
        D[t] = np.diag(np.concatenate([2 * wx, 2 * np.asarray(w_u)]))
        Rd = np.diag(rd)
        k = (1 if t < N else 0) + (1 if t > 0 else 0)  # rate terms touching u_t
        D[t, nx:, nx:] += k * Rd
    E = np.zeros((N, n, n))
    E[:, nx:, nx:] = -np.diag(rd)
    return D, E, np.zeros((N + 1, n))


@pytest.mark.parametrize("rate", [(0.0, 0.0), (0.5, 2.0)])
def test_cost_blocks_match_closed_form(rate):
    p = _di_params(rate=rate)
    Dw, Ew, qw = _closed_form_blocks(5, [1.0] * 4, [0.1] * 2, [9.0] * 4, rate)
    o = sr.OCP("linear", 4, 2, sr.problem_params(p, 0))
    X = torch.randn(6, 4, dtype=F64)
    U = torch.randn(6, 2, dtype=F64)
    D, E, q = o.cost_blocks(X, U, o.p)
    np.testing.assert_allclose(D.numpy(), Dw, atol=1e-13)
    np.testing.assert_allclose(E.numpy(), Ew, atol=1e-13)
    np.testing.assert_allclose(q.numpy(), qw, atol=1e-13)
    # the b200 closed-form blocks (turbompc_b200/problems/ocp.py)
    prog = OptimalControlProblem(LinearDynamics(4, 2), p)
    D2, E2, q2 = prog.get_cost_linearized_blocks(X[None].expand(2, 6, 4), U[None].expand(2, 6, 2), p)
    np.testing.assert_allclose(D2[0].numpy(), Dw, atol=1e-13)
    np.testing.assert_allclose(E2[0].numpy(), Ew, atol=1e-13)
    np.testing.assert_allclose(q2[0].numpy(), qw, atol=1e-13)


def test_terminal_reference_and_linear_weight_in_q():
    """q_N = -2 (w + w_f) r + w_lin and q_t = -2 w r (optimal_control_problem.py:1011-1028)."""
    p = _di_params()
    r = np.array([0.3, -0.2, 0.1, 0.5])
    p["reference_state_trajectory"] = torch.as_tensor(r)
    p["weights_linear_penalization_final_state"] = torch.as_tensor([1.0, 2.0, 3.0, 4.0])
    o = sr.OCP("linear", 4, 2, sr.problem_params(p, 0))
    _, _, q = o.cost_blocks(torch.zeros(6, 4, dtype=F64), torch.zeros(6, 2, dtype=F64), o.p)
    np.testing.assert_allclose(q[2, :4].numpy(), -2.0 * r, atol=1e-13)
    np.testing.assert_allclose(q[5, :4].numpy(), -2.0 * 10.0 * r + np.array([1.0, 2.0, 3.0, 4.0]), atol=1e-13)


def rescaled(p, nx, nu, u0=True):
    """Turn on rescale_optimization_variables (and a fixed initial control)."""
    p = dict(p)
    p["rescale_optimization_variables"] = True
    p["state_rescaling_min"] = torch.as_tensor(-np.linspace(1.0, 4.0, nx), dtype=F64)
    p["state_rescaling_max"] = torch.as_tensor(np.linspace(2.0, 5.0, nx), dtype=F64)
    p["control_rescaling_min"] = torch.as_tensor(np.linspace(-0.5, 0.0, nu), dtype=F64)
    p["control_rescaling_max"] = torch.as_tensor(np.linspace(5.0, 6.0, nu), dtype=F64)
    if u0:
        p["constrain_initial_control"] = True
        p["initial_control"] = torch.as_tensor(np.linspace(1.0, 2.0, nu), dtype=F64)
    return p


def _problem(kind, batch, N):
    from turbompc_b200.dynamics import Quadrotor12Dynamics
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    from turbompc_b200.problems.ocp import OptimalControlProblem, OptimalControlProblemObstacle
    from turbompc_b200.problems.quadrotor import make_obstacle_problem, make_quadrotor_problem
    if kind == "quadrotor":
        prog, p = make_quadrotor_problem(batch, N=N, seed=3, dtype=F64, device="cpu")
        return prog, p, dict(model="quadrotor12")
    if kind == "quadrotor_rescaled":
        _, p = make_quadrotor_problem(batch, N=N, seed=3, dtype=F64, device="cpu")
        p = rescaled(p, 12, 4)
        return OptimalControlProblem(Quadrotor12Dynamics(), p), p, dict(model="quadrotor12")
    if kind == "obstacles_rescaled":
        _, p = make_obstacle_problem(batch, N=N, seed=3, dtype=F64, device="cpu")
        p = rescaled(p, 12, 4, u0=False)
        return OptimalControlProblemObstacle(Quadrotor12Dynamics(), p), p, dict(model="quadrotor12", obstacles=True)
    if kind == "obstacles":
        prog, p = make_obstacle_problem(batch, N=N, seed=3, dtype=F64, device="cpu")
        return prog, p, dict(model="quadrotor12", obstacles=True)
    prog, p = make_learned_cost_problem(batch, N=N, hidden=16, seed=3, dtype=F64, device="cpu")
    return prog, p, dict(model="linear", mlp=True)


@pytest.mark.parametrize("kind", ["quadrotor", "obstacles", "cw_mlp", "quadrotor_rescaled", "obstacles_rescaled"])
def test_b200_qp_builder_matches_oracle_qp(kind):
    from turbompc_b200.solver import TurboMPCSolver
    prog, p, kw = _problem(kind, 3, 8)
    if kind == "quadrotor":
        p["weights_penalization_control_rate"] = torch.tensor([0.3, 0.1, 0.2, 0.4], dtype=F64)
    s = TurboMPCSolver(prog, {"num_sqp_iteration_max": 1})
    g = s.initial_guess(p)
    if kind.endswith("rescaled"):
        assert prog.rescale_optimization_variables
        assert s._build_qp_data(g.states, g.controls, p).n0 == (16 if kind == "quadrotor_rescaled" else 12)
    gen = torch.Generator().manual_seed(4)
    X = g.states + 0.05 * torch.randn(g.states.shape, generator=gen, dtype=F64)
    U = g.controls + 0.3 * torch.rand(g.controls.shape, generator=gen, dtype=F64)
    qd = s._build_qp_data(X, U, p).tensors()
    names = dict(D="D", E="E", q="q", A0="A0", A_minus="Am", A_plus="Ap", c0="c0", c="c", G="G", l="l", u="u")
    for b in range(3):
        o = sr.OCP(kw["model"], prog.num_state_variables, prog.num_control_variables, sr.problem_params(p, b),
                   obstacles=kw.get("obstacles", False), mlp=kw.get("mlp", False))
        q = o.qp(X[b], U[b], o.p)
        for k, kk in names.items():
            want = getattr(q, kk)[0]
            scale = max(1.0, float(np.abs(want).max()) if want.size else 1.0)
            assert float(np.abs(qd[k][b].numpy() - want).max() if want.size else 0.0) <= 1e-12 * scale, (kind, k)


def test_oracle_dynamics_jacobian_matches_finite_differences():
    prog, p, kw = _problem("quadrotor", 1, 4)
    o = sr.OCP("quadrotor12", 12, 4, sr.problem_params(p, 0))
    gen = torch.Generator().manual_seed(1)
    X = 0.3 * torch.randn(5, 12, generator=gen, dtype=F64)
    U = 2.0 + torch.rand(5, 4, generator=gen, dtype=F64)
    Am, _, c = o.dynamics_rows(X, U, o.p)
    h = 1e-6
    for j in range(16):
        e = torch.zeros(16, dtype=F64)
        e[j] = h
        xu = torch.cat([X[1], U[1]])
        fp = o.next_state((xu + e)[:12], (xu + e)[12:], o.p)
        fm = o.next_state((xu - e)[:12], (xu - e)[12:], o.p)
        np.testing.assert_allclose(Am[1, :, j].numpy(), ((fp - fm) / (2 * h)).numpy(), rtol=1e-6, atol=1e-8)
    # c = -f(y) + J y
    f1 = o.next_state(X[1], U[1], o.p)
    np.testing.assert_allclose(c[1].numpy(), (-f1 + Am[1] @ torch.cat([X[1], U[1]])).numpy(), atol=1e-12)


# --------------------------------------------------------------- VJP pins
CONVERGED = ref.ADMMConfig(max_iter=4000, pcg_max_iter=1, check_every=5, eps_abs=1e-13, eps_rel=1e-13,
                           adapt_rho_every=25, rho_f_factor=1000.0, alpha=1.6)


def _loss_and_cot(sol, Ws, Wc):
    return float(np.sum(Ws * sol.states) + np.sum(Wc * sol.controls))


def _oracle_fd_check(make, key, idxs, num_sqp, h, use_slack=False, rtol=1e-5):
    """Oracle VJP of L = <Ws, states> + <Wc, controls> w.r.t. p[key] at the
    given flat indices vs central differences of the oracle's converged solve."""
    cfg = ref.ADMMConfig(**{**CONVERGED.__dict__, "use_slack": use_slack})
    o = make(None)
    rng = np.random.default_rng(7)
    Ws = rng.normal(size=(o.T, o.nx))
    Wc = rng.normal(size=(o.T, o.nu))
    X0 = torch.zeros(o.T, o.nx, dtype=F64) + 1e-6
    U0 = torch.zeros(o.T, o.nu, dtype=F64) + 1e-6
    X0[:] = o.p["initial_state"]
    sol = sr.solve(o, X0, U0, cfg, num_sqp, linsys="dense")
    assert (sol.active_lower | sol.active_upper).any()
    grads, _ = sr.vjp(o, sol, Ws, Wc, weight_keys=(() if key == "initial_state" else ((key,),)))
    gk = grads["initial_state"] if key == "initial_state" else grads[(key,)]
    base = sr._get(o.p, (key,)).clone()
    for i in idxs:
        vals = []
        for sgn in (1, -1):
            w = base.clone()
            w.view(-1)[i] += sgn * h
            oo = make(w)
            vals.append(_loss_and_cot(sr.solve(oo, X0, U0, cfg, num_sqp, linsys="dense"), Ws, Wc))
        fd = (vals[0] - vals[1]) / (2 * h)
        g = float(np.asarray(gk).reshape(-1)[i])
        assert abs(g - fd) <= rtol * max(1.0, abs(fd)), (key, i, g, fd)
    return grads


def _di_ocp(key=None, slack=None, umax=0.6):
    def make(w):
        p = sr.problem_params(_di_params(batch=1, N=6, rate=(0.2, 0.0), umax=umax, slack=slack), 0)
        if w is not None:
            p = sr._set(p, (key,), w)
        return sr.OCP("linear", 4, 2, p, use_slack=slack is not None, eps_abs=1e-9, eps_rel=1e-9)
    return make


@pytest.mark.parametrize("key", ["weights_penalization_reference_state_trajectory",
                                 "weights_penalization_control_squared", "initial_state"])
def test_oracle_vjp_matches_finite_differences_linear(key):
    _oracle_fd_check(_di_ocp(key), key, range(4 if key != "weights_penalization_control_squared" else 2), 1,
                     h=1e-5)


def test_oracle_vjp_matches_finite_differences_nonlinear_learned_cost():
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    _, pfull = make_learned_cost_problem(1, N=4, hidden=6, seed=5, dtype=F64, device="cpu", u_max=0.05)
    key = "mlp_W1"

    def make(w):
        p = sr.problem_params(pfull, 0)
        if w is not None:
            p = sr._set(p, (key,), w)
        return sr.OCP("linear", 6, 3, p, mlp=True)

    _oracle_fd_check(make, key, [0, 7, 13, 30], 12, h=1e-5)


@pytest.mark.parametrize("key", ["initial_state", "initial_control", "weights_penalization_control_squared"])
def test_oracle_vjp_matches_finite_differences_rescaled_with_initial_control(key):
    """Rescaled variables and a fixed initial control (optimal_control_problem.py:
    284-325, 914-980; turbompc_solver.py:990-1018)."""
    def make(w):
        p = sr.problem_params(rescaled(_di_params(batch=1, N=6, rate=(0.2, 0.0), umax=0.6), 4, 2), 0)
        p["initial_control"] = torch.tensor([0.3, -0.2], dtype=F64)
        if w is not None:
            p = sr._set(p, (key,), w)
        return sr.OCP("linear", 4, 2, p, eps_abs=1e-9, eps_rel=1e-9)

    o = make(None)
    assert o.rescale and o.constrain_u0
    cfg = ref.ADMMConfig(**CONVERGED.__dict__)
    rng = np.random.default_rng(7)
    Ws, Wc = rng.normal(size=(o.T, 4)), rng.normal(size=(o.T, 2))
    X0 = torch.zeros(o.T, 4, dtype=F64)
    X0[:] = o.p["initial_state"]
    U0 = torch.zeros(o.T, 2, dtype=F64)
    sol = sr.solve(o, X0, U0, cfg, 1, linsys="dense")
    np.testing.assert_allclose(sol.controls[0], [0.3, -0.2], atol=1e-9)  # the initial control is fixed
    assert (sol.active_lower | sol.active_upper).any()
    wk = () if key in ("initial_state", "initial_control") else ((key,),)
    grads, _ = sr.vjp(o, sol, Ws, Wc, weight_keys=wk)
    g = grads[key] if key in grads else grads[(key,)]
    base = sr._get(o.p, (key,)).clone()
    h = 1e-5
    for i in range(base.numel()):
        vals = []
        for sgn in (1, -1):
            w = base.clone()
            w.view(-1)[i] += sgn * h
            vals.append(_loss_and_cot(sr.solve(make(w), X0, U0, cfg, 1, linsys="dense"), Ws, Wc))
        fd = (vals[0] - vals[1]) / (2 * h)
        assert abs(float(np.asarray(g).reshape(-1)[i]) - fd) <= 1e-5 * max(1.0, abs(fd)), (key, i, g, fd)


def test_oracle_vjp_matches_finite_differences_slack():
    """Soft constraints (turbompc_solver.py:587-612, 620-640): the slack
    branch of the backward QP, including dL/d(slack weight)."""
    make = _di_ocp("slack_penalization_weight", slack=5.0, umax=0.3)
    o = make(None)
    cfg = ref.ADMMConfig(**{**CONVERGED.__dict__, "use_slack": True})
    X0 = torch.zeros(o.T, 4, dtype=F64)
    X0[:] = o.p["initial_state"]
    U0 = torch.zeros(o.T, 2, dtype=F64)
    sol = sr.solve(o, X0, U0, cfg, 1, linsys="dense")
    assert (sol.active_lower | sol.active_upper).any()
    rng = np.random.default_rng(7)
    Ws, Wc = rng.normal(size=(o.T, 4)), rng.normal(size=(o.T, 2))
    grads, _ = sr.vjp(o, sol, Ws, Wc, weight_keys=(("weights_penalization_control_squared",),))
    h = 1e-5
    for key, g in (("slack_penalization_weight", grads["slack_penalization_weight"]),
                   ("weights_penalization_control_squared", grads[("weights_penalization_control_squared",)][0])):
        base = sr._get(o.p, (key,)).clone()
        vals = []
        for sgn in (1, -1):
            w = base.clone()
            w.view(-1)[0] += sgn * h
            p = sr._set(o.p, (key,), w)
            oo = sr.OCP("linear", 4, 2, p, use_slack=True, eps_abs=1e-9, eps_rel=1e-9)
            vals.append(_loss_and_cot(sr.solve(oo, X0, U0, cfg, 1, linsys="dense"), Ws, Wc))
        fd = (vals[0] - vals[1]) / (2 * h)
        assert abs(float(g) - fd) <= 1e-5 * max(1.0, abs(fd)), (key, float(g), fd)
