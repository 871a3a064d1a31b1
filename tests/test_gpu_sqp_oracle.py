"""Whole solves through the public API (TurboMPCSolver, forward_backend="b200")
against the whole-solve oracle (oracle/sqp_ref.py: the reference's SQP loop,
linearisation and ADMM restated on the CPU in float64, sharing no code with the
b200 path), at the benchmarks' shapes and fixed iteration counts:

  config 3  quadrotor N = 50, 5 SQP x 30 ADMM x 30 PCG (fp32: the 52-stage
            register-resident kernel; fp64: the shared-memory kernel)
  config 4  quadrotor N = 40 with 8 spheres, 10 SQP x 50 ADMM x 30 PCG, then a
            warm-started re-solve from the previous solution and ADMM state
  config 5  Clohessy-Wiltshire with the learned MLP stage cost, N = 60,
            3 SQP x 50 ADMM x 30 PCG (fp32: the 64-stage instance), and the VJP
            w.r.t. x0, the MLP parameters and the dynamics' A, B
  soft constraints: the VJP through slack variables, including the cotangent
            of slack_penalization_weight.

Tolerances (the parity bar): 1e-6 relative in fp64 and 1e-3 relative in fp32,
||a - b||_inf / ||b||_inf over the batch, on states, controls, y_g, y_f, z_g
and on every gradient.
"""
import functools

import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from oracle import sqp_ref as sr
from tests.helpers import rel_err
from turbompc_b200.solver import TurboMPCSolver

pytestmark = pytest.mark.gpu
F64 = torch.float64
TOL = {torch.float32: 1e-3, torch.float64: 1e-6}
# Active sets of the backward pass use eps_abs / eps_rel (turbompc_solver.py:
# 1387-1439); with no residual checks (check_termination_every = 0) they do
# not touch the ADMM iteration itself.
EPS_KKT = 1e-6
# Configuration 5 with the control box tightened to |u| <= 0.02 so that it is
# active (at the default 0.1 no row is active and y_g is zero).
CW_KW = (("u_max", 0.02),)


def _fixed(sqp, admm, pcg):
    return {"num_sqp_iteration_max": sqp, "tol_convergence": 0.0,
            "admm": {"max_iter": admm, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": EPS_KKT,
                     "eps_rel": EPS_KKT, "rho": 0.1, "pcg": {"max_iter": pcg, "tol_epsilon": 0.0}}}


def _ocfg(admm, pcg, use_slack=False):
    return ref.ADMMConfig(max_iter=admm, pcg_max_iter=pcg, check_every=0, eps_abs=0.0, eps_rel=0.0, pcg_eps=0.0,
                          adapt_rho_every=0, use_slack=use_slack)


def _make(kind, batch, N, dtype, device, **kw):
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    from turbompc_b200.problems.quadrotor import make_obstacle_problem, make_quadrotor_problem
    if kind == "quadrotor":
        return make_quadrotor_problem(batch, N=N, seed=21, dtype=dtype, device=device, **kw)
    if kind == "obstacles":
        return make_obstacle_problem(batch, N=N, seed=22, dtype=dtype, device=device, **kw)
    return make_learned_cost_problem(batch, N=N, seed=23, dtype=dtype, device=device, **kw)


MODEL = {"quadrotor": dict(model="quadrotor12"), "obstacles": dict(model="quadrotor12", obstacles=True),
         "cw_mlp": dict(model="linear", mlp=True)}


def _oracle_ocp(kind, prog, params, b, use_slack=False):
    return sr.OCP(nx=prog.num_state_variables, nu=prog.num_control_variables, p=sr.problem_params(params, b),
                  use_slack=use_slack, eps_abs=EPS_KKT, eps_rel=EPS_KKT, **MODEL[kind])


@functools.lru_cache(maxsize=None)
def _oracle_run(kind, batch, N, sqp, admm, pcg, warm, kw=(), linsys="pcg"):
    """Oracle solutions of the float64 problem (and, with warm, of a
    warm-started re-solve from the first solution).  linsys "dense" solves
    each ADMM linear system exactly (the direct backend's semantics)."""
    prog, params = _make(kind, batch, N, F64, "cpu", **dict(kw))
    s = TurboMPCSolver(prog, _fixed(sqp, admm, pcg))
    g = s.initial_guess(params)
    cfg = _ocfg(admm, pcg)
    sols = [sr.solve(_oracle_ocp(kind, prog, params, b), g.states[b], g.controls[b], cfg, sqp, linsys=linsys)
            for b in range(batch)]
    sols2 = None
    if warm:
        sols2 = [sr.solve(_oracle_ocp(kind, prog, params, b), sols[b].states, sols[b].controls, cfg, sqp,
                          admm_state0=sols[b].state, linsys=linsys) for b in range(batch)]
    return prog, params, sols, sols2


def _check_solution(sol, osols, dtype, what=""):
    tol = TOL[dtype]
    st = sol.admm_state
    pairs = [("states", sol.states, [o.states for o in osols]), ("controls", sol.controls, [o.controls for o in osols]),
             ("y_g", st.y_g, [o.state.y_g[0] for o in osols]), ("y_f0", st.y_f_0, [o.state.y_f0[0] for o in osols]),
             ("y_fdyn", st.y_f_dyn, [o.state.y_fdyn[0] for o in osols]),
             ("z_g", st.z_g, [o.state.z_g[0] for o in osols])]
    for name, got, want in pairs:
        e = rel_err(got.detach().cpu().numpy(), np.stack(want))
        assert e < tol, (what, name, e)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_config3_quadrotor_whole_solve_matches_oracle(dtype):
    B, N, sqp, admm, pcg = 4, 50, 5, 30, 30
    prog64, p64, osols, _ = _oracle_run("quadrotor", B, N, sqp, admm, pcg, False)
    prog, params = _make("quadrotor", B, N, dtype, "cuda")
    s = TurboMPCSolver(prog, _fixed(sqp, admm, pcg), forward_backend="b200")
    sol = s.solve(s.initial_guess(params), params)
    assert (sol.admm_iters[:, :sqp] == admm).all()
    _check_solution(sol, osols, dtype, "config 3")


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_config3_quadrotor_direct_backend_matches_oracle(dtype):
    """The direct backend ("b200_direct", the drop-in for the reference's
    default admm_fused_cudss): each ADMM linear system solved exactly, here by
    the batch-interleaved block-Cholesky kernels (n = 16 fp32; fp64 runs the
    warp-per-problem kernel, n > 12), against the oracle with dense solves."""
    B, N, sqp, admm = 4, 50, 5, 30
    _, _, osols, _ = _oracle_run("quadrotor", B, N, sqp, admm, 1, False, linsys="dense")
    prog, params = _make("quadrotor", B, N, dtype, "cuda")
    s = TurboMPCSolver(prog, _fixed(sqp, admm, 1), forward_backend="b200_direct")
    sol = s.solve(s.initial_guess(params), params)
    assert (sol.admm_iters[:, :sqp] == admm).all()
    _check_solution(sol, osols, dtype, "config 3 direct")


def test_quadrotor_control_rate_direct_backend_matches_oracle_fp32():
    """A control-rate penalty puts nonzero control rows into E_t, so the rows
    nx..n-1 of every W_t are not zero: the interleaved direct path must detect
    that and run its full kernel variant (W read whole); against the oracle
    with dense solves."""
    B, N, sqp, admm = 4, 50, 3, 30
    kw = (("rate_weight", 0.5),)
    _, _, osols, _ = _oracle_run("quadrotor", B, N, sqp, admm, 1, False, kw, linsys="dense")
    prog, params = _make("quadrotor", B, N, torch.float32, "cuda", **dict(kw))
    s = TurboMPCSolver(prog, _fixed(sqp, admm, 1), forward_backend="b200_direct")
    g = s.initial_guess(params)
    qp = s._build_qp_data(g.states, g.controls, params)
    assert bool((qp.cost.E[..., 12:, :] != 0).any())
    _check_solution(s.solve(g, params), osols, torch.float32, "quadrotor control rate direct")


def test_config4_and_5_direct_backend_match_oracle_fp32():
    """Obstacle rows (m = 12, warm-started re-solve) and the CW + MLP problem
    (n = 9: the interleaved kernels with padded stage blocks) on the direct
    backend against the oracle with dense solves."""
    B, N, sqp, admm = 2, 40, 10, 50
    _, _, osols, osols2 = _oracle_run("obstacles", B, N, sqp, admm, 1, True, linsys="dense")
    prog, params = _make("obstacles", B, N, torch.float32, "cuda")
    s = TurboMPCSolver(prog, _fixed(sqp, admm, 1), forward_backend="b200_direct")
    sol = s.solve(s.initial_guess(params), params)
    _check_solution(sol, osols, torch.float32, "config 4 direct")
    sol2 = s.solve(sol._replace(states=sol.states.detach(), controls=sol.controls.detach()), params)
    _check_solution(sol2, osols2, torch.float32, "config 4 direct warm start")
    B, N, sqp, admm = 3, 60, 3, 50
    _, _, osols, _ = _oracle_run("cw_mlp", B, N, sqp, admm, 1, False, CW_KW, linsys="dense")
    prog, params = _make("cw_mlp", B, N, torch.float32, "cuda", **dict(CW_KW))
    s = TurboMPCSolver(prog, _fixed(sqp, admm, 1), forward_backend="b200_direct")
    _check_solution(s.solve(s.initial_guess(params), params), osols, torch.float32, "config 5 direct")


def test_config4_obstacles_with_warm_start_matches_oracle_fp32():
    B, N, sqp, admm, pcg = 2, 40, 10, 50, 30
    _, _, osols, osols2 = _oracle_run("obstacles", B, N, sqp, admm, pcg, True)
    prog, params = _make("obstacles", B, N, torch.float32, "cuda")
    assert prog.num_inequality_constraints == 12
    s = TurboMPCSolver(prog, _fixed(sqp, admm, pcg), forward_backend="b200")
    sol = s.solve(s.initial_guess(params), params)
    _check_solution(sol, osols, torch.float32, "config 4")
    sol2 = s.solve(sol._replace(states=sol.states.detach(), controls=sol.controls.detach()), params)
    _check_solution(sol2, osols2, torch.float32, "config 4 warm start")


def test_config5_learned_cost_forward_matches_oracle_fp32():
    B, N, sqp, admm, pcg = 3, 60, 3, 50, 30
    _, _, osols, _ = _oracle_run("cw_mlp", B, N, sqp, admm, pcg, False, CW_KW)
    prog, params = _make("cw_mlp", B, N, torch.float32, "cuda", **dict(CW_KW))
    s = TurboMPCSolver(prog, _fixed(sqp, admm, pcg), forward_backend="b200")
    _check_solution(s.solve(s.initial_guess(params), params), osols, torch.float32, "config 5")


def _oracle_vjp(kind, prog, params, osols, Ws, Wc, keys, use_slack=False, Wsl=None):
    out = {}
    for b, o in enumerate(osols):
        ocp = _oracle_ocp(kind, prog, params, b, use_slack=use_slack)
        g, _ = sr.vjp(ocp, o, Ws[b], Wc[b], weight_keys=tuple(k for k in keys if k[0] not in
                                                                 ("initial_state", "slack_penalization_weight")),
                      dl_dslack=None if Wsl is None else Wsl[b])
        for k in keys:
            if k == ("initial_state",):
                out.setdefault(k, []).append(g["initial_state"])
            elif k == ("slack_penalization_weight",):
                out[k] = out.get(k, 0.0) + g["slack_penalization_weight"]
            else:
                out[k] = out.get(k, 0.0) + g[k]  # weights shared by the batch: cotangents add up
    return {k: (np.stack(v) if isinstance(v, list) else np.asarray(v)) for k, v in out.items()}


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_config5_vjp_matches_oracle(dtype):
    B, N, sqp, admm, pcg = 2, 60, 3, 50, 30
    kw = CW_KW + (("hidden", 16),)
    prog64, p64, osols, _ = _oracle_run("cw_mlp", B, N, sqp, admm, pcg, False, kw)
    prog, params = _make("cw_mlp", B, N, dtype, "cuda", **dict(kw))
    s = TurboMPCSolver(prog, _fixed(sqp, admm, pcg), forward_backend="b200", backward_backend="b200")
    rng = np.random.default_rng(3)
    Ws = rng.normal(size=(B, N + 1, 6))
    Wc = rng.normal(size=(B, N + 1, 3))
    dp = params["dynamics_state_dot_params"]
    leaves = {("initial_state",): params["initial_state"], ("mlp_W1",): params["mlp_W1"],
              ("mlp_b1",): params["mlp_b1"], ("mlp_w2",): params["mlp_w2"],
              ("dynamics_state_dot_params", "A"): dp["A"], ("dynamics_state_dot_params", "B"): dp["B"]}
    lv = {k: v.detach().clone().requires_grad_(True) for k, v in leaves.items()}
    weights = {"initial_state": lv[("initial_state",)], "mlp_W1": lv[("mlp_W1",)], "mlp_b1": lv[("mlp_b1",)],
               "mlp_w2": lv[("mlp_w2",)], "dynamics_state_dot_params": {
                   "A": lv[("dynamics_state_dot_params", "A")], "B": lv[("dynamics_state_dot_params", "B")]}}
    sol = s.solve(s.initial_guess(params), params, weights)
    tt = lambda a: torch.as_tensor(a, dtype=dtype, device="cuda")
    loss = (sol.states * tt(Ws)).sum() + (sol.controls * tt(Wc)).sum()
    grads = torch.autograd.grad(loss, list(lv.values()))
    want = _oracle_vjp("cw_mlp", prog64, p64, osols, Ws, Wc, list(lv.keys()))
    for k, g in zip(lv.keys(), grads):
        e = rel_err(g.cpu().numpy(), want[k])
        assert e < TOL[dtype], (k, e)


def _slack_problem(dtype, device, batch=3, N=12):
    from turbompc_b200.dynamics import LinearDynamics
    from turbompc_b200.problems.ocp import OptimalControlProblem
    dt = 0.1
    I2 = np.eye(2)
    Ad = np.block([[I2, dt * I2], [np.zeros((2, 2)), I2]])
    Bd = np.concatenate([0.5 * dt * dt * I2, dt * I2], 0)
    rng = np.random.default_rng(4)
    t = lambda a: torch.as_tensor(np.asarray(a, dtype=np.float64), dtype=dtype, device=device)
    params = {
        "horizon": N, "discretization_resolution": 1.0, "discretization_scheme": 0,
        "initial_state": t(rng.uniform(-2, 2, size=(batch, 4))),
        "reference_state_trajectory": t(np.zeros(4)), "reference_control_trajectory": t(np.zeros(2)),
        "penalize_control_reference": False,
        "weights_penalization_reference_state_trajectory": t(np.ones(4)),
        "weights_penalization_final_state": t(np.full(4, 9.0)),
        "weights_penalization_control_squared": t(np.full(2, 0.1)),
        "weights_penalization_control_rate": t(np.zeros(2)),
        "state_min_bounds": t(np.full(4, -10.0)), "state_max_bounds": t(np.full(4, 10.0)),
        "control_min_bounds": t(np.full(2, -0.3)), "control_max_bounds": t(np.full(2, 0.3)),
        "dynamics_state_dot_params": {"A": t(Ad - np.eye(4)), "B": t(Bd)},
        "use_slack_variables": True, "slack_penalization_weight": t(5.0),
    }
    return OptimalControlProblem(LinearDynamics(4, 2), params), params


def test_soft_constraint_vjp_matches_oracle_fp64():
    """turbompc_solver.py:587-612 / 620-640 on the GPU: gradients w.r.t. x0,
    the control weights and slack_penalization_weight, with a cotangent on the
    slacks too."""
    B, N, admm, pcg = 3, 12, 200, 20
    prog64, p64 = _slack_problem(F64, "cpu", B, N)
    s64 = TurboMPCSolver(prog64, _fixed(1, admm, pcg))
    g64 = s64.initial_guess(p64)
    cfg = _ocfg(admm, pcg, use_slack=True)
    osols = [sr.solve(_oracle_ocp_lin(prog64, p64, b), g64.states[b], g64.controls[b], cfg, 1) for b in range(B)]
    assert any((o.active_lower | o.active_upper).any() for o in osols)
    prog, params = _slack_problem(F64, "cuda", B, N)
    s = TurboMPCSolver(prog, _fixed(1, admm, pcg), forward_backend="b200", backward_backend="b200")
    x0 = params["initial_state"].detach().clone().requires_grad_(True)
    wu = params["weights_penalization_control_squared"].detach().clone().requires_grad_(True)
    sw = params["slack_penalization_weight"].detach().clone().requires_grad_(True)
    sol = s.solve(s.initial_guess(params), params, {"initial_state": x0, "weights_penalization_control_squared": wu,
                                                     "slack_penalization_weight": sw})
    _check_solution(sol, osols, F64, "slack forward")
    rng = np.random.default_rng(5)
    Ws, Wc = rng.normal(size=(B, N + 1, 4)), rng.normal(size=(B, N + 1, 2))
    Wsl = rng.normal(size=(B, N + 1, sol.slack.shape[-1]))
    tt = lambda a: torch.as_tensor(a, dtype=F64, device="cuda")
    loss = (sol.states * tt(Ws)).sum() + (sol.controls * tt(Wc)).sum() + (sol.slack * tt(Wsl)).sum()
    gx0, gwu, gsw = torch.autograd.grad(loss, [x0, wu, sw])
    want = {}
    for b, o in enumerate(osols):
        g, _ = sr.vjp(_oracle_ocp_lin(prog64, p64, b), o, Ws[b], Wc[b],
                      weight_keys=(("weights_penalization_control_squared",),), dl_dslack=Wsl[b])
        want.setdefault("x0", []).append(g["initial_state"])
        want["wu"] = want.get("wu", 0.0) + g[("weights_penalization_control_squared",)]
        want["sw"] = want.get("sw", 0.0) + g["slack_penalization_weight"]
    assert rel_err(gx0.cpu().numpy(), np.stack(want["x0"])) < 1e-6
    assert rel_err(gwu.cpu().numpy(), want["wu"]) < 1e-6
    assert rel_err(gsw.cpu().numpy(), np.asarray(want["sw"])) < 1e-6


def _oracle_ocp_lin(prog, params, b):
    return sr.OCP("linear", 4, 2, sr.problem_params(params, b), use_slack=True, eps_abs=EPS_KKT, eps_rel=EPS_KKT)


def _rescaled_quadrotor(batch, N, dtype, device):
    from tests.test_sqp_oracle import rescaled
    from turbompc_b200.dynamics import Quadrotor12Dynamics
    from turbompc_b200.problems.ocp import OptimalControlProblem
    _, p = _make("quadrotor", batch, N, dtype, device)
    p = {k: (v.to(dtype) if isinstance(v, torch.Tensor) and v.is_floating_point() else v)
         for k, v in rescaled(p, 12, 4).items()}
    p = {k: (v.to(device) if isinstance(v, torch.Tensor) else v) for k, v in p.items()}
    p["initial_control"] = torch.tensor([2.0, 2.5, 2.4, 2.6], dtype=dtype, device=device)
    return OptimalControlProblem(Quadrotor12Dynamics(), p), p


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_rescaled_variables_and_fixed_initial_control_match_oracle(dtype):
    """rescale_optimization_variables + constrain_initial_control
    (optimal_control_problem.py:284-325, 914-980): column-scaled QPs with
    row-scaled constraints and n0 = n initial rows, solved in scaled
    coordinates and unscaled after each ADMM solve (turbompc_solver.py:1582)."""
    B, N, sqp, admm, pcg = 3, 20, 3, 30, 30
    prog64, p64 = _rescaled_quadrotor(B, N, F64, "cpu")
    s64 = TurboMPCSolver(prog64, _fixed(sqp, admm, pcg))
    g64 = s64.initial_guess(p64)
    cfg = _ocfg(admm, pcg)
    osols = [sr.solve(_oracle_ocp("quadrotor", prog64, p64, b), g64.states[b], g64.controls[b], cfg, sqp)
             for b in range(B)]
    prog, params = _rescaled_quadrotor(B, N, dtype, "cuda")
    s = TurboMPCSolver(prog, _fixed(sqp, admm, pcg), forward_backend="b200")
    sol = s.solve(s.initial_guess(params), params)
    _check_solution(sol, osols, dtype, "rescaled + fixed initial control")
    # the fixed-count ADMM meets the initial-control rows to ~1e-4
    np.testing.assert_allclose(sol.controls[:, 0].cpu().numpy(), np.tile([2.0, 2.5, 2.4, 2.6], (B, 1)), atol=5e-3)
    if dtype == torch.float64:
        x0 = params["initial_state"].detach().clone().requires_grad_(True)
        u0 = params["initial_control"].detach().clone().requires_grad_(True)
        wx = params["weights_penalization_reference_state_trajectory"].detach().clone().requires_grad_(True)
        sol = s.solve(s.initial_guess(params), params, {"initial_state": x0, "initial_control": u0,
                                                         "weights_penalization_reference_state_trajectory": wx})
        rng = np.random.default_rng(8)
        Ws, Wc = rng.normal(size=(B, N + 1, 12)), rng.normal(size=(B, N + 1, 4))
        tt = lambda a: torch.as_tensor(a, dtype=dtype, device="cuda")
        loss = (sol.states * tt(Ws)).sum() + (sol.controls * tt(Wc)).sum()
        gx0, gu0, gwx = torch.autograd.grad(loss, [x0, u0, wx])
        want = {"x0": [], "u0": 0.0, "wx": 0.0}
        for b in range(B):
            g, _ = sr.vjp(_oracle_ocp("quadrotor", prog64, p64, b), osols[b], Ws[b], Wc[b],
                          weight_keys=(("weights_penalization_reference_state_trajectory",),))
            want["x0"].append(g["initial_state"])
            want["u0"] = want["u0"] + g["initial_control"]
            want["wx"] = want["wx"] + g[("weights_penalization_reference_state_trajectory",)]
        assert rel_err(gx0.cpu().numpy(), np.stack(want["x0"])) < 1e-6
        assert rel_err(gu0.cpu().numpy(), want["u0"]) < 1e-6
        assert rel_err(gwx.cpu().numpy(), want["wx"]) < 1e-6
