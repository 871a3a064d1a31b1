"""Differentiable solve: the role of jax.custom_vjp in
turbompc/solvers/turbompc_solver.py:1020-1096.

Forward: the SQP solve.  Backward (turbompc_solver.py:1052-1093):
  1. backward QP at the solution (turbompc_solver.py:544-618): cost/dynamics
     blocks at (states, controls), optionally D += lambda^T Hess f + mu^T Hess g
     (use_full_hessian), c0 = c = 0, G_active = (lower - upper) * G,
     q = -[dL/dstates, dL/dcontrols];
  2. the adjoint KKT solve on the GPU (tmpc_adjoint_kkt_solve_*) -> dz,
     equality multipliers y_eq_lin, inequality multipliers y_ineq_lin;
  3. mixed derivatives (turbompc_solver.py:781-966):
       dL/dtheta = -d/dtheta [ grad_z(f + y_eq*.g + y_ineq*.h) . dz
                               + g . y_eq_lin + h . y_ineq_lin ]
     with y_eq* / y_ineq* the forward multipliers (y_ineq* = -(lower - upper) y_g),
     g the equality constraints and h = lower (g - l) + upper (u - g) the active
     inequalities, evaluated by PyTorch autograd at the solution.
With soft (slack) constraints the active rows are folded into the adjoint QP
(turbompc_solver.py:587-605) and their multipliers, and the cotangent of
slack_penalization_weight, are recovered after the solve (:620-640).
theta ranges over the tensors in ``weights`` (and ``initial_state``) that
require grad; the initial-state cotangent equals the x0-row multipliers.
"""
from __future__ import annotations

from typing import Any, Dict, List, Tuple

import torch

from . import ops
from .qp_data import QPCostBlocks, QPData, QPEqualityBlocks, QPInequalityBlocks


def _leaves(weights: Dict[str, Any], params: Dict[str, Any]) -> List[Tuple[Tuple[str, ...], torch.Tensor]]:
    out = []

    def walk(prefix, d):
        for k, v in d.items():
            if isinstance(v, dict):
                walk(prefix + (k,), v)
            elif isinstance(v, torch.Tensor) and v.requires_grad:
                out.append((prefix + (k,), v))

    walk((), weights or {})
    x0 = params.get("initial_state")
    if isinstance(x0, torch.Tensor) and x0.requires_grad and ("initial_state",) not in [p for p, _ in out]:
        out.append((("initial_state",), x0))
    return out


def _replace(params: Dict[str, Any], path: Tuple[str, ...], value) -> Dict[str, Any]:
    p = dict(params)
    if len(path) == 1:
        p[path[0]] = value
    else:
        p[path[0]] = _replace(dict(p.get(path[0]) or {}), path[1:], value)
    return p


def _detach_params(params):
    out = {}
    for k, v in params.items():
        if isinstance(v, dict):
            out[k] = _detach_params(v)
        elif isinstance(v, torch.Tensor):
            out[k] = v.detach()
        else:
            out[k] = v
    return out


def backward_qp(solver, sol, params, dl_dstates, dl_dcontrols, dl_dslack=None):
    """turbompc_solver.py:544-618.  Returns (the QP the adjoint KKT solve
    takes, G_active = sign * G).  With soft (slack) constraints the active
    rows leave the KKT system: D += gamma G_act^T G_act and
    q = -(dL/dz - G_act^T dL/dslack) (turbompc_solver.py:587-605)."""
    prog = solver.program
    kkt = sol.kkt_state
    # true (unscaled) variables: cotangents are taken w.r.t. them; the
    # problem's row scaling of the constraints stays (turbompc_solver.py:553-560)
    qp = solver._build_qp_data(kkt.states, kkt.controls, params, apply_variable_scaling=False)
    D = qp.cost.D
    if solver._use_full_hessian:
        D = D + prog.get_dynamics_lagrangian_hessian(kkt.states, kkt.controls, params, sol.admm_state.y_f_dyn)
        if qp.m > 0:
            active = (kkt.ineq_active_lower_idx | kkt.ineq_active_upper_idx).to(D.dtype)
            D = D + prog.get_inequality_lagrangian_hessian(kkt.states, kkt.controls, params,
                                                           active * sol.admm_state.y_g)
    sign = kkt.ineq_active_lower_idx.to(D.dtype) - kkt.ineq_active_upper_idx.to(D.dtype)
    G = (qp.ineq.G * sign[..., None]).contiguous()
    dl = torch.cat([dl_dstates, dl_dcontrols], -1).to(D.dtype)
    eq = QPEqualityBlocks(qp.eq.A0, qp.eq.A_minus, qp.eq.A_plus, torch.zeros_like(qp.eq.c0),
                          torch.zeros_like(qp.eq.c))
    if qp.ineq.use_slack_variables and qp.m > 0:
        gamma = qp.ineq.slack_penalization_weight.to(D.dtype)
        if dl_dslack is None:
            dl_dslack = torch.zeros_like(sol.slack)
        D = D + gamma[:, None, None, None] * torch.einsum("btki,btkj->btij", G, G)
        q = -(dl - torch.einsum("btki,btk->bti", G, dl_dslack.to(D.dtype)))
        Nb, T, n = q.shape
        empty = torch.zeros(Nb, T, 0, dtype=D.dtype, device=D.device)
        ineq = QPInequalityBlocks(torch.zeros(Nb, T, 0, n, dtype=D.dtype, device=D.device), empty, empty.clone(),
                                  qp.ineq.slack_penalization_weight, False)
        return QPData(QPCostBlocks(D.contiguous(), qp.cost.E, q.contiguous()), eq, ineq), G
    return QPData(QPCostBlocks(D.contiguous(), qp.cost.E, (-dl).contiguous()), eq,
                  QPInequalityBlocks(G, torch.zeros_like(qp.ineq.l), torch.zeros_like(qp.ineq.u),
                                     qp.ineq.slack_penalization_weight, False)), G


class _SolveFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, solver, sol, params, paths, *leaf_values):
        ctx.solver, ctx.sol, ctx.params, ctx.paths = solver, sol, params, paths
        ctx.saved_leaf_values = [v.detach() for v in leaf_values]
        return sol.states.clone(), sol.controls.clone(), sol.slack.clone()

    @staticmethod
    def backward(ctx, g_states, g_controls, g_slack):
        solver, sol, params, paths = ctx.solver, ctx.sol, ctx.params, ctx.paths
        prog = solver.program
        kkt = sol.kkt_state
        dt = sol.states.dtype
        if g_states is None:
            g_states = torch.zeros_like(sol.states)
        if g_controls is None:
            g_controls = torch.zeros_like(sol.controls)
        m = sol.slack.shape[-1]
        soft = prog.use_slack_variables and m > 0
        if g_slack is None:
            g_slack = torch.zeros_like(sol.slack)
        with torch.no_grad():
            bq, G_act = backward_qp(solver, sol, params, g_states.to(dt), g_controls.to(dt), g_slack.to(dt))
            # The adjoint KKT system is solved in float64 whatever the solve's
            # precision: its condition number amplifies float32 rounding into
            # ~1e-3 relative errors in the multipliers (the x0 cotangent among
            # them), while the float32 forward solution itself is good to
            # ~1e-4.  One factorisation per problem, so the cost is small.
            dz, mult, status = ops.adjoint_kkt_solve(bq.map(
                lambda a: a.to(torch.float64) if a.is_floating_point() else a))
            dz, mult = dz.to(dt), mult.to(dt)
        nx = prog.num_state_variables
        Nb, T = sol.states.shape[0], sol.states.shape[1]
        n0 = bq.n0
        n_eq = n0 + (T - 1) * nx
        # equality_constraints orders its rows [x0, dynamics, u0]; the KKT
        # system orders them [A0 rows (x0 then u0), dynamics]
        # (turbompc_solver.py:736-744)
        y_eq_lin = torch.cat([mult[:, :nx], mult[:, n0:n_eq], mult[:, nx:n0]], 1)
        st = sol.admm_state
        lo_m, up_m = kkt.ineq_active_lower_idx.to(dt), kkt.ineq_active_upper_idx.to(dt)
        sign = lo_m - up_m
        dL_dgamma = None
        if soft:
            # turbompc_solver.py:620-640: the active-row multipliers and the
            # slack-weight cotangent from the adjoint step.
            act = torch.maximum(lo_m, up_m)
            g_dx = torch.einsum("btki,bti->btk", G_act, dz)
            gamma = sol_gamma(solver, params, Nb, dt, dz.device)
            y_ineq_lin = g_slack.to(dt) * act + gamma[:, None, None] * g_dx
            dL_dgamma = (sign * st.xi_g * act * g_dx).sum((-1, -2))
        else:
            y_ineq_lin = mult[:, n_eq:].reshape(Nb, T, m)
        y_eq_star = torch.cat([st.y_f_0[:, :nx], st.y_f_dyn.reshape(Nb, -1), st.y_f_0[:, nx:]], 1)
        y_ineq_star = -sign * st.y_g

        with torch.enable_grad():
            leaves = [torch.nn.Parameter(v.detach().clone()) for v in ctx.saved_leaf_values]
            p = params
            for path, leaf in zip(paths, leaves):
                p = _replace(p, path, leaf)
            xs = kkt.states.detach().clone().requires_grad_(True)
            us = kkt.controls.detach().clone().requires_grad_(True)

            def h_fn(x, u):
                g, l, uu = prog.inequality_values(x, u, p)
                return lo_m * (g - l) + up_m * (uu - g)

            F = prog.cost(xs, us, p).sum() + (y_eq_star * prog.equality_constraints(xs, us, p)).sum()
            if m > 0:
                F = F + (y_ineq_star * h_fn(xs, us)).sum()
            gx, gu = torch.autograd.grad(F, (xs, us), create_graph=True)
            phi = (gx * dz[..., :nx]).sum() + (gu * dz[..., nx:]).sum()
            phi = phi + (prog.equality_constraints(xs, us, p) * y_eq_lin).sum()
            if m > 0:
                phi = phi + (h_fn(xs, us) * y_ineq_lin).sum()
            grads = torch.autograd.grad(phi, leaves, allow_unused=True)
        out = [None if g is None else -g for g in grads]
        for i, path in enumerate(paths):
            if path == ("slack_penalization_weight",) and dL_dgamma is not None:
                leaf = ctx.saved_leaf_values[i]
                out[i] = (dL_dgamma.sum() if leaf.numel() == 1 else dL_dgamma).reshape(leaf.shape).to(leaf.dtype)
        return (None, None, None, None, *out)


def sol_gamma(solver, params, Nb, dtype, device):
    """The slack penalty weight per problem (Nb,), as the QP carries it."""
    sw = params.get("slack_penalization_weight", 0.0)
    return torch.as_tensor(sw, dtype=dtype, device=device).expand(Nb)


def make_differentiable_solve(solver):
    def solve(initial_guess, problem_params, weights=None):
        params = solver.make_params_with_weights(weights or {}, problem_params)
        leaves = _leaves(weights or {}, params) if torch.is_grad_enabled() else []
        pdet = _detach_params(params)
        sol = solver._solve_impl(initial_guess.states.detach(), initial_guess.controls.detach(), pdet,
                                 initial_guess.admm_state)
        if not leaves:
            return sol
        paths = [p for p, _ in leaves]
        vals = [v for _, v in leaves]
        states, controls, slack = _SolveFn.apply(solver, sol, pdet, paths, *vals)
        return sol._replace(states=states, controls=controls, slack=slack)

    return solve
