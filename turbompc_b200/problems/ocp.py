"""Batched quadratic-tracking optimal control problem and its linearisation
into stage-blocked QP data (turbompc/problems/optimal_control_problem.py).

Everything is batched over a leading problem axis ``Nb``:
    states (Nb, T, nx), controls (Nb, T, nu), T = horizon + 1.
Problem parameters (``params``) follow the reference's keys; each tensor is
broadcast against (Nb, T, dim) (so a (dim,) weight is shared by every problem
and stage, an (Nb, dim) tensor is per problem, an (Nb, T, dim) tensor per
problem and stage).  Required keys:

    horizon, discretization_resolution, discretization_scheme,
    initial_state (Nb, nx), initial_guess_final_state (Nb, nx) or (nx,),
    reference_state_trajectory, reference_control_trajectory,
    weights_penalization_reference_state_trajectory,
    weights_penalization_final_state, weights_penalization_control_squared,
    weights_penalization_control_rate ((nu,) or (nu, nu)),
    penalize_control_reference (bool)
Optional: state_min_bounds / state_max_bounds / control_min_bounds /
control_max_bounds, weights_linear_penalization_final_state,
dynamics_state_dot_params (dict of tensors broadcast against (Nb, N, ...)),
use_slack_variables, slack_penalization_weight,
rescale_optimization_variables with state_rescaling_min / _max (nx,) and
control_rescaling_min / _max (nu,) (optimal_control_problem.py:284-325),
constrain_initial_control with initial_control ((nu,) or (Nb, nu);
optimal_control_problem.py:914-980).

With rescaling, the constraint rows this class returns are row-scaled as the
reference's are (dynamics and initial rows by 1 / state_diff, the initial
control rows by 1 / control_diff, box rows by 1 / their variable's scale,
obstacle rows by 1 / mean(state_diff[:dim])); the solver then applies the
column scaling z = diag(state_diff, control_diff) z_hat (qp_data.py:178-210).
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from ..dynamics.integrators import DiscretizationScheme, predict_next_state

REQUIRED = ("horizon", "discretization_resolution", "discretization_scheme", "initial_state",
            "reference_state_trajectory", "reference_control_trajectory",
            "weights_penalization_reference_state_trajectory", "weights_penalization_final_state",
            "weights_penalization_control_squared", "weights_penalization_control_rate")


def _t(x, like: torch.Tensor):
    return torch.as_tensor(x, dtype=like.dtype, device=like.device)


def _bt(w: torch.Tensor, Nb: int, T: int, d: int) -> torch.Tensor:
    """Broadcast a (d,), (Nb, d) or (Nb, T, d) weight to (Nb, T, d)."""
    if w.dim() == 2:
        w = w[:, None, :]
    return w.expand(Nb, T, d)


class OptimalControlProblem:
    """Quadratic tracking OCP (optimal_control_problem.py:123-1332), batched."""

    def __init__(self, dynamics, params: Dict[str, Any]):
        missing = [k for k in REQUIRED if k not in params]
        if missing:
            raise KeyError(f"[OptimalControlProblem] missing params: {missing}")
        self._dynamics = dynamics
        self._params = dict(params)
        self._scheme = DiscretizationScheme(int(params["discretization_scheme"]))
        if self._scheme == DiscretizationScheme.IMPLICIT:
            raise NotImplementedError("implicit trapezoid integration is not supported by the b200 backend")
        self._use_slack = bool(params.get("use_slack_variables", False))
        self._penalize_control_reference = bool(params.get("penalize_control_reference", False))
        self._rescale = bool(params.get("rescale_optimization_variables", False))
        self._constrain_u0 = bool(params.get("constrain_initial_control", False))
        if self._constrain_u0 and "initial_control" not in params:
            raise ValueError("initial_control must be provided when constrain_initial_control is True.")
        if self._rescale:
            self.rescaling(params, torch.zeros(1, dtype=torch.float64))  # shape checks
        self._set_active_bounds(params)

    # ------------------------------------------------------------------ sizes
    @property
    def dynamics(self):
        return self._dynamics

    @property
    def params(self) -> Dict[str, Any]:
        return self._params

    @property
    def horizon(self) -> int:
        return int(self._params["horizon"])

    @property
    def num_state_variables(self) -> int:
        return self._dynamics.num_states

    @property
    def num_control_variables(self) -> int:
        return self._dynamics.num_controls

    @property
    def use_slack_variables(self) -> bool:
        return self._use_slack

    @property
    def constrain_initial_control(self) -> bool:
        return self._constrain_u0

    @property
    def rescale_optimization_variables(self) -> bool:
        return self._rescale

    @property
    def num_initial_equalities(self) -> int:
        """Rows of A0: nx, or nx + nu with a fixed initial control."""
        return self.num_state_variables + (self.num_control_variables if self._constrain_u0 else 0)

    # ------------------------------------------------------------ rescaling
    def rescaling(self, params, like):
        """(state_diff (nx,), control_diff (nu,)) with x = state_diff * x_hat,
        u = control_diff * u_hat; ones without rescaling
        (optimal_control_problem.py:284-325)."""
        nx, nu = self.num_state_variables, self.num_control_variables
        if not self._rescale:
            return (torch.ones(nx, dtype=like.dtype, device=like.device),
                    torch.ones(nu, dtype=like.dtype, device=like.device))
        vals = {}
        for k, dim in (("state_rescaling_min", nx), ("state_rescaling_max", nx), ("control_rescaling_min", nu),
                       ("control_rescaling_max", nu)):
            if k not in params:
                raise KeyError(f"{k} is required with rescale_optimization_variables")
            v = _t(params[k], like)
            if tuple(v.shape) != (dim,):
                raise ValueError(f"{k} must have shape ({dim},), got {tuple(v.shape)}")
            vals[k] = v
        return ((vals["state_rescaling_max"] - vals["state_rescaling_min"]) / 2.0,
                (vals["control_rescaling_max"] - vals["control_rescaling_min"]) / 2.0)

    def scale_states_controls(self, states, controls, params):
        sd, cd = self.rescaling(params, states)
        return states / sd, controls / cd

    def unscale_states_controls(self, states, controls, params):
        sd, cd = self.rescaling(params, states)
        return states * sd, controls * cd

    def dynamics_plus_rows(self, params, like, Nb):
        """A_plus = -[I 0] (the coefficient of z_{t+1} in the explicit-scheme
        dynamics rows), row-scaled like A_minus."""
        nx, nu, N = self.num_state_variables, self.num_control_variables, self.horizon
        sd, _ = self.rescaling(params, like)
        Ap = torch.zeros(Nb, N, nx, nx + nu, dtype=like.dtype, device=like.device)
        Ap[..., :nx] = -torch.diag(1.0 / sd)
        return Ap

    @property
    def num_inequality_constraints(self) -> int:
        return int(self._state_mask.sum()) + int(self._control_mask.sum()) + self._num_extra_inequalities()

    def _num_extra_inequalities(self) -> int:
        return 0

    @property
    def state_independent_cost(self) -> bool:
        """True: the tracking cost's blocks (D, E, q) depend on the parameters
        only, not on the linearisation point (subclasses with a nonquadratic
        cost return False)."""
        return True

    @property
    def state_independent_inequalities(self) -> bool:
        """True when the inequality rows (box bounds only) do not depend on
        the linearisation point."""
        return self._num_extra_inequalities() == 0

    # --------------------------------------------------------------- bounds
    def _set_active_bounds(self, params):
        """Active box bounds: any finite entry with |bound| < 1e6 (optimal_control_problem.py:177-186)."""
        nx, nu = self.num_state_variables, self.num_control_variables

        def mask(lo_key, hi_key, dim):
            if lo_key not in params or hi_key not in params:
                return torch.zeros(dim, dtype=torch.bool)
            lo = torch.as_tensor(params[lo_key]).reshape(-1, dim)
            hi = torch.as_tensor(params[hi_key]).reshape(-1, dim)
            return ((lo > -1e6) | (hi < 1e6)).any(dim=0).cpu()

        all4 = all(k in params for k in ("state_min_bounds", "state_max_bounds", "control_min_bounds",
                                         "control_max_bounds"))
        if not all4:  # step_inequality_constraints needs all four (optimal_control_problem.py:433-440)
            self._state_mask = torch.zeros(nx, dtype=torch.bool)
            self._control_mask = torch.zeros(nu, dtype=torch.bool)
        else:
            self._state_mask = mask("state_min_bounds", "state_max_bounds", nx)
            self._control_mask = mask("control_min_bounds", "control_max_bounds", nu)

    # ----------------------------------------------------------- guesses
    def initial_guess(self, params=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Straight-line states from initial_state to initial_guess_final_state
        (+1e-6), controls 1e-6 (optimal_control_problem.py:815-839)."""
        params = params or self._params
        x0 = params["initial_state"]
        xf = _t(params.get("initial_guess_final_state", torch.zeros_like(x0)), x0).expand_as(x0)
        N = self.horizon
        a = torch.arange(N + 1, dtype=x0.dtype, device=x0.device) / N
        states = x0[:, None, :] * (1 - a)[None, :, None] + xf[:, None, :] * a[None, :, None] + 1e-6
        controls = torch.zeros(x0.shape[0], N + 1, self.num_control_variables, dtype=x0.dtype,
                               device=x0.device) + 1e-6
        return states, controls

    # ------------------------------------------------------------- dynamics
    def _dyn_params(self, params, like):
        dp = params.get("dynamics_state_dot_params") or {}
        return {k: (_t(v, like) if not isinstance(v, (int, float)) else v) for k, v in dp.items()}

    def next_states(self, states, controls, params):
        dt = float(params["discretization_resolution"])
        N = self.horizon
        return predict_next_state(self._dynamics, dt, self._scheme, self._dyn_params(params, states),
                                  states[:, :N], controls[:, :N])

    def linearized_dynamics_rows(self, states, controls, params):
        """(A_minus (Nb, N, nx, n), c (Nb, N, nx)) of the QP: from the CUDA
        linearisation kernel for a built-in model with scalar parameters on a
        CUDA device, else from get_dynamics_linearized_matrices (forward-mode
        autodiff of the integrator in PyTorch, any dynamics)."""
        cm = getattr(self._dynamics, "cuda_model", None)
        spec = cm(self._dyn_params(params, states)) if (cm is not None and states.is_cuda) else None
        if spec is not None and self._scheme in (DiscretizationScheme.EULER, DiscretizationScheme.MIDPOINT,
                                                 DiscretizationScheme.RUNGEKUTTA4):
            from .. import ops
            Am, c = ops.linearize_dynamics(spec[0], spec[1], int(self._scheme),
                                           float(params["discretization_resolution"]), states, controls)
            if self._rescale:
                rs = 1.0 / self.rescaling(params, states)[0]
                Am, c = (Am * rs[:, None]).contiguous(), (c * rs).contiguous()
            return Am, c
        _, _, As, Bs, Cs = self.get_dynamics_linearized_matrices(states, controls, params)
        return torch.cat([As, Bs], dim=-1).contiguous(), Cs[:, 1:].contiguous()

    def get_dynamics_linearized_matrices(self, states, controls, params):
        """Explicit integrators (optimal_control_problem.py:1217-1272):
        x_{t+1} = f(x_t, u_t) ~ f(y, v) + A (x - y) + B (u - v) gives
        -I x_{t+1} + A x_t + B u_t = -f(y, v) + A y + B v.
        Returns (As_next, Bs_next, As, Bs, Cs) with Cs = [x0, c_1..c_N]."""
        nx, nu, N = self.num_state_variables, self.num_control_variables, self.horizon
        dt = float(params["discretization_resolution"])
        dp = self._dyn_params(params, states)
        xs, us = states[:, :N], controls[:, :N]

        def f(xu):
            return predict_next_state(self._dynamics, dt, self._scheme, dp, xu[..., :nx], xu[..., nx:])

        xu = torch.cat([xs, us], dim=-1)
        n = nx + nu
        basis = torch.eye(n, dtype=xu.dtype, device=xu.device)[:, None, None, :].expand(n, *xu.shape)
        val, jac = torch.func.vmap(lambda v: torch.func.jvp(f, (xu,), (v,)), out_dims=(None, 0))(basis)
        J = jac.permute(1, 2, 3, 0)  # (Nb, N, nx, n)
        As, Bs = J[..., :nx], J[..., nx:]
        c = -val + torch.einsum("btij,btj->bti", J, xu)
        Cs = torch.cat([params["initial_state"][:, None, :], c], dim=1)
        eye = torch.eye(nx, dtype=states.dtype, device=states.device)
        As_next = (-eye).expand(states.shape[0], N, nx, nx)
        Bs_next = torch.zeros_like(Bs)
        if self._rescale:  # row scaling 1 / state_diff (optimal_control_problem.py:1322-1331)
            rs = 1.0 / self.rescaling(params, states)[0]
            As_next, As, Bs, Cs = As_next * rs[:, None], As * rs[:, None], Bs * rs[:, None], Cs * rs
        return As_next, Bs_next, As, Bs, Cs

    # ----------------------------------------------------------------- cost
    def _weights(self, params, like):
        wx = _t(params["weights_penalization_reference_state_trajectory"], like)
        wu = _t(params["weights_penalization_control_squared"], like)
        wf = _t(params["weights_penalization_final_state"], like)
        rd = _t(params["weights_penalization_control_rate"], like)
        nu = self.num_control_variables
        if rd.shape[-1] == nu and (rd.dim() == 1 or rd.shape[-2:] != (nu, nu)):
            rd = torch.diag_embed(rd)
        return wx, wu, wf, rd

    def get_cost_linearized_blocks(self, states, controls, params):
        """D, E, q of the tracking cost (optimal_control_problem.py:1068-1174)
        in closed form: stage cost sum wx (x - xr)^2 + wu (u - ur)^2
        + 0.5 du^T Rd du (du = u_{t+1} - u_t); terminal (wx + wf)(x - xr)^2 +
        wlin x + wu (u - ur)^2.  With H_minus / H_plus / H_pm the blocks of the
        pairwise stage Hessian, D_0 = H_minus, D_t = H_plus + H_minus,
        D_N = H_plus + H_term, E_t = H_pm and q = gradient - Hessian z."""
        Nb, T, nx = states.shape
        nu = controls.shape[-1]
        n = nx + nu
        N = T - 1
        like = states
        wx, wu, wf, rd = self._weights(params, like)
        xr = _t(params["reference_state_trajectory"], like).expand(Nb, T, nx)
        ur = _t(params["reference_control_trajectory"], like).expand(Nb, T, nu)
        if not self._penalize_control_reference:
            ur = torch.zeros_like(ur)
        wx_t = _bt(wx, Nb, T, nx)
        wu_t = _bt(wu, Nb, T, nu)
        wf_b = wf.expand(Nb, nx)
        diag = torch.cat([2 * wx_t, 2 * wu_t], dim=-1).clone()
        diag[:, N, :nx] = 2 * (wx_t[:, N] + wf_b)
        D = torch.diag_embed(diag)
        rdb = rd.expand(Nb, N, nu, nu) if rd.dim() < 4 else rd
        # control-rate Hessian: +Rd on (u_t, u_t) for t < N, +Rd on (u_{t+1}, u_{t+1}), -Rd across.
        D[:, :N, nx:, nx:] += rdb
        D[:, 1:, nx:, nx:] += rdb
        E = torch.zeros(Nb, N, n, n, dtype=like.dtype, device=like.device)
        E[:, :, nx:, nx:] = -rdb
        q = torch.cat([-2 * wx_t * xr, -2 * wu_t * ur], dim=-1).clone()
        q[:, N, :nx] = -2 * (wx_t[:, N] + wf_b) * xr[:, N]
        if "weights_linear_penalization_final_state" in params:
            q[:, N, :nx] += _t(params["weights_linear_penalization_final_state"], like)
        return D, E, q

    def cost(self, states, controls, params):
        """Total tracking cost per problem (optimal_control_problem.py:1030-1066)."""
        Nb, T, nx = states.shape
        N = T - 1
        wx, wu, wf, rd = self._weights(params, states)
        xr = _t(params["reference_state_trajectory"], states).expand_as(states)
        ur = _t(params["reference_control_trajectory"], states).expand_as(controls)
        if not self._penalize_control_reference:
            ur = torch.zeros_like(ur)
        nu = controls.shape[-1]
        wx_t, wu_t = _bt(wx, Nb, T, nx), _bt(wu, Nb, T, nu)
        c = (wx_t[:, :N] * (states[:, :N] - xr[:, :N]) ** 2).sum((-1, -2))
        c = c + (wu_t * (controls - ur) ** 2).sum((-1, -2))
        du = controls[:, 1:] - controls[:, :-1]
        rdb = rd.expand(Nb, N, nu, nu) if rd.dim() < 4 else rd
        c = c + 0.5 * torch.einsum("bti,btij,btj->b", du, rdb, du)
        c = c + ((wx_t[:, N] + wf.expand(Nb, nx)) * (states[:, N] - xr[:, N]) ** 2).sum(-1)
        if "weights_linear_penalization_final_state" in params:
            c = c + (_t(params["weights_linear_penalization_final_state"], states) * states[:, N]).sum(-1)
        return c

    # ---------------------------------------------------------- inequalities
    def _box(self, params, like, Nb, T):
        nx, nu = self.num_state_variables, self.num_control_variables
        sm, cm = self._state_mask.to(like.device), self._control_mask.to(like.device)

        def b(key, dim):
            return _t(params[key], like).expand(Nb, T, dim) if key in params else None

        if int(sm.sum()) + int(cm.sum()) == 0:
            z = torch.zeros(Nb, T, 0, dtype=like.dtype, device=like.device)
            return z, z
        lo = torch.cat([b("state_min_bounds", nx)[..., sm], b("control_min_bounds", nu)[..., cm]], dim=-1)
        hi = torch.cat([b("state_max_bounds", nx)[..., sm], b("control_max_bounds", nu)[..., cm]], dim=-1)
        return lo, hi

    def get_inequalities_linearized_matrices(self, states, controls, params):
        """Box rows (selection of the active entries; optimal_control_problem.py:413-471)
        plus the linearisation of any extra constraints (``_extra_inequalities``):
        G = dg/dz, l = l - (g - G z), u = u - (g - G z)."""
        Nb, T, nx = states.shape
        nu = controls.shape[-1]
        n = nx + nu
        sel = torch.cat([torch.eye(nx, dtype=states.dtype, device=states.device)[self._state_mask.to(states.device)],
                         torch.zeros(int(self._state_mask.sum()), nu, dtype=states.dtype, device=states.device)], 1)
        selu = torch.cat([torch.zeros(int(self._control_mask.sum()), nx, dtype=states.dtype, device=states.device),
                          torch.eye(nu, dtype=states.dtype, device=states.device)[self._control_mask.to(states.device)]],
                         1)
        Gbox = torch.cat([sel, selu], 0).expand(Nb, T, -1, n)
        lo, hi = self._box(params, states, Nb, T)
        if self._rescale:  # g / scale (optimal_control_problem.py:460-469)
            bs = self._box_scale(params, states)
            Gbox, lo, hi = Gbox / bs[:, None], lo / bs, hi / bs
        extra = self._extra_inequalities_linearized(states, controls, params)
        if extra is None:
            return Gbox.contiguous(), lo.contiguous(), hi.contiguous()
        Ge, le, ue = extra
        if self._rescale:
            es = self._extra_row_scale(params, states)
            Ge, le, ue = Ge * es, le * es, ue * es
        return (torch.cat([Gbox, Ge], 2).contiguous(), torch.cat([lo, le], 2).contiguous(),
                torch.cat([hi, ue], 2).contiguous())

    def _extra_inequalities_linearized(self, states, controls, params):
        return None

    def _box_scale(self, params, like):
        """Scale of each active box row (its variable's state / control diff)."""
        sd, cd = self.rescaling(params, like)
        return torch.cat([sd[self._state_mask.to(like.device)], cd[self._control_mask.to(like.device)]])

    def _extra_row_scale(self, params, like):
        """Row scale of the extra (nonlinear) inequality rows under rescaling."""
        return 1.0

    # ------------------------------------- nonlinear constraint functions (backward)
    def equality_constraints(self, states, controls, params):
        """[x_0 - initial_state, f(x_t, u_t) - x_{t+1}] flattened per problem,
        (Nb, n0 + N*nx) (optimal_control_problem.py:841-912, explicit schemes);
        its Jacobian is the QP's [A0; A_minus/A_plus] rows."""
        x0c = states[:, 0] - _t(params["initial_state"], states)
        dyn = self.next_states(states, controls, params) - states[:, 1:]
        sd, cd = self.rescaling(params, states)
        rows = torch.cat([x0c[:, None], dyn], 1) / sd
        out = [rows.reshape(states.shape[0], -1)]
        if self._constrain_u0:  # appended last, as optimal_control_problem.py:895-910
            out.append((controls[:, 0] - _t(params["initial_control"], states)) / cd)
        return torch.cat(out, dim=1)

    def inequality_values(self, states, controls, params):
        """Nonlinear g(x, u) with its bounds, each (Nb, T, m), in the row order of
        get_inequalities_linearized_matrices."""
        Nb, T, _ = states.shape
        z = torch.cat([states, controls], -1)
        nx = self.num_state_variables
        sm, cm = self._state_mask.to(states.device), self._control_mask.to(states.device)
        g = torch.cat([states[..., sm], controls[..., cm]], -1)
        lo, hi = self._box(params, states, Nb, T)
        if self._rescale:
            bs = self._box_scale(params, states)
            g, lo, hi = g / bs, lo / bs, hi / bs
        extra = self._extra_inequality_values(states, controls, params)
        if extra is not None:
            es = self._extra_row_scale(params, states) if self._rescale else 1.0
            g = torch.cat([g, extra[0] * es], -1)
            lo = torch.cat([lo, extra[1] * es], -1)
            hi = torch.cat([hi, extra[2] * es], -1)
        del z, nx
        return g, lo, hi

    def _extra_inequality_values(self, states, controls, params):
        return None

    def _stagewise_hessian(self, fn, z):
        """Per-stage Hessians of sum(fn(z)) where fn is separable over (Nb, T):
        z (Nb, T', n) -> (Nb, T', n, n), one forward-over-reverse pass per
        column (the stage blocks are independent, so one tangent serves all)."""
        n = z.shape[-1]

        def grad_fn(zz):
            with torch.enable_grad():
                zz = zz.detach().requires_grad_(True) if not zz.requires_grad else zz
                return torch.autograd.grad(fn(zz).sum(), zz, create_graph=True)[0]

        cols = []
        for k in range(n):
            v = torch.zeros_like(z)
            v[..., k] = 1.0
            _, hv = torch.func.jvp(lambda zz: torch.func.grad(lambda q: fn(q).sum())(zz), (z,), (v,))
            cols.append(hv)
        del grad_fn
        return torch.stack(cols, dim=-1)

    def get_dynamics_lagrangian_hessian(self, states, controls, params, lambdas):
        """sum_i lambda_{t,i} Hess_{(x,u)} [f(x_t, u_t)]_i for t < N, zero at N
        (optimal_control_problem.py:1334-1442, explicit schemes)."""
        nx = self.num_state_variables
        N = self.horizon
        dt = float(params["discretization_resolution"])
        dp = self._dyn_params(params, states)
        lam = lambdas.detach()

        rs = 1.0 / self.rescaling(params, states)[0]

        def fn(zz):
            return (lam * rs * predict_next_state(self._dynamics, dt, self._scheme, dp, zz[..., :nx],
                                                  zz[..., nx:])).sum(-1)

        z = torch.cat([states[:, :N], controls[:, :N]], -1).detach()
        H = self._stagewise_hessian(fn, z)
        return torch.cat([H, torch.zeros_like(H[:, :1])], dim=1)

    def get_inequality_lagrangian_hessian(self, states, controls, params, mus):
        """sum_i mu_{t,i} Hess_{(x,u)} g_i(x_t, u_t) (optimal_control_problem.py:1444-1481)."""
        nx = self.num_state_variables
        mu = mus.detach()

        def fn(zz):
            g, _, _ = self.inequality_values(zz[..., :nx], zz[..., nx:], params)
            return (mu * g).sum(-1)

        z = torch.cat([states, controls], -1).detach()
        return self._stagewise_hessian(fn, z)

    def get_initial_equality_linearized_matrices(self, params, like):
        """A0 = [I 0], c0 = initial_state, plus [0 I], initial_control with a
        fixed initial control; row-scaled under rescaling
        (optimal_control_problem.py:914-980)."""
        nx, nu = self.num_state_variables, self.num_control_variables
        x0 = _t(params["initial_state"], like)
        Nb = x0.shape[0]
        sd, cd = self.rescaling(params, like)
        A0 = torch.cat([torch.diag(1.0 / sd), torch.zeros(nx, nu, dtype=like.dtype, device=like.device)], 1)
        A0 = A0.expand(Nb, nx, nx + nu)
        c0 = x0 / sd
        if self._constrain_u0:
            Au = torch.cat([torch.zeros(nu, nx, dtype=like.dtype, device=like.device), torch.diag(1.0 / cd)], 1)
            A0 = torch.cat([A0, Au.expand(Nb, nu, nx + nu)], 1)
            u0 = _t(params["initial_control"], like).expand(Nb, nu)
            c0 = torch.cat([c0, u0 / cd], 1)
        return A0.contiguous(), c0.contiguous()


class OptimalControlProblemObstacle(OptimalControlProblem):
    """Spherical obstacles (turbompc/problems/obstacle_avoidance.py:13-52):
    g_k = 1 - ||p - c_k|| / (r_k + 0.001) <= 0 for p = state[:dim].
    params: obstacles_centers (Nb, K, dim), obstacles_radii (Nb, K),
    obstacles_dimension."""

    def _num_extra_inequalities(self) -> int:
        return int(torch.as_tensor(self._params["obstacles_radii"]).shape[-1])

    def _extra_inequality_values(self, states, controls, params):
        dim = int(params["obstacles_dimension"])
        c = _t(params["obstacles_centers"], states)
        r = _t(params["obstacles_radii"], states)
        diff = states[..., :dim][:, :, None, :] - c[:, None, :, :]
        g = 1.0 - diff.norm(dim=-1) / (r[:, None, :] + 0.001)
        return g, torch.full_like(g, -1e9), torch.zeros_like(g)

    def _extra_inequalities_linearized(self, states, controls, params):
        """The obstacle rows: one CUDA kernel (tmpc_obstacle_rows_*) on GPU
        tensors, PyTorch otherwise."""
        dim = int(params["obstacles_dimension"])
        c = _t(params["obstacles_centers"], states)  # (Nb, K, dim)
        r = _t(params["obstacles_radii"], states)  # (Nb, K)
        if states.is_cuda:
            from .. import ops
            # the rescaling row scale is applied by the caller
            return ops.obstacle_rows(states, c, r, dim, states.shape[-1] + controls.shape[-1])
        return self._obstacle_rows_torch(states, controls, c, r, dim)

    def _obstacle_rows_torch(self, states, controls, c, r, dim):
        """The same rows in PyTorch operations (host tensors; the CUDA
        kernel's test reference)."""
        Nb, T, nx = states.shape
        nu = controls.shape[-1]
        p = states[..., :dim]  # (Nb, T, dim)
        diff = p[:, :, None, :] - c[:, None, :, :]  # (Nb, T, K, dim)
        dist = diff.norm(dim=-1).clamp_min(1e-12)
        scale = 1.0 / (r[:, None, :] + 0.001)
        g = 1.0 - dist * scale
        dg = -diff / dist[..., None] * scale[..., None]  # (Nb, T, K, dim)
        K = c.shape[1]
        G = torch.zeros(Nb, T, K, nx + nu, dtype=states.dtype, device=states.device)
        G[..., :dim] = dg
        off = g - (dg * p[:, :, None, :]).sum(-1)
        lo = torch.full_like(g, -1e9) - off
        hi = torch.zeros_like(g) - off
        return G, lo, hi

    def _extra_row_scale(self, params, like):
        """obstacle_avoidance.py:40-45: 1 / mean(state_diff[:dim])."""
        dim = int(params["obstacles_dimension"])
        return 1.0 / self.rescaling(params, like)[0][:dim].mean()
