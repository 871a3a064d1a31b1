"""CPU restatement of TurboMPC's SQP solve, of its QP linearisation and of its
custom-VJP backward pass.

TEST INFRASTRUCTURE ONLY.  Nothing in ``turbompc_b200`` imports this module;
only ``tests/`` use it, as the checker.  It imports nothing from
``turbompc_b200``: the problem functions (dynamics, integrators, stage and
terminal costs, inequality rows) are written again here, per problem, and
every derivative is taken by automatic differentiation exactly where the
reference takes one (torch.func on the CPU in float64 standing in for
jax.grad / jax.hessian / jax.jacfwd).  The ADMM inner solve and the adjoint
KKT solve are the NumPy restatements in ``oracle/admm_ref.py``.

Reference functions restated (paths relative to the reference project root):

  turbompc/dynamics/integrators.py:21-76          predict_next_state (explicit schemes)
  turbompc/problems/optimal_control_problem.py
      :413-471    step_inequality_constraints (box rows, active-bound masks :177-186)
      :580-626    get_inequalities_linearized_matrices
      :841-912    equality_constraints (explicit schemes)
      :914-980    get_initial_equality_linearized_matrices
      :982-1030   stage_cost / terminal_cost
      :1068-1174  get_cost_linearized_blocks (grad / Hessian of the pairwise stage cost)
      :1217-1272  get_dynamics_linearized_matrices (explicit schemes)
      :1334-1442  get_dynamics_lagrangian_hessian (explicit schemes)
      :1444-1481  get_inequality_lagrangian_hessian
  turbompc/problems/obstacle_avoidance.py:16-52   spherical obstacle rows
  turbompc/solvers/turbompc_solver.py
      :269-292    identify_active_inequalities
      :1098-1156  _build_qp_data (no variable rescaling)
      :1158-1225  first-order convergence error
      :1387-1439  _build_kkt_state
      :1519-1760  _solve_impl (per problem, as under jax.vmap)
      :544-618    _build_backward_qp (hard and slack branches)
      :620-640    _recover_slack_active_ineq_gradient
      :706-779    _solve_backward_qp_direct
      :781-860    _compute_mixed_derivatives (jacfwd over the weights)
      :862-880    _forward_multipliers
      :930-966    _assemble_parameter_gradient
      :990-1018   _build_problem_params_cotangent (initial_state cotangent)

The learned stage cost of benchmark configuration 5 (s * w2 . tanh(W1 z + b1)
added to every stage, z = [x, u]) is written through the reference's own
extension point: it is added to ``stage_cost`` for t < N and to
``terminal_cost`` at t = N.

Problems are solved one at a time (a Python loop over the batch stands in for
jax.vmap); the oracle is meant for batches of a few to a few dozen problems.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch
from torch.func import grad, hessian, jacfwd, vmap

from . import admm_ref as ref

F64 = torch.float64
GRAVITY = 9.81

# Keys whose per-problem form carries one leading batch axis (the rank that
# marks a per-problem tensor); everything else is shared by the batch.
_PER_PROBLEM_RANK = {
    "initial_state": 2, "initial_guess_final_state": 2, "initial_control": 2,
    "reference_state_trajectory": 3, "reference_control_trajectory": 3,
    "weights_penalization_reference_state_trajectory": 2, "weights_penalization_control_squared": 2,
    "weights_penalization_final_state": 2, "obstacles_centers": 3, "obstacles_radii": 2,
    "slack_penalization_weight": 1,
}


def _f64(v):
    if isinstance(v, torch.Tensor):
        return v.detach().to("cpu", F64) if not v.requires_grad else v.to("cpu", F64)
    if isinstance(v, np.ndarray):
        return torch.as_tensor(v, dtype=F64)
    return v


def problem_params(params: Dict, b: int) -> Dict:
    """Parameters of problem b of a batched params dict (CPU float64)."""
    out = {}
    for k, v in params.items():
        if isinstance(v, dict):
            out[k] = {kk: _f64(vv) for kk, vv in v.items()}
            continue
        v = _f64(v)
        if isinstance(v, torch.Tensor) and _PER_PROBLEM_RANK.get(k) == v.dim():
            v = v[b]
        out[k] = v
    return out


# ---------------------------------------------------------------------------
# Dynamics and integrators
# ---------------------------------------------------------------------------
def state_dot(model: str, x, u, dp):
    """Continuous dynamics of the models the benchmarks use.

    quadrotor12: 12-state rigid body, state [p, (roll, pitch, yaw), v (world),
      omega (body)], four rotor thrusts, "+" layout, R = Rz(yaw) Ry(pitch) Rx(roll);
      torques (L (f2 - f4), L (f3 - f1), k (f1 - f2 + f3 - f4)); mass, inertia
      (diagonal), arm length L and yaw coefficient k from ``dp`` (defaults 1 kg,
      0.01, 0.1 m, 0.01 m).
    linear: A x + B u (+ b) (turbompc/dynamics/linear_dynamics.py:45-68).
    """
    if model == "linear":
        out = dp["A"] @ x + dp["B"] @ u
        return out + dp["b"] if "b" in dp else out
    if model != "quadrotor12":
        raise ValueError(model)
    m = dp.get("mass", 1.0)
    J = dp.get("inertia", (0.01, 0.01, 0.01))
    Jx, Jy, Jz = J[0], J[1], J[2]
    L = dp.get("arm_length", 0.1)
    k = dp.get("yaw_coefficient", 0.01)
    phi, th, psi = x[3], x[4], x[5]
    wx, wy, wz = x[9], x[10], x[11]
    thrust = (u[0] + u[1] + u[2] + u[3]) / m
    euler_rates = torch.stack([
        wx + torch.sin(phi) * torch.tan(th) * wy + torch.cos(phi) * torch.tan(th) * wz,
        torch.cos(phi) * wy - torch.sin(phi) * wz,
        (torch.sin(phi) * wy + torch.cos(phi) * wz) / torch.cos(th)])
    # third column of Rz(psi) Ry(th) Rx(phi) times the collective thrust
    acc = torch.stack([
        (torch.cos(psi) * torch.sin(th) * torch.cos(phi) + torch.sin(psi) * torch.sin(phi)) * thrust,
        (torch.sin(psi) * torch.sin(th) * torch.cos(phi) - torch.cos(psi) * torch.sin(phi)) * thrust,
        torch.cos(th) * torch.cos(phi) * thrust - GRAVITY])
    tau = torch.stack([L * (u[1] - u[3]), L * (u[2] - u[0]), k * (u[0] - u[1] + u[2] - u[3])])
    wdot = torch.stack([(tau[0] - (Jz - Jy) * wy * wz) / Jx, (tau[1] - (Jx - Jz) * wz * wx) / Jy,
                        (tau[2] - (Jy - Jx) * wx * wy) / Jz])
    return torch.cat([x[6:9], euler_rates, acc, wdot])


def predict_next_state(model, dt, scheme, dp, x, u):
    """turbompc/dynamics/integrators.py:21-76 (Euler 0, midpoint 1, RK4 2)."""
    f = lambda s: state_dot(model, s, u, dp)
    if scheme == 0:
        return x + dt * f(x)
    if scheme == 1:
        return x + dt * f(x + 0.5 * dt * f(x))
    if scheme == 2:
        k1 = f(x)
        k2 = f(x + 0.5 * dt * k1)
        k3 = f(x + 0.5 * dt * k2)
        k4 = f(x + dt * k3)
        return x + (1.0 / 6.0) * (k1 + 2 * k2 + 2 * k3 + k4) * dt
    raise NotImplementedError("implicit integration is not restated")


# ---------------------------------------------------------------------------
# The optimal control problem (one problem)
# ---------------------------------------------------------------------------
@dataclass
class OCP:
    """One problem of the batch: model, sizes, flags and its parameters."""

    model: str
    nx: int
    nu: int
    p: Dict
    obstacles: bool = False
    mlp: bool = False
    use_slack: bool = False
    eps_abs: float = 1e-9
    eps_rel: float = 1e-9
    state_mask: torch.Tensor = field(default=None)
    control_mask: torch.Tensor = field(default=None)

    def __post_init__(self):
        p = self.p
        self.N = int(p["horizon"])
        self.T = self.N + 1
        self.n = self.nx + self.nu
        self.dt = float(p["discretization_resolution"])
        self.scheme = int(p["discretization_scheme"])
        # optimal_control_problem.py:168-171
        self.rescale = bool(p.get("rescale_optimization_variables", False))
        self.constrain_u0 = bool(p.get("constrain_initial_control", False))
        # optimal_control_problem.py:177-186 and :433-440
        keys = ("state_min_bounds", "state_max_bounds", "control_min_bounds", "control_max_bounds")
        if all(k in p for k in keys):
            lo_x, hi_x = p["state_min_bounds"].reshape(-1, self.nx), p["state_max_bounds"].reshape(-1, self.nx)
            lo_u, hi_u = p["control_min_bounds"].reshape(-1, self.nu), p["control_max_bounds"].reshape(-1, self.nu)
            self.state_mask = ((lo_x > -1e6) | (hi_x < 1e6)).any(0)
            self.control_mask = ((lo_u > -1e6) | (hi_u < 1e6)).any(0)
        else:
            self.state_mask = torch.zeros(self.nx, dtype=torch.bool)
            self.control_mask = torch.zeros(self.nu, dtype=torch.bool)

    # ---- rescaling (optimal_control_problem.py:284-349)
    def rescaling(self, p):
        if not self.rescale:
            return torch.ones(self.nx, dtype=F64), torch.ones(self.nu, dtype=F64)
        sd = (p["state_rescaling_max"] - p["state_rescaling_min"]) / 2.0
        cd = (p["control_rescaling_max"] - p["control_rescaling_min"]) / 2.0
        return sd, cd

    # ---- cost (optimal_control_problem.py:982-1030)
    def _refs(self, p):
        T, nx, nu = self.T, self.nx, self.nu
        rx = p["reference_state_trajectory"].expand(T, nx) if p["reference_state_trajectory"].dim() < 2 \
            else p["reference_state_trajectory"]
        ru = p["reference_control_trajectory"]
        ru = ru.expand(T, nu) if ru.dim() < 2 else ru
        if not bool(p.get("penalize_control_reference", False)):
            ru = torch.zeros_like(ru)
        return rx, ru

    def _rate(self, p):
        rd = p["weights_penalization_control_rate"]
        return torch.diag(rd) if rd.dim() == 1 else rd

    def _mlp(self, z, p):
        return p["mlp_scale"] * (p["mlp_w2"] @ torch.tanh(p["mlp_W1"] @ z + p["mlp_b1"]))

    def stage_cost(self, x, u, xn, un, rx, ru, p):
        z = torch.cat([x, u])
        w = torch.cat([p["weights_penalization_reference_state_trajectory"],
                       p["weights_penalization_control_squared"]])
        c = torch.sum(w * (z - torch.cat([rx, ru])) ** 2)
        du = un - u
        c = c + 0.5 * (du @ (self._rate(p) @ du))
        if self.mlp:
            c = c + self._mlp(z, p)
        return c

    def terminal_cost(self, x, u, rx, ru, p):
        w = p["weights_penalization_reference_state_trajectory"] + p["weights_penalization_final_state"]
        c = torch.sum(w * (x - rx) ** 2)
        if "weights_linear_penalization_final_state" in p:
            c = c + torch.sum(p["weights_linear_penalization_final_state"] * x)
        c = c + torch.sum(p["weights_penalization_control_squared"] * (u - ru) ** 2)
        if self.mlp:
            c = c + self._mlp(torch.cat([x, u]), p)
        return c

    def cost(self, X, U, p):
        rx, ru = self._refs(p)
        sc = vmap(lambda x, u, xn, un, a, b: self.stage_cost(x, u, xn, un, a, b, p))(
            X[:-1], U[:-1], X[1:], U[1:], rx[:-1], ru[:-1])
        return sc.sum() + self.terminal_cost(X[-1], U[-1], rx[-1], ru[-1], p)

    def cost_blocks(self, X, U, p):
        """D, E, q (optimal_control_problem.py:1068-1174)."""
        n, N = self.n, self.N
        rx, ru = self._refs(p)
        Z = torch.cat([X, U], -1)
        pairs = torch.cat([Z[:-1], Z[1:]], -1)

        def pair_cost(zz, a, b):
            return self.stage_cost(zz[:self.nx], zz[self.nx:n], zz[n:n + self.nx], zz[n + self.nx:], a, b, p)

        g = vmap(grad(pair_cost))(pairs, rx[:-1], ru[:-1])
        H = vmap(hessian(pair_cost))(pairs, rx[:-1], ru[:-1])
        Hm, Hp, Hpm = H[:, :n, :n], H[:, n:, n:], H[:, :n, n:]
        qm = g[:, :n] - (Hm @ Z[:-1, :, None] + Hpm @ Z[1:, :, None])[..., 0]
        qp = g[:, n:] - (Hpm.transpose(-1, -2) @ Z[:-1, :, None] + Hp @ Z[1:, :, None])[..., 0]
        term = lambda zz: self.terminal_cost(zz[:self.nx], zz[self.nx:], rx[-1], ru[-1], p)
        tg, tH = grad(term)(Z[-1]), hessian(term)(Z[-1])
        D = torch.zeros(self.T, n, n, dtype=F64)
        q = torch.zeros(self.T, n, dtype=F64)
        D[0] = Hm[0]
        D[1:N] = Hp[:-1] + Hm[1:]
        D[N] = Hp[-1] + tH
        q[0] = qm[0]
        q[1:N] = qp[:-1] + qm[1:]
        q[N] = qp[-1] + tg - tH @ Z[-1]
        return D, Hpm.clone(), q

    # ---- dynamics (optimal_control_problem.py:841-912, 1217-1272)
    def _dp(self, p):
        return p.get("dynamics_state_dot_params") or {}

    def next_state(self, x, u, p):
        return predict_next_state(self.model, self.dt, self.scheme, self._dp(p), x, u)

    def dynamics_rows(self, X, U, p):
        """A_minus = [A B], A_plus = [-I 0], c (N, nx), each row scaled by
        1 / state_diff under rescaling (optimal_control_problem.py:1322-1331)."""
        N, nx = self.N, self.nx

        def f(xu):
            return self.next_state(xu[:nx], xu[nx:], p)

        XU = torch.cat([X[:N], U[:N]], -1)
        val = vmap(f)(XU)
        J = vmap(jacfwd(f))(XU)
        c = -val + (J @ XU[..., None])[..., 0]
        Ap = torch.zeros(N, nx, self.n, dtype=F64)
        Ap[:, :, :nx] = -torch.eye(nx, dtype=F64)
        rs = 1.0 / self.rescaling(p)[0]
        return J * rs[:, None], Ap * rs[:, None], c * rs

    def equality_constraints(self, X, U, p):
        """optimal_control_problem.py:841-912 (explicit schemes)."""
        sd, cd = self.rescaling(p)
        x0c = X[0] - p["initial_state"]
        nxt = vmap(lambda x, u: self.next_state(x, u, p))(X[:-1], U[:-1])
        rows = torch.cat([x0c[None], nxt - X[1:]]) / sd
        out = [rows.reshape(-1)]
        if self.constrain_u0:
            out.append((U[0] - p["initial_control"]) / cd)
        return torch.cat(out)

    # ---- inequalities (optimal_control_problem.py:413-471; obstacle_avoidance.py:16-52)
    def step_inequality(self, x, u, p):
        parts_g, parts_l, parts_u = [], [], []
        if bool(self.state_mask.any()) or bool(self.control_mask.any()):
            xl = p["state_min_bounds"].expand(self.nx)[self.state_mask]
            xh = p["state_max_bounds"].expand(self.nx)[self.state_mask]
            ul = p["control_min_bounds"].expand(self.nu)[self.control_mask]
            uh = p["control_max_bounds"].expand(self.nu)[self.control_mask]
            sc = torch.ones(int(self.state_mask.sum()) + int(self.control_mask.sum()), dtype=F64)
            if self.rescale:  # optimal_control_problem.py:460-469
                sd, cd = self.rescaling(p)
                sc = torch.cat([sd[self.state_mask], cd[self.control_mask]])
            parts_g.append(torch.cat([x[self.state_mask], u[self.control_mask]]) / sc)
            parts_l.append(torch.cat([xl, ul]) / sc)
            parts_u.append(torch.cat([xh, uh]) / sc)
        if self.obstacles:
            dim = int(p["obstacles_dimension"])
            c, r = p["obstacles_centers"], p["obstacles_radii"]
            g = 1.0 - torch.linalg.vector_norm(x[:dim] - c, dim=-1) / (r + 0.001)
            rs = 1.0 / self.rescaling(p)[0][:dim].mean() if self.rescale else 1.0  # obstacle_avoidance.py:40-45
            parts_g.append(g * rs)
            parts_l.append(torch.full_like(g, -1e9) * rs)
            parts_u.append(torch.zeros_like(g) * rs)
        if not parts_g:
            z = torch.zeros(0, dtype=F64)
            return z, z, z
        return torch.cat(parts_g), torch.cat(parts_l), torch.cat(parts_u)

    @property
    def m(self):
        g, _, _ = self.step_inequality(torch.zeros(self.nx, dtype=F64), torch.zeros(self.nu, dtype=F64), self.p)
        return int(g.shape[0])

    def inequality_rows(self, X, U, p):
        """G (T, m, n), l, u (T, m) (optimal_control_problem.py:580-626)."""
        nx = self.nx
        gfun = lambda xu: self.step_inequality(xu[:nx], xu[nx:], p)[0]
        XU = torch.cat([X, U], -1)
        G = torch.stack([jacfwd(gfun)(XU[t]) if self.m > 0 else torch.zeros(0, self.n, dtype=F64)
                         for t in range(self.T)])
        l_list, u_list, off_list = [], [], []
        for t in range(self.T):
            g, lo, hi = self.step_inequality(X[t], U[t], p)
            off = g - G[t] @ XU[t]
            l_list.append(lo - off)
            u_list.append(hi - off)
        return G, torch.stack(l_list), torch.stack(u_list)

    def inequality_values(self, X, U, p):
        vals = [self.step_inequality(X[t], U[t], p) for t in range(self.T)]
        return (torch.stack([v[0] for v in vals]), torch.stack([v[1] for v in vals]),
                torch.stack([v[2] for v in vals]))

    # ---- Lagrangian Hessians (optimal_control_problem.py:1334-1481)
    def dynamics_lagrangian_hessian(self, X, U, p, lam):
        nx = self.nx

        rs = 1.0 / self.rescaling(p)[0]

        def s(xu, l_):
            return l_ @ (rs * self.next_state(xu[:nx], xu[nx:], p))

        XU = torch.cat([X[:-1], U[:-1]], -1)
        H = vmap(hessian(s))(XU, lam)
        return torch.cat([H, torch.zeros(1, self.n, self.n, dtype=F64)])

    def inequality_lagrangian_hessian(self, X, U, p, mu):
        nx = self.nx
        XU = torch.cat([X, U], -1)
        return torch.stack([hessian(lambda xu: mu[t] @ self.step_inequality(xu[:nx], xu[nx:], p)[0])(XU[t])
                            for t in range(self.T)])

    # ---- the QP (turbompc_solver.py:1098-1156)
    def qp(self, X, U, p, apply_variable_scaling=True):
        D, E, q = self.cost_blocks(X, U, p)
        Am, Ap, c = self.dynamics_rows(X, U, p)
        G, l, u = self.inequality_rows(X, U, p)
        sd, cd = self.rescaling(p)
        # optimal_control_problem.py:914-980
        A0 = torch.cat([torch.diag(1.0 / sd), torch.zeros(self.nx, self.nu, dtype=F64)], 1)
        c0 = p["initial_state"] / sd
        if self.constrain_u0:
            A0 = torch.cat([A0, torch.cat([torch.zeros(self.nu, self.nx, dtype=F64), torch.diag(1.0 / cd)], 1)])
            c0 = torch.cat([c0, p["initial_control"] / cd])
        if self.rescale and apply_variable_scaling:  # qp_data.py:178-210, z = diag(sc) z_hat
            sc = torch.cat([sd, cd])
            D, E, q = D * sc[:, None] * sc[None, :], E * sc[:, None] * sc[None, :], q * sc
            A0, Am, Ap, G = A0 * sc, Am * sc, Ap * sc, G * sc
        sw = float(p.get("slack_penalization_weight", 0.0))
        a = lambda t: t.detach().numpy()[None]
        return ref.QP(D=a(D), E=a(E), q=a(q), A0=a(A0), Am=a(Am), Ap=a(Ap), c0=a(c0), c=a(c), G=a(G), l=a(l),
                      u=a(u), slack_weight=np.array([sw]), use_slack=self.use_slack)


# ---------------------------------------------------------------------------
# SQP loop (turbompc_solver.py:1519-1760) for one problem
# ---------------------------------------------------------------------------
def identify_active_inequalities(g, l, u, eps_abs, eps_rel):
    """turbompc_solver.py:269-292."""
    dl, du = g - l, u - g
    use_upper = du < dl
    bound = np.where(use_upper, np.abs(u), np.abs(l))
    active = np.minimum(dl, du) <= eps_abs + eps_rel * bound
    return active & ~use_upper, active & use_upper


def first_order_error(qp: ref.QP, z, st: ref.ADMMState, slacks):
    """turbompc_solver.py:1158-1225; returns (conv, eq, ineq, g_for_bounds)."""
    stat = ref._inf(ref.apply_P(qp, z) + qp.q + ref.apply_Ct(qp, st.y_f0, st.y_fdyn) + ref.apply_Gt(qp, st.y_g))
    Cx0, Cx = ref.apply_C_parts(qp, z)
    eq = np.maximum(ref._inf(Cx0 - qp.c0), ref._inf(Cx - qp.c))
    g = ref.apply_G(qp, z)
    gb = g + slacks if qp.use_slack else g
    if qp.G.shape[2] > 0:
        ineq = ref._inf(np.maximum(np.maximum(qp.l - gb, 0.0), np.maximum(gb - qp.u, 0.0)))
    else:
        ineq = np.zeros_like(stat)
    conv = np.maximum(stat, np.maximum(eq, ineq))
    if qp.use_slack and qp.G.shape[2] > 0:
        conv = np.maximum(conv, ref._inf(qp.slack_weight[:, None, None] * slacks + st.y_g))
    return conv, eq, ineq, gb


@dataclass
class Solution:
    states: np.ndarray
    controls: np.ndarray
    state: ref.ADMMState
    num_iter: int
    conv: float
    active_lower: np.ndarray
    active_upper: np.ndarray
    admm_iters: List[int]


def build_kkt_active_sets(ocp: OCP, st: ref.ADMMState, g, l, u):
    """turbompc_solver.py:1387-1439 (active sets only)."""
    if ocp.use_slack:
        return st.xi_g[0] > 1e-12, st.xi_g[0] < -1e-12
    pl, pu = identify_active_inequalities(g, l, u, ocp.eps_abs, ocp.eps_rel)
    y = st.y_g[0]
    if y.shape[-1] == 0:
        return pl, pu
    dl, du = y < -ocp.eps_abs, y > ocp.eps_abs
    und = ~(dl | du)
    return dl | (und & pl), du | (und & pu)


def solve(ocp: OCP, X0, U0, cfg: ref.ADMMConfig, num_sqp: int, tol: float = 0.0, rho: float = 0.1,
          admm_state0: Optional[ref.ADMMState] = None, linsys: str = "pcg") -> Solution:
    """One problem's SQP solve (first-order criterion, no line search).
    linsys "pcg" runs the reference's PCG inside ADMM; "dense" solves each
    Schur system exactly (for converged solves)."""
    p = ocp.p
    X = torch.as_tensor(X0, dtype=F64)
    U = torch.as_tensor(U0, dtype=F64)
    qp = ocp.qp(X, U, p)
    st = admm_state0.copy() if admm_state0 is not None else ref.initial_state(qp, rho)
    slacks = st.xi_g
    z_prev = torch.cat([X, U], -1).numpy()[None]
    conv = math.inf
    it = 0
    iters = []
    lo = up = None
    while (it < num_sqp and conv > tol) or it < 1:
        st_new, n_it = ref.admm_solve(qp, st, cfg, linsys=linsys)
        iters.append(int(n_it[0]))
        z_new = st_new.x  # QP (scaled) coordinates
        sd, cd = ocp.rescaling(p)
        Xn = torch.as_tensor(z_new[0, :, :ocp.nx]) * sd
        Un = torch.as_tensor(z_new[0, :, ocp.nx:]) * cd
        z_true = torch.cat([Xn, Un], -1).numpy()[None]
        step = float(np.max(np.abs(z_true - z_prev)))
        if st_new.xi_g.shape[-1] > 0:
            step += float(np.max(np.abs(st_new.xi_g - slacks)))
        if it + 1 < num_sqp:
            qp_next = ocp.qp(Xn, Un, p)
            cv, _, _, g = first_order_error(qp_next, z_new, st_new, st_new.xi_g)
            conv_new = float(cv[0])
        else:
            qp_next = qp
            conv_new = step if it == 0 else conv
            g = ref.apply_G(qp, z_new)
            if qp.use_slack:
                g = g + st_new.xi_g
        lo, up = build_kkt_active_sets(ocp, st_new, g[0], qp_next.l[0], qp_next.u[0])
        X, U, st, slacks, z_prev, qp, conv = Xn, Un, st_new, st_new.xi_g, z_true, qp_next, conv_new
        it += 1
    return Solution(X.numpy(), U.numpy(), st, it, conv, lo, up, iters)


def solve_batch(make_ocp, B, X0, U0, cfg, num_sqp, tol=0.0, rho=0.1, states0=None):
    """Solve problems 0..B-1 (make_ocp(b) -> OCP); X0, U0 (B, T, .) initial guesses."""
    return [solve(make_ocp(b), X0[b], U0[b], cfg, num_sqp, tol, rho,
                  None if states0 is None else states0[b]) for b in range(B)]


# ---------------------------------------------------------------------------
# Backward pass (turbompc_solver.py:544-1018) for one problem
# ---------------------------------------------------------------------------
def vjp(ocp: OCP, sol: Solution, dl_dstates, dl_dcontrols, weight_keys=(), dl_dslack=None,
        use_full_hessian=True, eps_reg=1e-12):
    """Cotangents of the weights named in ``weight_keys`` (paths into
    ocp.p, a tuple of keys each) and of initial_state, for the loss
    cotangents dl_dstates (T, nx), dl_dcontrols (T, nu), dl_dslack (T, m).

    Returns {"initial_state": (nx,), path: array shaped like the weight,
    "slack_penalization_weight": scalar (slack problems)} and the adjoint
    solution (dz (T, n), y_eq_lin, y_ineq_lin)."""
    p = ocp.p
    X = torch.as_tensor(sol.states, dtype=F64)
    U = torch.as_tensor(sol.controls, dtype=F64)
    st = sol.state
    nx, n, T, N = ocp.nx, ocp.n, ocp.T, ocp.N
    qp = ocp.qp(X, U, p, apply_variable_scaling=False)  # turbompc_solver.py:553-560
    m = qp.G.shape[2]
    D = qp.D[0].copy()
    lo = sol.active_lower.astype(np.float64)
    up = sol.active_upper.astype(np.float64)
    if use_full_hessian:
        D = D + ocp.dynamics_lagrangian_hessian(X, U, p, torch.as_tensor(st.y_fdyn[0])).numpy()
        if m > 0:
            mu = torch.as_tensor((np.maximum(lo, up)) * st.y_g[0])
            D = D + ocp.inequality_lagrangian_hessian(X, U, p, mu).numpy()
    sign = lo - up
    G_act = qp.G[0] * sign[..., None]
    dl = np.concatenate([dl_dstates, dl_dcontrols], -1)
    slack_branch = ocp.use_slack and m > 0
    if dl_dslack is None:
        dl_dslack = np.zeros((T, m))
    if slack_branch:
        gamma = float(qp.slack_weight[0])
        Dk = D + gamma * np.swapaxes(G_act, -1, -2) @ G_act
        qk = -(dl - np.einsum("tmi,tm->ti", G_act, dl_dslack))
        Gk = np.zeros((T, 0, n))
    else:
        Dk, qk, Gk = D, -dl, G_act
    kq = ref.QP(D=Dk[None], E=qp.E, q=qk[None], A0=qp.A0, Am=qp.Am, Ap=qp.Ap, c0=np.zeros_like(qp.c0),
                c=np.zeros_like(qp.c), G=Gk[None], l=np.zeros((1, T, Gk.shape[1])), u=np.zeros((1, T, Gk.shape[1])))
    K, rhs = ref.assemble_backward_kkt(kq, eps_reg)
    solv = np.linalg.solve(K, rhs[..., None])[0, :, 0]
    dz = solv[:T * n].reshape(T, n)
    mult = solv[T * n:]
    n0 = qp.A0.shape[1]
    n_eq = n0 + N * nx
    # [x0 rows, dynamics rows, u0 rows], the order of equality_constraints
    # (turbompc_solver.py:736-744)
    y_eq_lin = np.concatenate([mult[:nx], mult[n0:n_eq], mult[nx:n0]])
    dL_dgamma = 0.0
    if slack_branch:
        act = np.maximum(lo, up)
        g_dx = np.einsum("tmi,ti->tm", G_act, dz)
        y_ineq_lin = (dl_dslack * act + gamma * g_dx).reshape(-1)
        dL_dgamma = float(np.sum(sign * st.xi_g[0] * act * g_dx))
    else:
        y_ineq_lin = mult[n_eq:n_eq + T * m]
    # forward multipliers (turbompc_solver.py:862-880)
    y_eq_star = np.concatenate([st.y_f0[0, :nx], st.y_fdyn[0].reshape(-1), st.y_f0[0, nx:]])
    y_ineq_star = (-sign * st.y_g[0]).reshape(-1)

    # turbompc_solver.py:990-1018: the x0 / u0 row multipliers, unscaled
    sd, cd = ocp.rescaling(p)
    out = {"initial_state": mult[:nx] / sd.numpy()}
    if ocp.constrain_u0:
        out["initial_control"] = mult[nx:n0] / cd.numpy()
    if weight_keys:
        leaves = [_get(p, k) for k in weight_keys]
        yes, yis = torch.as_tensor(y_eq_star), torch.as_tensor(y_ineq_star)
        dzt = torch.as_tensor(dz)
        yel, yil = torch.as_tensor(y_eq_lin), torch.as_tensor(y_ineq_lin)
        lo_t, up_t = torch.as_tensor(lo).reshape(-1), torch.as_tensor(up).reshape(-1)

        def bundle(*vals):
            pp = p
            for k, v in zip(weight_keys, vals):
                pp = _set(pp, k, v)

            def active_ineq(Xv, Uv):
                if m == 0:
                    return torch.zeros(0, dtype=F64)
                g, l_, u_ = ocp.inequality_values(Xv, Uv, pp)
                return lo_t * (g - l_).reshape(-1) + up_t * (u_ - g).reshape(-1)

            def lagr(Xv, Uv):
                val = ocp.cost(Xv, Uv, pp) + yes @ ocp.equality_constraints(Xv, Uv, pp)
                return val + yis @ active_ineq(Xv, Uv)

            gx, gu = grad(lagr, argnums=(0, 1))(X, U)
            # turbompc_solver.py:930-966: -(F_z . dz + g . y_eq_lin + h . y_ineq_lin)
            phi = (gx * dzt[:, :nx]).sum() + (gu * dzt[:, nx:]).sum()
            phi = phi + ocp.equality_constraints(X, U, pp) @ yel + active_ineq(X, U) @ yil
            return -phi

        J = jacfwd(bundle, argnums=tuple(range(len(leaves))))(*leaves)
        for k, jk in zip(weight_keys, J):
            out[k] = jk.detach().numpy()
    if slack_branch:
        out["slack_penalization_weight"] = dL_dgamma
    return out, (dz, y_eq_lin, y_ineq_lin)


def _get(p, path):
    v = p
    for k in path:
        v = v[k]
    return v


def _set(p, path, value):
    q = dict(p)
    if len(path) == 1:
        q[path[0]] = value
    else:
        q[path[0]] = _set(q[path[0]], path[1:], value)
    return q
