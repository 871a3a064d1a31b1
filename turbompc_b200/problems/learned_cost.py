"""Benchmark configuration 5: differentiable MPC with a learned stage cost on the
Clohessy-Wiltshire relative-motion model.

Stage cost (every stage t, z_t = [x_t, u_t]):
    l(z_t) = tracking terms of OptimalControlProblem + s * MLP(z_t)
    MLP(z) = w2 . tanh(W1 z + b1)          (hidden width H, tanh; 2 layers)
quadratised at each SQP iterate (turbompc/problems/optimal_control_problem.py:
1068-1174 restated for this cost) with the exact gradient and Hessian of the
MLP term:
    a = W1 z + b1,  th = tanh(a),  d = 1 - th^2
    grad = s W1^T (w2 * d),   Hess = s W1^T diag(w2 * (-2 th d)) W1.
``mlp_scale`` s is chosen by the generator so that the MLP Hessian's norm
stays below half the smallest tracking-Hessian entry: D stays positive
definite for every iterate (the quadratised QP remains convex).

Cost parameters (W1, b1, w2, and the dynamics' A, B) are ordinary params
entries, so gradients with respect to them flow through the solver's VJP.
"""
from __future__ import annotations

import numpy as np
import torch

from ..dynamics import LinearDynamics
from .ocp import OptimalControlProblem, _t


class OptimalControlProblemLearnedCost(OptimalControlProblem):
    @property
    def state_independent_cost(self) -> bool:
        return False

    def _mlp(self, params, like):
        return (_t(params["mlp_W1"], like), _t(params["mlp_b1"], like), _t(params["mlp_w2"], like),
                float(params["mlp_scale"]))

    def get_cost_linearized_blocks(self, states, controls, params):
        """Tracking blocks plus the MLP term's exact quadratisation: one CUDA
        kernel (tmpc_mlp_cost_blocks_*) on GPU tensors, PyTorch otherwise."""
        D, E, q = super().get_cost_linearized_blocks(states, controls, params)
        W1, b1, w2, s = self._mlp(params, states)
        if states.is_cuda and states.shape[-1] + controls.shape[-1] <= 16:
            from .. import ops
            D, q = D.contiguous(), q.contiguous()
            ops.mlp_cost_blocks_(D, q, states, controls, W1.detach(), b1.detach(), w2.detach(), s)
            return D, E, q
        return self._mlp_blocks_torch(D, E, q, states, controls, W1, b1, w2, s)

    def _mlp_blocks_torch(self, D, E, q, states, controls, W1, b1, w2, s):
        """The same quadratisation in PyTorch operations (host tensors; the
        CUDA kernel's test reference)."""
        z = torch.cat([states, controls], -1)  # (Nb, T, n)
        a = torch.einsum("hn,btn->bth", W1, z) + b1
        th = torch.tanh(a)
        d = 1 - th * th
        grad = s * torch.einsum("hn,bth->btn", W1, w2 * d)
        curv = s * (w2 * (-2.0 * th * d))  # (Nb, T, H)
        H = torch.einsum("hi,bth,hj->btij", W1, curv, W1)
        D = D + H
        q = q + grad - torch.einsum("btij,btj->bti", H, z)
        return D, E, q

    def cost(self, states, controls, params):
        c = super().cost(states, controls, params)
        W1, b1, w2, s = self._mlp(params, states)
        z = torch.cat([states, controls], -1)
        mlp = torch.einsum("h,bth->bt", w2, torch.tanh(torch.einsum("hn,btn->bth", W1, z) + b1))
        return c + s * mlp.sum(-1)


def cw_matrices(mean_motion=0.0011):
    """Continuous Clohessy-Wiltshire A (6x6), B (6x3)."""
    n = mean_motion
    A = np.zeros((6, 6))
    A[0:3, 3:6] = np.eye(3)
    A[3, 0] = 3 * n * n
    A[3, 4] = 2 * n
    A[4, 3] = -2 * n
    A[5, 2] = -n * n
    B = np.zeros((6, 3))
    B[3:6, :] = np.eye(3)
    return A, B


def make_learned_cost_problem(batch, N=60, dt=10.0, hidden=64, seed=0, mean_motion=0.0011, u_max=0.1,
                              dtype=torch.float32, device="cuda"):
    """Config 5 workload: CW relative motion as a linear model (A, B are
    parameters so that gradients reach them), RK4, |u| <= u_max, tracking to
    the origin plus the MLP term; MLP weights ~ N(0, 1/fan_in), seeded.
    Nondimensional units (the configuration fixes none): unit tracking
    weights on every state and control, terminal weight 10x, initial
    positions ~ N(0, 1) and velocities ~ N(0, 0.1^2).  With these scales the
    fixed-count solve is well conditioned (a 1e-14 relative perturbation of
    the MLP weights moves the 3 x 30 x 10 solution by ~1e-12); with metric
    units (positions ~100 m, weights ~1e-4) the same perturbation moved it by
    several percent, so fixed-count parity would be unattainable."""
    rng = np.random.default_rng(seed)
    nx, nu = 6, 3
    n = nx + nu
    A, B = cw_matrices(mean_motion)
    W1 = rng.normal(0.0, 1.0 / np.sqrt(n), size=(hidden, n))
    b1 = rng.normal(0.0, 1.0, size=hidden)
    w2 = rng.normal(0.0, 1.0 / np.sqrt(hidden), size=hidden)
    wx = np.ones(nx)
    wu = np.ones(nu)
    # |Hess MLP| <= s * 0.77 * sum_h |w2_h| ||W1_h||^2 <= 0.5 * min(2 wx, 2 wu)
    bound = 0.7699 * float(np.sum(np.abs(w2) * np.sum(W1 * W1, axis=1)))
    scale = 0.5 * 2.0 * min(wx.min(), wu.min()) / bound
    x0 = np.concatenate([rng.normal(0.0, 1.0, size=(batch, 3)), rng.normal(0.0, 0.1, size=(batch, 3))], 1)
    t = lambda a: torch.as_tensor(a, dtype=dtype, device=device)
    params = {
        "horizon": N, "discretization_resolution": dt, "discretization_scheme": 2,
        "initial_state": t(x0), "initial_guess_final_state": t(np.zeros(nx)),
        "reference_state_trajectory": t(np.zeros(nx)), "reference_control_trajectory": t(np.zeros(nu)),
        "penalize_control_reference": False,
        "weights_penalization_reference_state_trajectory": t(wx),
        "weights_penalization_final_state": t(10.0 * wx),
        "weights_penalization_control_squared": t(wu),
        "weights_penalization_control_rate": t(np.zeros(nu)),
        "state_min_bounds": t(np.full(nx, -1e9)), "state_max_bounds": t(np.full(nx, 1e9)),
        "control_min_bounds": t(np.full(nu, -u_max)), "control_max_bounds": t(np.full(nu, u_max)),
        "dynamics_state_dot_params": {"A": t(A), "B": t(B)},
        "mlp_W1": t(W1), "mlp_b1": t(b1), "mlp_w2": t(w2), "mlp_scale": scale,
    }
    return OptimalControlProblemLearnedCost(LinearDynamics(nx, nu), params), params
