"""Benchmark configuration 3 (and the config-4 obstacle variant): batched
quadrotor tracking MPC with seeded synthetic initial states and set-points.

Choices the configuration leaves open (recorded here):
tracking weights w_x = [10]*3 (position) + [1]*3 (angles) + [1]*3 (velocity)
+ [0.1]*3 (rates); terminal extra weight 10 w_x; thrust weight 0.1 around
hover thrust m g / 4 (penalize_control_reference); no rate penalty; thrust
box [0, 5] N (m = 4 active rows); initial-guess final state = set-point.
"""
from __future__ import annotations

import numpy as np
import torch

from ..dynamics import Quadrotor12Dynamics
from .ocp import OptimalControlProblem, OptimalControlProblemObstacle

HOVER_THRUST = 1.0 * 9.81 / 4.0


def quadrotor_params(batch, N=50, dt=0.02, seed=0, dtype=torch.float32, device="cuda"):
    rng = np.random.default_rng(seed)
    x0 = rng.normal(0.0, 0.3, size=(batch, 12))
    pref = rng.uniform(-1.0, 1.0, size=(batch, 3))
    xr = np.zeros((batch, 12))
    xr[:, :3] = pref
    t = lambda a: torch.as_tensor(a, dtype=dtype, device=device)
    wx = np.array([10.0] * 3 + [1.0] * 3 + [1.0] * 3 + [0.1] * 3)
    return {
        "horizon": N, "discretization_resolution": dt, "discretization_scheme": 2,
        "initial_state": t(x0), "initial_guess_final_state": t(xr),
        "reference_state_trajectory": t(xr)[:, None, :].expand(batch, N + 1, 12).contiguous(),
        "reference_control_trajectory": t(np.full(4, HOVER_THRUST)),
        "penalize_control_reference": True,
        "weights_penalization_reference_state_trajectory": t(wx),
        "weights_penalization_final_state": t(10.0 * wx),
        "weights_penalization_control_squared": t(np.full(4, 0.1)),
        "weights_penalization_control_rate": t(np.zeros(4)),
        "state_min_bounds": t(np.full(12, -1e9)), "state_max_bounds": t(np.full(12, 1e9)),
        "control_min_bounds": t(np.zeros(4)), "control_max_bounds": t(np.full(4, 5.0)),
        "dynamics_state_dot_params": {},
    }


def make_quadrotor_problem(batch, N=50, dt=0.02, seed=0, dtype=torch.float32, device="cuda", rate_weight=0.0):
    """Config 3; rate_weight > 0 adds a control-rate penalty (the QP's E blocks
    then couple consecutive stages' controls)."""
    params = quadrotor_params(batch, N, dt, seed, dtype, device)
    if rate_weight:
        params["weights_penalization_control_rate"] = torch.full((4,), float(rate_weight), dtype=dtype, device=device)
    return OptimalControlProblem(Quadrotor12Dynamics(), params), params


def make_obstacle_problem(batch, N=40, dt=0.02, n_obstacles=8, seed=0, dtype=torch.float32, device="cuda"):
    """Config 4: 8 spheres per problem, centres U(-3,3)^3, radii U(0.2,0.5);
    spheres that contain x0 or the set-point are resampled."""
    params = quadrotor_params(batch, N, dt, seed, dtype, device)
    rng = np.random.default_rng(seed + 1)
    x0 = params["initial_state"][:, :3].cpu().numpy()
    xr = params["initial_guess_final_state"][:, :3].cpu().numpy()
    c = rng.uniform(-3.0, 3.0, size=(batch, n_obstacles, 3))
    r = rng.uniform(0.2, 0.5, size=(batch, n_obstacles))
    for _ in range(100):
        bad = ((np.linalg.norm(c - x0[:, None], axis=-1) < r + 0.1)
               | (np.linalg.norm(c - xr[:, None], axis=-1) < r + 0.1))
        if not bad.any():
            break
        c[bad] = rng.uniform(-3.0, 3.0, size=(int(bad.sum()), 3))
    params["obstacles_centers"] = torch.as_tensor(c, dtype=dtype, device=device)
    params["obstacles_radii"] = torch.as_tensor(r, dtype=dtype, device=device)
    params["obstacles_dimension"] = 3
    return OptimalControlProblemObstacle(Quadrotor12Dynamics(), params), params
