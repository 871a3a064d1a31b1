"""Clohessy-Wiltshire relative motion (benchmark configuration 5).

State [x, y, z, vx, vy, vz] in the Hill frame, control = acceleration (3,).
    x_dd = 3 n^2 x + 2 n y_d + ux ;  y_d d = -2 n x_d + uy ;  z_dd = -n^2 z + uz
The mean motion n (rad/s) comes from params["mean_motion"] (default 0.0011).
"""
from __future__ import annotations

import torch

from .base import Dynamics


class ClohessyWiltshireDynamics(Dynamics):
    def __init__(self):
        super().__init__({"num_states": 6, "num_controls": 3,
                          "names_states": ["x", "y", "z", "vx", "vy", "vz"], "names_controls": ["ax", "ay", "az"]})

    def cuda_model(self, params=None):
        """(model id, parameter list) for the CUDA linearisation kernel, or None."""
        n = (params or {}).get("mean_motion", 0.0011)
        if isinstance(n, torch.Tensor):
            return None
        return 2, [float(n)]

    def state_dot(self, state, control, params=None):
        n = (params or {}).get("mean_motion", 0.0011)
        x, z = state[..., 0], state[..., 2]
        vx, vy, vz = state[..., 3], state[..., 4], state[..., 5]
        ax = 3 * n * n * x + 2 * n * vy + control[..., 0]
        ay = -2 * n * vx + control[..., 1]
        az = -n * n * z + control[..., 2]
        return torch.stack([vx, vy, vz, ax, ay, az], dim=-1)
