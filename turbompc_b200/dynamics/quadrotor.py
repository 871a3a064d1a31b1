"""12-state rigid-body quadrotor with four rotor thrusts (benchmark configuration 3).

State  x = [p (3, world), Euler angles (roll phi, pitch theta, yaw psi),
            v (3, world-frame velocity), omega (3, body rates)]
Control u = [f1, f2, f3, f4] rotor thrusts in N ("+" layout: rotors 1/3 on the
body x axis, 2/4 on the body y axis; 1 and 3 spin opposite to 2 and 4).

    p_dot     = v
    eta_dot   = W(phi, theta) omega
    v_dot     = R(phi, theta, psi) [0, 0, sum f] / m - [0, 0, g]
    omega_dot = J^-1 (tau - omega x J omega)
    tau       = [L (f2 - f4), L (f3 - f1), k (f1 - f2 + f3 - f4)]

with R = Rz(psi) Ry(theta) Rx(phi).  Parameters (mass 1 kg and
J = diag(0.01) from the configuration; arm length L = 0.1 m and yaw moment
coefficient k = 0.01 m chosen here) may be overridden through params keys
``mass``, ``inertia`` (3,), ``arm_length``, ``yaw_coefficient``.
"""
from __future__ import annotations

import torch

from .base import Dynamics

GRAVITY = 9.81
DEFAULTS = dict(mass=1.0, inertia=(0.01, 0.01, 0.01), arm_length=0.1, yaw_coefficient=0.01)


class Quadrotor12Dynamics(Dynamics):
    def __init__(self):
        super().__init__({
            "num_states": 12, "num_controls": 4,
            "names_states": ["x", "y", "z", "roll", "pitch", "yaw", "vx", "vy", "vz", "wx", "wy", "wz"],
            "names_controls": ["f1", "f2", "f3", "f4"]})

    def cuda_model(self, params=None):
        """(model id, parameter list) for the CUDA linearisation kernel, or
        None when a parameter is a tensor (per-problem values)."""
        params = params or {}
        m = params.get("mass", DEFAULTS["mass"])
        J = params.get("inertia", DEFAULTS["inertia"])
        L = params.get("arm_length", DEFAULTS["arm_length"])
        k = params.get("yaw_coefficient", DEFAULTS["yaw_coefficient"])
        vals = [m, *(J if not isinstance(J, torch.Tensor) else [None]), L, k]
        if any(v is None or isinstance(v, torch.Tensor) for v in vals) or len(vals) != 6:
            return None
        return 1, [float(v) for v in vals]

    def state_dot(self, state, control, params=None):
        params = params or {}
        m = params.get("mass", DEFAULTS["mass"])
        J = params.get("inertia", None)
        if J is None:
            Jx = Jy = Jz = DEFAULTS["inertia"][0]
        else:
            Jx, Jy, Jz = J[..., 0], J[..., 1], J[..., 2]
        L = params.get("arm_length", DEFAULTS["arm_length"])
        k = params.get("yaw_coefficient", DEFAULTS["yaw_coefficient"])
        phi, th, psi = state[..., 3], state[..., 4], state[..., 5]
        v = state[..., 6:9]
        wx, wy, wz = state[..., 9], state[..., 10], state[..., 11]
        f1, f2, f3, f4 = control[..., 0], control[..., 1], control[..., 2], control[..., 3]
        sph, cph = torch.sin(phi), torch.cos(phi)
        sth, cth = torch.sin(th), torch.cos(th)
        sps, cps = torch.sin(psi), torch.cos(psi)
        tth = sth / cth
        phid = wx + sph * tth * wy + cph * tth * wz
        thd = cph * wy - sph * wz
        psid = (sph * wy + cph * wz) / cth
        F = (f1 + f2 + f3 + f4) / m
        # third column of R = Rz Ry Rx
        ax = (cps * sth * cph + sps * sph) * F
        ay = (sps * sth * cph - cps * sph) * F
        az = cth * cph * F - GRAVITY
        tx = L * (f2 - f4)
        ty = L * (f3 - f1)
        tz = k * (f1 - f2 + f3 - f4)
        wxd = (tx - (Jz - Jy) * wy * wz) / Jx
        wyd = (ty - (Jx - Jz) * wz * wx) / Jy
        wzd = (tz - (Jy - Jx) * wx * wy) / Jz
        return torch.stack([v[..., 0], v[..., 1], v[..., 2], phid, thd, psid, ax, ay, az, wxd, wyd, wzd], dim=-1)
