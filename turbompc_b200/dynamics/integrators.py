"""Explicit integrators (turbompc/dynamics/integrators.py:12-76)."""
from __future__ import annotations

import enum


class DiscretizationScheme(enum.IntEnum):
    EULER = 0
    MIDPOINT = 1
    RUNGEKUTTA4 = 2
    IMPLICIT = 10


def predict_next_state(dynamics, dt, scheme, params, state, control):
    """One step of the scheme (zero-order hold on the control)."""
    scheme = DiscretizationScheme(int(scheme))
    f = lambda x: dynamics.state_dot(x, control, params)
    if scheme == DiscretizationScheme.EULER:
        return state + dt * f(state)
    if scheme == DiscretizationScheme.MIDPOINT:
        return state + dt * f(state + 0.5 * dt * f(state))
    if scheme == DiscretizationScheme.RUNGEKUTTA4:
        k1 = f(state)
        k2 = f(state + 0.5 * dt * k1)
        k3 = f(state + 0.5 * dt * k2)
        k4 = f(state + dt * k3)
        return state + (1.0 / 6.0) * (k1 + 2 * k2 + 2 * k3 + k4) * dt
    raise NotImplementedError("implicit trapezoid integration is not on the b200 path")
