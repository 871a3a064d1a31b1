"""Dynamics interface (mirrors turbompc/dynamics/base_dynamics.py:16-131).

``state_dot(state, control, params)`` works on arbitrary leading batch
dimensions: state (..., nx), control (..., nu); params is a dict of tensors
broadcastable against the leading dimensions.
"""
from __future__ import annotations

from typing import Any, Dict

import torch


class Dynamics:
    def __init__(self, parameters: Dict[str, Any]):
        self._params = parameters

    @property
    def params(self) -> Dict[str, Any]:
        return self._params

    @property
    def num_states(self) -> int:
        return int(self._params["num_states"])

    @property
    def num_controls(self) -> int:
        return int(self._params["num_controls"])

    @property
    def names_states(self):
        return self._params.get("names_states", [f"x{i}" for i in range(self.num_states)])

    @property
    def names_controls(self):
        return self._params.get("names_controls", [f"u{i}" for i in range(self.num_controls)])

    def state_dot(self, state: torch.Tensor, control: torch.Tensor, params: Dict[str, Any]) -> torch.Tensor:
        raise NotImplementedError


class LinearDynamics(Dynamics):
    """x_dot = A x + B u + b (turbompc/dynamics/linear_dynamics.py:45-68).
    params: A (..., nx, nx), B (..., nx, nu), b (..., nx)."""

    def __init__(self, num_states: int = 4, num_controls: int = 2):
        super().__init__({"num_states": num_states, "num_controls": num_controls})

    def state_dot(self, state, control, params):
        out = torch.einsum("...ij,...j->...i", params["A"], state) + torch.einsum("...ij,...j->...i", params["B"],
                                                                                 control)
        if "b" in params:
            out = out + params["b"]
        return out
