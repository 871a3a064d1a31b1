"""Dynamics models and integrators (batched PyTorch)."""
from .base import Dynamics, LinearDynamics
from .integrators import DiscretizationScheme, predict_next_state
from .quadrotor import Quadrotor12Dynamics
from .spacecraft import ClohessyWiltshireDynamics

__all__ = ["Dynamics", "LinearDynamics", "DiscretizationScheme", "predict_next_state", "Quadrotor12Dynamics",
           "ClohessyWiltshireDynamics"]
