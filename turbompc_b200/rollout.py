"""Batched closed-loop MPC rollout on the GPU (the harness of
turbompc/utils/timing.py:69-122, ``build_rollout_fn``, run for a whole batch of
environments at once instead of ``jit(vmap(rollout))``).

Each simulation step solves the MPC problem from the current states (the
``initial_state`` weight), applies the first control of every solution,
advances the states with one step of the problem's integrator and adds the
step cost; with ``warm_start`` the next solve starts from the previous
solution (states, controls and ADMM state), otherwise every solve restarts
from the fixed initial guess (the reference's cold-start rollout, which keeps
automatic and finite-difference gradients consistent).

Gradients flow through the rollout: the solves are differentiable with
respect to the tensors in ``weights`` (the solver's VJP) and the simulation
step is plain PyTorch.
"""
from __future__ import annotations

from typing import Any, Callable, Dict, Optional, Tuple

import torch

from .dynamics.integrators import predict_next_state


def quadratic_step_cost(program, params) -> Callable[[torch.Tensor, torch.Tensor], torch.Tensor]:
    """Default step cost: the problem's stage tracking terms,
    sum w_x (x - x_ref)^2 + w_u (u - u_ref)^2 (first stage of the references)."""
    def cost(x, u):
        wx = torch.as_tensor(params["weights_penalization_reference_state_trajectory"], dtype=x.dtype,
                             device=x.device)
        wu = torch.as_tensor(params["weights_penalization_control_squared"], dtype=x.dtype, device=x.device)
        xr = torch.as_tensor(params["reference_state_trajectory"], dtype=x.dtype, device=x.device)
        ur = torch.as_tensor(params["reference_control_trajectory"], dtype=x.dtype, device=x.device)
        if xr.dim() == 3:
            xr = xr[:, 0]
        if not params.get("penalize_control_reference", False):
            ur = torch.zeros_like(ur)
        if ur.dim() == 3:
            ur = ur[:, 0]
        return (wx * (x - xr) ** 2).sum(-1) + (wu * (u - ur) ** 2).sum(-1)
    return cost


def closed_loop_rollout(solver, problem_params: Dict[str, Any], initial_states: torch.Tensor, num_steps: int,
                        weights: Optional[Dict[str, Any]] = None, warm_start: bool = True,
                        step_cost: Optional[Callable[[torch.Tensor, torch.Tensor], torch.Tensor]] = None
                        ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Roll ``num_steps`` MPC steps for every environment of the batch.

    Returns (total cost (Nb,), ADMM iteration counts (num_steps, Nb, SQP
    iterations), visited states (num_steps + 1, Nb, nx))."""
    program = solver.program
    dt = float(problem_params["discretization_resolution"])
    scheme = int(problem_params["discretization_scheme"])
    dyn_params = program._dyn_params(dict(problem_params, **(weights or {})), initial_states)
    step_cost = step_cost or quadratic_step_cost(program, problem_params)
    state = initial_states
    guess = solver.initial_guess(dict(problem_params, initial_state=state.detach()))
    total = torch.zeros(state.shape[0], dtype=state.dtype, device=state.device)
    iters, visited = [], [state]
    for _ in range(num_steps):
        w = dict(weights or {})
        w["initial_state"] = state
        sol = solver.solve(guess, problem_params, w)
        u = sol.controls[:, 0]
        state = predict_next_state(program.dynamics, dt, scheme, dyn_params, state, u)
        total = total + step_cost(state, u)
        iters.append(sol.admm_iters)
        visited.append(state)
        if warm_start:
            guess = sol._replace(states=sol.states.detach(), controls=sol.controls.detach())
    return total, torch.stack(iters), torch.stack(visited)
