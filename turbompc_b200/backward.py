"""Differentiable solve (the role of jax.custom_vjp in
turbompc/solvers/turbompc_solver.py:1020-1096)."""
from __future__ import annotations


def make_differentiable_solve(solver):
    def solve(initial_guess, problem_params, weights=None):
        params = solver.make_params_with_weights(weights or {}, problem_params)
        return solver._solve_impl(initial_guess.states, initial_guess.controls, params, initial_guess.admm_state)

    return solve
