"""Gradient accuracy of the differentiable MPC rollout against finite
differences, swept over solver tolerances (the protocol of
benchmarking/linear-system/benchmark_turbompc_gradient_accuracy.py, on the
batched GPU rollout of turbompc_b200.rollout).

For every tolerance and seed: a batch of closed-loop LTI MPC rollouts
(cold-started solves, as the reference's gradient benchmark), the total cost
sum_t (|x_t|^2 + |u_t|^2) over the batch, and its gradient with respect to the
diagonal tracking weights Q (state) and R (control) twice: by the solver's VJP
(automatic) and by central finite differences of the same rollout.  Reported
per tolerance, over the seeds: cosine similarity, relative and absolute L2
error for Q, R and both together (mean, std, median, min, max).

    python -m turbompc_b200.gradient_accuracy [--tolerances 1e-3 1e-5 1e-7]
        [--n_seeds 10] [--batch_size 64] [--horizon 40] [--sim_steps 50]
        [--n_state 8] [--n_ctrl 4] [--umax 1.0] [--admm_max_iter 1000]
        [--fd_eps 1e-5] [--forward b200_direct] [--out results.json]

Problem data follow benchmarking/linear-system/utils.py:28-62 (A = I + 0.1 N(0,1)
with its eigenvalues pulled inside the unit circle, B ~ N(0,1), b ~ 0.01 N(0,1),
x0 ~ 5 N(0,1), Q = I, R = I; the legacy NumPy generator seeded with the seed) and
benchmark_problem_setup.py (dt = 1 Euler with A_c = A - I, |u| <= umax, no
terminal weight).  Computed in float64.
"""
from __future__ import annotations

import argparse
import json
from typing import Any, Dict, List

import numpy as np
import torch

from .dynamics import LinearDynamics
from .problems.ocp import OptimalControlProblem
from .rollout import closed_loop_rollout
from .solver import TurboMPCSolver

KEYS = ("weights_penalization_reference_state_trajectory", "weights_penalization_control_squared")


def problem_data(batch: int, seed: int, nx: int, nu: int):
    """(Q, R, A, B, b, x0) as benchmarking/linear-system/utils.py:28-62."""
    rs = np.random.RandomState(seed)
    Q, R = np.eye(nx), np.eye(nu)
    A = np.eye(nx) + 0.1 * rs.randn(nx, nx)
    lam, V = np.linalg.eig(A)
    mag = np.abs(lam)
    lam = np.where(mag < 1 - 1e-2, lam, lam / (mag + 1e-2))
    A = (V @ np.diag(lam) @ np.linalg.inv(V)).real
    B = rs.randn(nx, nu)
    b = 0.01 * rs.randn(nx)
    x0 = rs.randn(batch, nx) * 5.0
    return Q, R, A, B, b, x0


def make_problem(seed: int, batch: int, horizon: int, nx: int, nu: int, umax: float, device="cuda",
                 dtype=torch.float64):
    Q, R, A, B, b, x0 = problem_data(batch, seed, nx, nu)
    t = lambda a: torch.as_tensor(np.array(a), dtype=dtype, device=device)
    N = horizon - 1
    params = {
        "horizon": N, "discretization_resolution": 1.0, "discretization_scheme": 0,
        "initial_state": t(x0), "initial_guess_final_state": t(np.zeros(nx)),
        "reference_state_trajectory": t(np.zeros(nx)), "reference_control_trajectory": t(np.zeros(nu)),
        "penalize_control_reference": False,
        "weights_penalization_reference_state_trajectory": t(np.diag(Q)),
        "weights_penalization_final_state": t(np.zeros(nx)),
        "weights_penalization_control_squared": t(np.diag(R)),
        "weights_penalization_control_rate": t(np.zeros(nu)),
        "state_min_bounds": t(-1e7 * np.ones(nx)), "state_max_bounds": t(1e7 * np.ones(nx)),
        "control_min_bounds": t(-umax * np.ones(nu)), "control_max_bounds": t(umax * np.ones(nu)),
        "dynamics_state_dot_params": {"A": t(A - np.eye(nx)), "B": t(B), "b": t(b)},
    }
    return OptimalControlProblem(LinearDynamics(nx, nu), params), params


def solver_params(tol: float, admm_max_iter: int, sqp_iter: int = 1) -> Dict[str, Any]:
    """benchmark_turbompc_gradient_accuracy.py:81-102."""
    return {"num_sqp_iteration_max": sqp_iter, "tol_convergence": tol,
            "admm": {"max_iter": admm_max_iter, "check_termination_every": 1, "eps_abs": tol, "eps_rel": tol,
                     "relaxation_parameter": 1.0, "pcg": {"tol_epsilon": 1e-12}}}


def _metrics(ad: np.ndarray, fd: np.ndarray) -> Dict[str, float]:
    ad, fd = ad.ravel(), fd.ravel()
    cos = float(ad @ fd / (np.linalg.norm(ad) * np.linalg.norm(fd) + 1e-12))
    return {"cos": cos, "rel_l2": float(np.linalg.norm(ad - fd) / (np.linalg.norm(fd) + 1e-12)),
            "abs_l2": float(np.linalg.norm(ad - fd))}


def seed_gradients(seed: int, tol: float, args) -> Dict[str, Dict[str, float]]:
    prog, params = make_problem(seed, args.batch_size, args.horizon, args.n_state, args.n_ctrl, args.umax)
    solver = TurboMPCSolver(prog, solver_params(tol, args.admm_max_iter), forward_backend=args.forward,
                            backward_backend="b200", use_full_hessian=True)
    x0 = params["initial_state"]
    step_cost = lambda x, u: (x * x).sum(-1) + (u * u).sum(-1)

    def total(weights):
        cost, _, _ = closed_loop_rollout(solver, params, x0, args.sim_steps, weights=weights, warm_start=False,
                                         step_cost=step_cost)
        return cost.sum()

    leaves = {k: params[k].detach().clone().requires_grad_(True) for k in KEYS}
    g_ad = torch.autograd.grad(total(leaves), [leaves[k] for k in KEYS])
    g_fd = []
    with torch.no_grad():
        for k in KEYS:
            base = params[k].detach().clone()
            g = torch.zeros_like(base)
            for i in range(base.numel()):
                vals = []
                for sgn in (1.0, -1.0):
                    w = base.clone()
                    w.view(-1)[i] += sgn * args.fd_eps
                    vals.append(total({kk: (w if kk == k else params[kk]) for kk in KEYS}).item())
                g.view(-1)[i] = (vals[0] - vals[1]) / (2 * args.fd_eps)
            g_fd.append(g)
    ad = [a.cpu().numpy() for a in g_ad]
    fd = [f.cpu().numpy() for f in g_fd]
    return {"Q": _metrics(ad[0], fd[0]), "R": _metrics(ad[1], fd[1]),
            "all": _metrics(np.concatenate([a.ravel() for a in ad]), np.concatenate([f.ravel() for f in fd]))}


def run(args) -> Dict[str, Any]:
    out: Dict[str, Any] = {}
    for tol in args.tolerances:
        per: List[Dict[str, Dict[str, float]]] = []
        for seed in range(args.n_seeds):
            m = seed_gradients(seed, tol, args)
            per.append(m)
            if not args.quiet:
                print(f"tol={tol:.0e} seed={seed:3d} cos(Q)={m['Q']['cos']:.6f} cos(R)={m['R']['cos']:.6f} "
                      f"cos(all)={m['all']['cos']:.6f} rel_l2(all)={m['all']['rel_l2']:.2e}", flush=True)
        agg: Dict[str, Any] = {"n_seeds": args.n_seeds}
        for part in ("Q", "R", "all"):
            for metric in ("cos", "rel_l2", "abs_l2"):
                v = np.array([p[part][metric] for p in per])
                agg[f"{metric}_{part}"] = {"mean": float(v.mean()), "std": float(v.std()),
                                           "median": float(np.median(v)), "min": float(v.min()),
                                           "max": float(v.max())}
        out[f"{tol:.0e}"] = agg
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--tolerances", type=float, nargs="+", default=[1e-3, 1e-5, 1e-7])
    ap.add_argument("--n_seeds", type=int, default=10)
    ap.add_argument("--batch_size", type=int, default=64)
    ap.add_argument("--horizon", type=int, default=40)
    ap.add_argument("--sim_steps", type=int, default=50)
    ap.add_argument("--n_state", type=int, default=8)
    ap.add_argument("--n_ctrl", type=int, default=4)
    ap.add_argument("--umax", type=float, default=1.0)
    ap.add_argument("--admm_max_iter", type=int, default=1000)
    ap.add_argument("--fd_eps", type=float, default=1e-5)
    ap.add_argument("--forward", default="b200_direct", help="forward backend (b200 or b200_direct)")
    ap.add_argument("--out", default="", help="write the aggregated results as JSON")
    ap.add_argument("--quiet", action="store_true")
    args = ap.parse_args(argv)
    res = run(args)
    print(json.dumps({"gradient_accuracy": res, "config": vars(args)}))
    if args.out:
        with open(args.out, "w") as f:
            json.dump({"gradient_accuracy": res, "config": vars(args)}, f, indent=1)
    return res


if __name__ == "__main__":
    main()
