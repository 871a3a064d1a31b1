"""Shared test helpers: problem builders and the relative error metric."""
import numpy as np

from oracle import admm_ref as ref
from turbompc_b200.problems import synthetic


def oracle_qp(blocks, dtype=np.float64, slack_weight=None, use_slack=False):
    kw = {k: np.asarray(v, dtype=dtype) for k, v in blocks.items()}
    sw = None if slack_weight is None else np.asarray(slack_weight, dtype=dtype)
    return ref.QP(**kw, slack_weight=sw, use_slack=use_slack)


def rel_err(a, b, tiny=1e-30):
    """||a - b||_inf / max(||b||_inf, tiny) (the parity metric)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if b.size == 0:
        return 0.0
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), tiny))


def dense_blocks(batch, nx, nu, N, m, seed=0):
    return synthetic.random_dense(batch, nx, nu, N, m, seed=seed)


def oracle_admm_solve(qp, state0, cfg, slack_weight=None, out=None, workspace=None):
    """Drop-in for turbompc_b200.ops.admm_solve backed by the NumPy oracle in
    fp64 (test infrastructure: runs the SQP loop with the oracle's ADMM so the
    GPU kernels can be compared with it inside whole solves)."""
    import torch
    from turbompc_b200.ops import ADMMState as TState
    t = qp.tensors()
    f = lambda a: a.detach().cpu().numpy().astype(np.float64)
    sw = None if slack_weight is None else f(torch.as_tensor(slack_weight).expand(qp.Nb))
    q = ref.QP(D=f(t["D"]), E=f(t["E"]), q=f(t["q"]), A0=f(t["A0"]), Am=f(t["A_minus"]), Ap=f(t["A_plus"]),
               c0=f(t["c0"]), c=f(t["c"]), G=f(t["G"]), l=f(t["l"]), u=f(t["u"]), slack_weight=sw,
               use_slack=bool(cfg.use_slack))
    s = ref.ADMMState(x=f(state0.x_blocks), y_g=f(state0.y_g), y_f0=f(state0.y_f_0), y_fdyn=f(state0.y_f_dyn),
                      z_g=f(state0.z_g), xi_g=f(state0.xi_g), rho=f(state0.rho_bar))
    rc = ref.ADMMConfig(max_iter=cfg.max_iter, pcg_max_iter=cfg.pcg_max_iter, check_every=cfg.check_every,
                        eps_abs=cfg.eps_abs, eps_rel=cfg.eps_rel, sigma=cfg.sigma, rho_f_factor=cfg.rho_f_factor,
                        alpha=cfg.alpha, pcg_eps=cfg.pcg_eps, use_slack=bool(cfg.use_slack),
                        adapt_rho_every=cfg.adapt_rho_every, adaptive_rho_tolerance=cfg.adaptive_rho_tolerance,
                        rho_min=cfg.rho_min, rho_max=cfg.rho_max)
    so, it = ref.admm_solve(q, s, rc)
    dev, dt = state0.x_blocks.device, state0.x_blocks.dtype
    g = lambda a: torch.as_tensor(a, dtype=dt, device=dev)
    st = TState(g(so.x), g(so.y_g), g(so.y_f0), g(so.y_fdyn), g(so.z_g), g(so.xi_g), g(so.rho))
    return st, torch.as_tensor(it, dtype=torch.int64, device=dev), torch.zeros(qp.Nb, dtype=torch.int32, device=dev)


def wide_problem(batch, nx, nu, N, m, seed):
    """Stable LTI dynamics (A = I + 0.1 G, the configuration-2 generator) with
    every QP term non-zero: q, c, a small coupling E (P stays positive
    definite) and m general G rows with |G z| <= 1; well conditioned at wide
    blocks (cond(S) ~ 1e2 at n = 48..96), unlike random_dense, whose random
    dynamics grow along the horizon at nx = 32."""
    rng = np.random.default_rng(seed)
    b = synthetic.random_lti(batch, nx, nu, N, seed=seed)
    n, T = nx + nu, N + 1
    b["q"] = rng.normal(size=(batch, T, n))
    b["c"] = 0.1 * rng.normal(size=(batch, N, nx))
    b["E"] = 0.02 * rng.normal(size=(batch, N, n, n)) / np.sqrt(n)
    b["G"] = rng.normal(size=(batch, T, m, n)) / np.sqrt(n)
    b["l"] = -np.ones((batch, T, m))
    b["u"] = np.ones((batch, T, m))
    return b
