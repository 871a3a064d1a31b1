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
