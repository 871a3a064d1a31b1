"""Parity pins against the reference itself: tests/golden/*.npz hold outputs
of the reference's own admmFusedKernel / pcgBlkTridiSingleBlock (compiled
unmodified from the reference sources, run on a B200 by
tests/golden/make_golden.py).  The CPU tests pin the NumPy oracle; the GPU
tests compare the B200 kernels directly with the reference's outputs."""
import ast
import glob
import os

import numpy as np
import pytest
import torch

from oracle import admm_ref as ref
from tests.helpers import rel_err

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ADMM_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "admm_*.npz")))
PCG_CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(HERE, "pcg_*.npz")))
KEYS = (("x_out", "x"), ("z_g_out", "z_g"), ("y_g_out", "y_g"), ("y_f_0_out", "y_f0"), ("y_f_dyn_out", "y_fdyn"),
        ("xi_g_out", "xi_g"), ("rho_bar_out", "rho"))


def _load(name):
    z = np.load(os.path.join(HERE, name + ".npz"))
    return {k: z[k] for k in z.files}


def _tol(dt):
    return 1e-6 if dt == "float64" else 1e-3


def _oracle_qp(f, dt):
    blocks = {k[3:]: f[k].astype(dt) for k in f if k.startswith("in_")}
    sw = float(f["slack"])
    use = sw >= 0
    return ref.QP(**blocks, slack_weight=np.full(blocks["D"].shape[0], max(sw, 0.0), dtype=dt), use_slack=use)


def test_golden_fixtures_present():
    assert len(ADMM_CASES) >= 4 and len(PCG_CASES) >= 2


@pytest.mark.parametrize("name", ADMM_CASES)
def test_oracle_matches_reference_fused_admm(name):
    f = _load(name)
    dt = np.dtype(str(f["dtype"]))
    cfg = ast.literal_eval(str(f["cfg"]))
    qp = _oracle_qp(f, dt)
    c = ref.ADMMConfig(**{k: cfg[k] for k in ("max_iter", "pcg_max_iter", "check_every", "eps_abs", "eps_rel",
                                              "sigma", "rho_f_factor", "alpha", "pcg_eps", "adapt_rho_every",
                                              "adaptive_rho_tolerance", "rho_min", "rho_max")},
                      use_slack=qp.use_slack)
    st, it = ref.admm_solve(qp, ref.initial_state(qp, 0.1), c)
    assert (it == f["out_iters_out"]).all(), (it, f["out_iters_out"])
    for gk, ok in KEYS:
        assert rel_err(getattr(st, ok), f["out_" + gk]) < _tol(str(dt)), gk


@pytest.mark.parametrize("name", PCG_CASES)
def test_oracle_matches_reference_pcg(name):
    f = _load(name)
    dt = np.dtype(str(f["dtype"]))
    x, it = ref.pcg(f["S"].astype(dt), f["P"].astype(dt), f["rhs"].astype(dt), f["x0"].astype(dt), 30, 0.0)
    assert (it == f["out_iters"]).all()
    assert rel_err(x, f["out_x"]) < _tol(str(dt))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ADMM_CASES)
def test_b200_fused_admm_matches_reference_kernel(name):
    from turbompc_b200 import ops
    from turbompc_b200.problems import synthetic

    f = _load(name)
    dt = str(f["dtype"])
    tdt = torch.float64 if dt == "float64" else torch.float32
    cfg = ast.literal_eval(str(f["cfg"]))
    sw = float(f["slack"])
    use = sw >= 0
    blocks = {k[3:]: f[k] for k in f if k.startswith("in_")}
    Nb = blocks["D"].shape[0]
    qd = synthetic.to_qpdata(blocks, dtype=tdt, device="cuda")
    c = ops.AdmmConfig(**{k: cfg[k] for k in ("max_iter", "pcg_max_iter", "check_every", "eps_abs", "eps_rel",
                                              "sigma", "rho_f_factor", "alpha", "pcg_eps", "adapt_rho_every",
                                              "adaptive_rho_tolerance", "rho_min", "rho_max")}, use_slack=use)
    out, it, st = ops.admm_solve(qd, ops.admm_initial_state(qd, 0.1), c,
                                 slack_weight=np.full(Nb, sw) if use else None)
    assert (it.cpu().numpy() == f["out_iters_out"]).all()
    got = dict(zip(("x", "y_g", "y_f0", "y_fdyn", "z_g", "xi_g", "rho"), [t.cpu().numpy() for t in out]))
    for gk, ok in KEYS:
        assert rel_err(got[ok], f["out_" + gk]) < _tol(dt), gk


@pytest.mark.gpu
@pytest.mark.parametrize("name", PCG_CASES)
def test_b200_pcg_matches_reference_kernel(name):
    from turbompc_b200 import ops

    f = _load(name)
    dt = str(f["dtype"])
    tdt = torch.float64 if dt == "float64" else torch.float32
    g = lambda a: torch.as_tensor(a, dtype=tdt, device="cuda")
    x, it = ops.pcg_solve(g(f["S"]), g(f["P"]), g(f["rhs"]), g(f["x0"]), 0.0, 30)
    assert (it.cpu().numpy() == f["out_iters"]).all()
    assert rel_err(x.cpu().numpy(), f["out_x"]) < _tol(dt)
