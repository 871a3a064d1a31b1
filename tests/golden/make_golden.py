"""Generate tests/golden/*.npz by running the REFERENCE's own CUDA kernels
(admmFusedKernel, pcgBlkTridiSingleBlock — compiled unmodified from the
reference tree by oracle/build_ref.sh) on seeded inputs.  Needs a GPU and
oracle/_ref/libtmpc_refcuda.so:

    bash oracle/build_ref.sh && python tests/golden/make_golden.py [case ...]

(no case names: regenerate every fixture).
S and Phiinv (computed in JAX by the reference before it calls the kernel,
admm.py:719-724) come from the NumPy restatement; the fixtures therefore pin
the kernels' ADMM/PCG semantics, and test_golden.py pins compute_S_Phiinv
against the reference's known answers separately.
"""
import ctypes as C
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import admm_ref as ref  # noqa: E402
from turbompc_b200.problems import synthetic  # noqa: E402

LIB = os.path.join(ROOT, "oracle", "_ref", "libtmpc_refcuda.so")


class RefAdmmArgs(C.Structure):
    _fields_ = ([(k, C.c_void_p) for k in (
        "x_out", "iters_out", "x_blocks_out", "z_g_out", "y_g_out", "y_f_0_out", "y_f_dyn_out", "xi_g_out",
        "rho_bar_out", "kernel_ns_out", "S_work", "Phiinv_work", "S", "Phiinv", "D", "E", "q", "A0", "A_minus",
        "A_plus", "G", "l", "u", "c0", "c", "x0", "z_g0", "y_g0", "y_f_0", "y_f_dyn", "xi_g0", "rho_bar",
        "slack_weight")]
        + [(k, C.c_int32) for k in ("T", "n", "nx", "n0", "m", "Nb", "max_iter", "pcg_max_iter", "check_every",
                                    "adapt_rho_every", "use_slack")]
        + [(k, C.c_double) for k in ("eps_abs", "eps_rel", "sigma", "rho_f_factor", "alpha", "pcg_eps",
                                     "adaptive_rho_tolerance", "rho_min", "rho_max")])


def run_ref_admm(lib, blocks, dt, cfg, rho=0.1, slack=None):
    qo = ref.QP(**{k: np.asarray(v, dtype=np.float64) for k, v in blocks.items()})
    d = qo.dims
    B, T, N, n, nx, n0, m = (d[k] for k in ("B", "T", "N", "n", "nx", "n0", "m"))
    st0 = ref.initial_state(qo, rho)
    S, P = ref.compute_S_Phiinv(qo, st0.rho * cfg["rho_f_factor"], cfg["sigma"], st0.rho)
    tt = torch.float64 if dt == np.float64 else torch.float32
    g = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=tt, device="cuda")
    ins = dict(S=g(S), Phiinv=g(P), D=g(qo.D), E=g(qo.E), q=g(qo.q), A0=g(qo.A0), A_minus=g(qo.Am),
               A_plus=g(qo.Ap), G=g(qo.G), l=g(qo.l), u=g(qo.u), c0=g(qo.c0), c=g(qo.c), x0=g(st0.x),
               z_g0=g(st0.z_g), y_g0=g(st0.y_g), y_f_0=g(st0.y_f0), y_f_dyn=g(st0.y_fdyn), xi_g0=g(st0.xi_g),
               rho_bar=g(st0.rho), slack_weight=g(np.full(B, slack or 0.0)))
    outs = dict(x_out=torch.empty(B, T, n, dtype=tt, device="cuda"),
                iters_out=torch.empty(B, dtype=torch.int32, device="cuda"),
                x_blocks_out=torch.empty(B, T, n, dtype=tt, device="cuda"),
                z_g_out=torch.empty(B, T, m, dtype=tt, device="cuda"),
                y_g_out=torch.empty(B, T, m, dtype=tt, device="cuda"),
                y_f_0_out=torch.empty(B, n0, dtype=tt, device="cuda"),
                y_f_dyn_out=torch.empty(B, N, nx, dtype=tt, device="cuda"),
                xi_g_out=torch.empty(B, T, m, dtype=tt, device="cuda"),
                rho_bar_out=torch.empty(B, dtype=tt, device="cuda"),
                kernel_ns_out=torch.empty(B, dtype=tt, device="cuda"),
                S_work=torch.empty(B, T, n, 4 * n, dtype=tt, device="cuda"),
                Phiinv_work=torch.empty(B, T, n, 3 * n, dtype=tt, device="cuda"))
    a = RefAdmmArgs()
    for k, v in {**ins, **outs}.items():
        setattr(a, k, v.data_ptr() if v.numel() else None)
    for k, v in dict(T=T, n=n, nx=nx, n0=n0, m=m, Nb=B, use_slack=int(slack is not None)).items():
        setattr(a, k, v)
    for k in ("max_iter", "pcg_max_iter", "check_every", "adapt_rho_every"):
        setattr(a, k, int(cfg[k]))
    for k in ("eps_abs", "eps_rel", "sigma", "rho_f_factor", "alpha", "pcg_eps", "adaptive_rho_tolerance",
              "rho_min", "rho_max"):
        setattr(a, k, float(cfg[k]))
    fn = lib.ref_admm_fused_f64 if dt == np.float64 else lib.ref_admm_fused_f32
    rc = fn(C.byref(a), C.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == 0, rc
    res = {k: v.cpu().numpy() for k, v in outs.items() if k not in ("S_work", "Phiinv_work", "kernel_ns_out")}
    return res


CFG = dict(max_iter=50, pcg_max_iter=20, check_every=0, adapt_rho_every=0, eps_abs=0.0, eps_rel=0.0, pcg_eps=0.0,
           sigma=1e-6, rho_f_factor=1000.0, alpha=1.6, adaptive_rho_tolerance=5.0, rho_min=1e-6, rho_max=1e6)


def _problem_qp(kind, batch):
    """First-SQP-iteration QP blocks (float64 NumPy, reference layout) of the
    benchmark problems: the config-3 quadrotor (n = 16, T = 51) or the config-5
    Clohessy-Wiltshire problem with the learned stage cost (n = 9, T = 61)."""
    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    from turbompc_b200.problems.quadrotor import make_quadrotor_problem
    from turbompc_b200.solver import TurboMPCSolver

    if kind == "quadrotor":
        ocp, p = make_quadrotor_problem(batch, N=50, seed=11, dtype=torch.float64, device="cpu")
    else:
        # thrust box tightened to |u| <= 0.01 so that it is active (non-zero y_g)
        ocp, p = make_learned_cost_problem(batch, N=60, seed=12, dtype=torch.float64, device="cpu", u_max=0.01)
    s = TurboMPCSolver(ocp, {"num_sqp_iteration_max": 1})
    g = s.initial_guess(p)
    t = {k: v.numpy() for k, v in s._build_qp_data(g.states, g.controls, p).tensors().items()}
    return dict(D=t["D"], E=t["E"], q=t["q"], A0=t["A0"], Am=t["A_minus"], Ap=t["A_plus"], c0=t["c0"], c=t["c"],
                G=t["G"], l=t["l"], u=t["u"])


def main():
    only = set(sys.argv[1:])
    lib = C.CDLL(LIB)
    cases = {
        "admm_config1_f64": (synthetic.double_integrator(batch=8, N=20), np.float64, dict(CFG), None),
        "admm_config1_f32": (synthetic.double_integrator(batch=8, N=20), np.float32, dict(CFG), None),
        "admm_dense16_f64": (synthetic.random_dense(4, 12, 4, 10, 4, seed=21), np.float64,
                             dict(CFG, max_iter=15, pcg_max_iter=30), None),
        "admm_slack_adapt_f64": (synthetic.random_dense(4, 4, 2, 10, 3, seed=3), np.float64,
                                 dict(CFG, max_iter=60, pcg_max_iter=6, check_every=5, adapt_rho_every=10,
                                      eps_abs=1e-3, eps_rel=1e-3, rho_f_factor=100.0), 10.0),
        # The benchmark shapes in fp32 (30 ADMM x 30 PCG, fixed counts): the
        # register-resident b200 kernel's 52- and 64-stage instances.
        "admm_quadrotor16_f32": (lambda: _problem_qp("quadrotor", 16), np.float32,
                                 dict(CFG, max_iter=30, pcg_max_iter=30), None),
        "admm_cw9_f32": (lambda: _problem_qp("cw", 16), np.float32, dict(CFG, max_iter=30, pcg_max_iter=30), None),
    }
    for name, (blocks, dt, cfg, slack) in cases.items():
        if only and name not in only:
            continue
        if callable(blocks):
            blocks = blocks()
        out = run_ref_admm(lib, blocks, dt, cfg, slack=slack)
        np.savez_compressed(os.path.join(HERE, name + ".npz"),
                            **{"in_" + k: np.asarray(v) for k, v in blocks.items()},
                            **{"out_" + k: v for k, v in out.items()},
                            cfg=np.array(repr(cfg)), slack=np.array(-1.0 if slack is None else slack),
                            dtype=np.array(np.dtype(dt).name))
        print(name, "iters", out["iters_out"][:4])
    # PCG (pcgBlkTridiSingleBlock) on random LTI Schur systems
    for dt in (np.float64, np.float32):
        if only and ("pcg_lti9_" + ("f64" if dt == np.float64 else "f32")) not in only:
            continue
        b = synthetic.random_lti(6, 6, 3, 32, seed=32)
        qo = ref.QP(**b)
        S, P = ref.compute_S_Phiinv(qo, np.full(6, 100.0), 1e-6, np.full(6, 0.1))
        rng = np.random.default_rng(1)
        rhs = rng.normal(size=(6, 33, 9))
        x0 = 0.1 * rng.normal(size=rhs.shape)
        tt = torch.float64 if dt == np.float64 else torch.float32
        g = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=tt, device="cuda")
        xo = torch.empty(6, 33, 9, dtype=tt, device="cuda")
        it = torch.empty(6, dtype=torch.int32, device="cuda")
        gs = [g(S), g(P), g(rhs), g(x0)]
        fn = lib.ref_pcg_f64 if dt == np.float64 else lib.ref_pcg_f32
        fn.argtypes = [C.c_void_p] * 7 + [C.c_double, C.c_int, C.c_int, C.c_int, C.c_int]
        rc = fn(torch.cuda.current_stream().cuda_stream, xo.data_ptr(), it.data_ptr(), *[t.data_ptr() for t in gs],
                0.0, 30, 33, 9, 6)
        torch.cuda.synchronize()
        assert rc == 0
        name = "pcg_lti9_" + ("f64" if dt == np.float64 else "f32")
        np.savez_compressed(os.path.join(HERE, name + ".npz"), S=S, P=P, rhs=rhs, x0=x0, out_x=xo.cpu().numpy(),
                            out_iters=it.cpu().numpy(), dtype=np.array(np.dtype(dt).name))
        print(name, it.cpu().numpy())


if __name__ == "__main__":
    main()
