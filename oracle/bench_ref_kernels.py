"""Time the reference's own CUDA kernels against the b200 kernels on the same
GPU and the same inputs (the GPU bar of the benchmark).

TEST / MEASUREMENT INFRASTRUCTURE: the reference kernels come from
oracle/_ref/libtmpc_refcuda.so (admm_fused.cu, pcg_blktridi.cu and
common/block_tridi.cu compiled unmodified for sm_100a by oracle/build_ref.sh).

    python oracle/bench_ref_kernels.py [--batch 32768] [--reps 3]

Prints one JSON line per comparison:
  * admmFusedKernel (turbompc/solvers/admm/csrc/admm_fused.cu:504) vs
    tmpc_admm_solve_f32 on the configuration-3 quadrotor QPs (fp32, 30 ADMM x
    30 PCG, fixed counts).  The reference receives S and Phiinv precomputed
    (the reference computes them in JAX before the launch, admm.py:719-724);
    that assembly is NOT in its timed region, while the b200 launch assembles
    them itself inside its timed region.
  * pcgBlkTridiSingleBlock (pcg_blktridi.cu:96) vs tmpc_pcg_solve_* (the same
    reference-layout operators) and tmpc_pcg_solve_stream_* (stream layout) on
    configuration-2 points with T*n <= 1024 (the reference's single-CTA path;
    above that it runs a host-synchronised multi-kernel loop sequentially over
    the batch, pcg_blktridi.cu:433-477).
The reference kernel forms per-problem offsets as 32-bit products
(`bid * S_work_stride`, admm_fused.cu:567-585, with S_work_stride = T*n*4n),
so a batch with Nb*T*n*4n >= 2^31 makes it address outside its buffers: at
the configuration-3 shape that is every batch above 41,120 problems (at the
benchmark's 65,536 it raised an illegal-address error on a B200).  This
script refuses such batches for the reference and compares at 32,768.
Timing: CUDA events on the current stream, one warm-up launch, the mean of
`reps` launches; inputs are larger than L2 at the default sizes.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from tests.golden.make_golden import LIB, RefAdmmArgs  # noqa: E402
from turbompc_b200 import _ffi, ops  # noqa: E402
from turbompc_b200.problems import synthetic  # noqa: E402


def _time(fn, reps):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


INT32_MAX = 2 ** 31 - 1


def admm_compare(lib, batch, reps, admm=30, pcg=30):
    from turbompc_b200.problems.quadrotor import make_quadrotor_problem
    from turbompc_b200.solver import TurboMPCSolver

    T, n = 51, 16
    if batch * T * n * 4 * n > INT32_MAX:
        raise SystemExit(f"batch {batch}: the reference kernel's 32-bit offsets overflow above "
                         f"{INT32_MAX // (T * n * 4 * n)} problems (admm_fused.cu:567-585); not launched")

    ocp, p = make_quadrotor_problem(batch, N=50, seed=1000, dtype=torch.float32, device="cuda")
    s = TurboMPCSolver(ocp, {"num_sqp_iteration_max": 1})
    g = s.initial_guess(p)
    qd = s._build_qp_data(g.states, g.controls, p)
    cfg = ops.AdmmConfig(max_iter=admm, pcg_max_iter=pcg, check_every=0, adapt_rho_every=0, eps_abs=0.0,
                         eps_rel=0.0, pcg_eps=0.0)
    s0 = ops.admm_initial_state(qd, 0.1)
    B, T, n, nx, n0, m = qd.Nb, qd.T, qd.n, qd.nx, qd.n0, qd.m
    N = T - 1
    S, P, _ = ops.schur_assemble(qd, s0.rho_bar, cfg.sigma, cfg.rho_f_factor)
    t = qd.tensors()
    e = lambda *sh, dt=torch.float32: torch.empty(*sh, dtype=dt, device="cuda")
    outs = dict(x_out=e(B, T, n), iters_out=e(B, dt=torch.int32), x_blocks_out=e(B, T, n), z_g_out=e(B, T, m),
                y_g_out=e(B, T, m), y_f_0_out=e(B, n0), y_f_dyn_out=e(B, N, nx), xi_g_out=e(B, T, m),
                rho_bar_out=e(B), kernel_ns_out=e(B), S_work=e(B, T, n, 4 * n), Phiinv_work=e(B, T, n, 3 * n))
    ins = dict(S=S, Phiinv=P, D=t["D"], E=t["E"], q=t["q"], A0=t["A0"], A_minus=t["A_minus"], A_plus=t["A_plus"],
               G=t["G"], l=t["l"], u=t["u"], c0=t["c0"], c=t["c"], x0=s0.x_blocks, z_g0=s0.z_g, y_g0=s0.y_g,
               y_f_0=s0.y_f_0, y_f_dyn=s0.y_f_dyn, xi_g0=s0.xi_g, rho_bar=s0.rho_bar,
               slack_weight=torch.zeros(B, device="cuda"))
    a = RefAdmmArgs()
    for k, v in {**ins, **outs}.items():
        setattr(a, k, v.data_ptr() if v.numel() else None)
    for k, v in dict(T=T, n=n, nx=nx, n0=n0, m=m, Nb=B, use_slack=0, max_iter=admm, pcg_max_iter=pcg,
                     check_every=0, adapt_rho_every=0).items():
        setattr(a, k, v)
    for k in ("eps_abs", "eps_rel", "sigma", "rho_f_factor", "alpha", "pcg_eps", "adaptive_rho_tolerance",
              "rho_min", "rho_max"):
        setattr(a, k, float(getattr(cfg, k)))
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def ref_launch():
        rc = lib.ref_admm_fused_f32(C.byref(a), stream)
        if rc != 0:
            raise RuntimeError(f"reference admm launch failed: {rc}")

    out = ops.empty_state_like(s0)
    ws_n = ops.admm_workspace_bytes(qd, cfg)
    ws = torch.empty(max(ws_n, 16), dtype=torch.uint8, device="cuda")
    ms_ref = _time(ref_launch, reps)
    ms_b200 = _time(lambda: ops.admm_solve(qd, s0, cfg, out=out, workspace=ws), reps)
    err = max(_rel(out.x_blocks, outs["x_blocks_out"]), _rel(out.y_g, outs["y_g_out"]),
              _rel(out.y_f_dyn, outs["y_f_dyn_out"]))
    print(json.dumps({"compare": "admm_fused", "workload": f"quadrotor-12 N=50 QPs, batch {B}, fp32, {admm} ADMM x "
                      f"{pcg} PCG (fixed counts)", "reference_kernel": "admmFusedKernel (S/Phiinv precomputed, "
                      "assembly not timed)", "b200_kernel": "tmpc_admm_solve_f32 (assembly inside the launch)",
                      "reference_ms": round(ms_ref, 3), "b200_ms": round(ms_b200, 3),
                      "speedup": round(ms_ref / ms_b200, 2), "reference_solves_per_s": round(B / ms_ref * 1e3, 1),
                      "b200_solves_per_s": round(B / ms_b200 * 1e3, 1), "max_rel_diff_x_yg_yf": err}), flush=True)
    del outs, ins, S, P


def pcg_compare(lib, points, reps, iters=30):
    for nx, nu, N, batch, dt in points:
        tdt = torch.float32 if dt == "f32" else torch.float64
        n, T = nx + nu, N + 1
        if T * n > 1024 or batch * T * n * 3 * n > INT32_MAX:
            print(json.dumps({"compare": "pcg", "nx": nx, "nu": nu, "N": N, "batch": batch,
                              "skipped": "outside the reference's single-CTA path or its 32-bit offsets"}))
            continue
        small = synthetic.to_qpdata(synthetic.random_lti(64, nx, nu, N, seed=1000 + nx + N), dtype=tdt,
                                    device="cuda")
        S64, P64, _ = ops.schur_assemble(small, 0.1, 1e-6, 1000.0)
        rep = (batch + 63) // 64
        S = S64.repeat(rep, 1, 1, 1)[:batch].contiguous()
        P = P64.repeat(rep, 1, 1, 1)[:batch].contiguous()
        g = torch.Generator(device="cuda").manual_seed(7)
        rhs = torch.randn(batch, T, n, generator=g, device="cuda", dtype=tdt)
        x0 = torch.zeros_like(rhs)
        xr = torch.empty_like(rhs)
        it = torch.empty(batch, dtype=torch.int32, device="cuda")
        fn = lib.ref_pcg_f64 if dt == "f64" else lib.ref_pcg_f32
        fn.argtypes = [C.c_void_p] * 7 + [C.c_double, C.c_int, C.c_int, C.c_int, C.c_int]
        stream = torch.cuda.current_stream().cuda_stream

        def ref_launch():
            rc = fn(stream, xr.data_ptr(), it.data_ptr(), S.data_ptr(), P.data_ptr(), rhs.data_ptr(), x0.data_ptr(),
                    0.0, iters, T, n, batch)
            if rc != 0:
                raise RuntimeError(f"reference pcg launch failed: {rc}")

        ms_ref = _time(ref_launch, reps)
        xb = [None]

        def ours_ref_layout():
            xb[0], _ = ops.pcg_solve(S, P, rhs, x0, 0.0, iters)

        ms_ours = _time(ours_ref_layout, reps)
        err = _rel(xb[0], xr)
        del S, P
        o64, _ = ops.schur_assemble_stream(small, 0.1, 1e-6, 1000.0)
        per = o64.numel() // 64
        ob = o64[:64 * per].view(64, per).repeat(rep, 1)[:batch].contiguous().view(-1)
        dims = _ffi.TmpcDims(batch, T, n, nx, 0, 0)
        xs = torch.empty_like(rhs)
        ms_stream = _time(lambda: ops.pcg_solve_stream(ob, dims, rhs, x0, 0.0, iters, x_out=xs), reps)
        err_s = _rel(xs, xr)
        del ob
        print(json.dumps({"compare": "pcg", "nx": nx, "nu": nu, "N": N, "batch": batch, "dtype": dt,
                          "pcg_iters": iters, "reference_kernel": "pcgBlkTridiSingleBlock",
                          "reference_ms": round(ms_ref, 3), "b200_ref_layout_ms": round(ms_ours, 3),
                          "b200_stream_ms": round(ms_stream, 3),
                          "speedup_ref_layout": round(ms_ref / ms_ours, 2),
                          "speedup_stream": round(ms_ref / ms_stream, 2), "max_rel_diff": max(err, err_s)}),
              flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=32768)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--skip-admm", action="store_true")
    ap.add_argument("--pcg-points", default="6,3,32,65536,f32;6,3,64,16384,f32;12,4,32,16384,f32;"
                                            "6,3,32,65536,f64;12,4,32,16384,f64")
    args = ap.parse_args()
    if not os.path.exists(LIB):
        print(json.dumps({"unavailable": f"{LIB} not built (oracle/build_ref.sh)"}))
        return
    lib = C.CDLL(LIB)
    _ffi.load(build_if_missing=False)
    if not args.skip_admm:
        admm_compare(lib, args.batch, args.reps)
    pts = []
    for item in filter(None, args.pcg_points.split(";")):
        f = item.split(",")
        pts.append((int(f[0]), int(f[1]), int(f[2]), int(f[3]), f[4]))
    pcg_compare(lib, pts, args.reps)


if __name__ == "__main__":
    main()
