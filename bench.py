"""Benchmark: MPC solves/sec, quadrotor N=50, batch 65536 (benchmark configuration 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

A step is one full SQP solve (5 SQP x 30 ADMM, fixed counts) of the whole
batch.  Each ADMM iteration's linear system is solved exactly by the block
Cholesky factor (``--backend direct``, the default: forward backend
"b200_direct", the drop-in for the reference's default admm_fused_cudss,
turbompc/solvers/turbompc_solver.py:309) or by 30 PCG iterations
(``--backend pcg``: "b200", the drop-in for admm_fused_pcg); the default run
also reports the PCG variant of the same workload inside its line.  For N > 1 (one process per GPU under torchrun) the 65536
problems are split into contiguous shards (strong scaling, no collective on
the data path); the step time is the max over ranks.  Rank 0 prints one JSON
line.  ``--impl reference`` times the CPU restatement of the reference's
algorithm (oracle/, the reference's JAX CPU install is not available) on the
host cores for the same workload (bounded sample, scaled).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SQP, ADMM, PCG = 5, 30, 30
N_HORIZON, BATCH = 50, 65536
METRIC = "MPC solves/sec (quadrotor N=50, batch 65536)"
# DRAM bytes (read + write) per problem of one fused ADMM launch on this
# workload, from the ncu capture summarised in
# profiles/admm_rows_quadrotor_b592_fp32.txt (592 problems, scaled per problem:
# the kernel reads each problem's QP once and writes its state once, so the
# traffic grows in proportion to the problems processed).
NCU_DRAM_BYTES_PER_PROBLEM = 257.2e3
# DRAM bytes (read + write) per problem of one launch of il_admm_kernel (the
# 30 ADMM iterations of the direct path), from the ncu capture summarised in
# profiles/il_admm_quadrotor_b8192_fp32.txt (8192 problems; 48.84 GB; the compact
# variant: A+ = [-I 0], the unit rows of G and the zero rows of W detected, so
# none of them is streamed).
NCU_DIRECT_DRAM_BYTES_PER_PROBLEM = 5.962e6


def direct_bytes_per_problem_iteration(T, n, nx, m, n0, w, ap_identity=False, g_select=False, w_rows=None):
    """Bytes one problem must move in one ADMM iteration of the interleaved
    direct path (il_admm_kernel): the factor read in both sweeps (L_t^-1
    packed and W_t: E_f = T n(n+1)/2 + N n^2 values, twice), the QP rows of
    the iteration (A-, A+, G, q, c, l, u) once, and the state it updates
    (x, y_fdyn, z_g, y_g read and written; gamma and the forward-sweep vector
    y written once and read once).  With ap_identity (A+_t = [-I 0], which the
    kernel detects and then does not stream) A+ is not counted, with g_select
    (every inequality row a unit vector on the same columns in every stage,
    likewise detected) G is not counted.  w_rows: the rows of each W_t that
    are not exact zeros (nx when the rows of Phi_t for stage t+1's controls
    vanish, which the library detects after each factor; n otherwise): only
    those rows are read."""
    N = T - 1
    wr = n if w_rows is None else w_rows
    ef = T * n * (n + 1) // 2 + N * wr * n
    rows = (1 if ap_identity else 2) * N * nx * n + (0 if g_select else T * m * n)
    vecs = T * n + N * nx + 2 * T * m
    state = 2 * (T * n + N * nx + 2 * T * m) + 2 * T * n + 2 * T * n
    return w * (2 * ef + rows + vecs + state)


def direct_launches_per_solve(n0, m, check_every=0, compact=True):
    """Kernel launches of one direct-path ADMM call (fixed counts): scalars in,
    the structure checks of A+ and G (G: its columns, then the rows), the
    interleaving of each non-empty QP / state array (A+ and G launch and exit
    for structured groups), assembly, factor, the zero-row check of W, first
    gamma, the iteration kernel (compact and full variants: two launches in
    fp32), the conversions back, scalars out."""
    conv_in = 6 + (3 if n0 else 0) + (6 if m else 0)  # q A- A+ c x y_fdyn; A0 c0 y_f0; G l u z_g y_g xi_g
    conv_out = 2 + (1 if n0 else 0) + (3 if m else 0)
    checks = 1 + (2 if m else 0)
    return 1 + checks + conv_in + 4 + (2 if compact else 1) + conv_out + 1


def algorithmic_bytes_per_problem_launch(T, n, nx, m, n0, w, admm=ADMM, pcg=PCG):
    """Bytes one problem moves in one ADMM solve (one SQP iteration) under the
    streaming model: B_pcg = 2(2T-1)n^2 w per PCG iteration, B_admm per ADMM
    iteration, plus reading the QP and writing S / Phiinv once."""
    N = T - 1
    b_pcg = 2 * (2 * T - 1) * n * n * w
    b_admm = w * (2 * N * nx * n + T * m * n + T * n + N * nx + n0 * n + n0 + 2 * T * m)
    b_sqp = w * (T * n * n + N * n * n + 2 * N * nx * n + T * m * n + nx * n + T * n + N * nx + 2 * T * m) + b_pcg
    return admm * (pcg * b_pcg + b_admm) + b_sqp


def rows_kernel_flops_per_problem(T, n, nx, m, n0, admm=ADMM, pcg=PCG):
    """Floating-point operations one problem costs the fused register-resident
    ADMM kernel in one launch (one SQP iteration), counted from its code at
    the problem's true block size n (padding excluded):
      per PCG iteration   six n x n block-row products per stage (Theta^-1 r,
                          the two off-diagonal blocks of S on w, Theta^-1 u,
                          the two off-diagonal blocks on z) = 12 T n^2, plus
                          the two inner products and the x, r, p, s updates;
      per ADMM iteration  the PCG set-up (S x, one preconditioner application,
                          one S z: 9 block products = 18 T n^2), gamma
                          (C^T and G^T products), the constraint products
                          C x and G x, relaxation and dual updates;
      per launch          the operator build: Theta (G^T G and A^T A terms),
                          Theta^-1 (Gauss-Jordan, 2 n^3 per stage), Phi."""
    N = T - 1
    f_pcg = 12 * T * n * n + 16 * T * n
    f_setup = 18 * T * n * n + 8 * T * n
    f_admm = 8 * N * nx * n + 4 * T * m * n + 4 * n0 * n + 20 * T * n + 12 * T * m + 6 * N * nx
    f_build = T * (2 * m * n * n + 2 * n ** 3) + 6 * N * nx * n * n + 2 * n0 * n * n
    return admm * (pcg * f_pcg + f_setup + f_admm) + f_build


def fp32_peak_tflops():
    """FP32 CUDA-core peak of one B200 (148 SMs x 128 FP32 lanes x 2 flop per
    FMA x the maximum SM clock); MEASURED_PEAKS.json holds no FP32 figure, so
    this is the nominal number at its measured maximum clock."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            mhz = float(json.load(f)["sm_max_mhz"])
    except (OSError, KeyError, ValueError):
        mhz = 1965.0
    return 148 * 128 * 2 * mhz * 1e6 / 1e12


# Shared-memory pipe share (l1tex data-pipe wavefronts, % of peak) of the
# fused kernel on this workload, from the ncu capture summarised in
# profiles/admm_rows_quadrotor_b592_fp32.txt.
NCU_SMEM_PIPE_SHARE = 0.502


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def pcg_roofline(T, n, nx, m, n0, shard, kms, hbm):
    """Roofline object of the register-resident PCG kernel (on-chip bound)."""
    flops = rows_kernel_flops_per_problem(T, n, nx, m, n0) * shard
    achieved = flops / (kms / 1e3) / 1e12
    fpk = fp32_peak_tflops()
    model_gbs = algorithmic_bytes_per_problem_launch(T, n, nx, m, n0, 4) * shard / (kms / 1e3) / 1e9
    dram = NCU_DRAM_BYTES_PER_PROBLEM * shard
    kernel = "admm_rows_kernel" if (T <= 64 and 8 < n <= 16) else "admm_fused_kernel"
    return {
        "bound": "fp32", "achieved": achieved, "peak": fpk, "unit": "TFLOP/s", "frac": achieved / fpk,
        "peak_source": "nominal FP32 CUDA-core peak (148 SMs x 128 lanes x 2 x max SM clock); "
                       "MEASURED_PEAKS.json has no FP32 figure",
        "traffic": dram, "kernel": kernel, "kernel_ms_per_launch": kms,
        "flops_per_problem_launch": flops / shard, "smem_pipe_share": NCU_SMEM_PIPE_SHARE,
        "dram_frac": dram / (kms / 1e3) / 1e9 / hbm, "model_frac": model_gbs / hbm,
        "note": "the operators stay on chip (registers and shared memory), so the kernel is bound on chip, not by "
                "HBM: frac = its own FP32 flops (counted from the code at the true block size) per launch time over "
                "the FP32 peak; smem_pipe_share = shared-memory pipe share from ncu; traffic = measured DRAM bytes "
                "per launch (ncu, scaled per problem); dram_frac = that traffic over the launch time as a share of "
                "the measured HBM copy peak; model_frac = the streaming model's bytes (S and Phiinv re-read every "
                "PCG iteration) per launch time over that peak, > 1 because those bytes are never moved"}


def direct_roofline(T, n, nx, m, n0, shard, ims, kms, hbm, pk_kind, ap_identity=False, g_select=False,
                    w_rows=None):
    """Roofline object of the interleaved direct path's iteration kernel
    (il_admm_kernel, HBM bound): algorithmic bytes of its ADMM iterations
    over its launch time (CUDA events recorded by the library on the launch
    stream, tmpc_admm_iteration_timing)."""
    bytes_launch = ADMM * direct_bytes_per_problem_iteration(T, n, nx, m, n0, 4, ap_identity, g_select,
                                                             w_rows) * shard
    achieved = bytes_launch / (ims / 1e3) / 1e9
    return {
        "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
        "peak_source": f"{pk_kind} HBM copy bandwidth (MEASURED_PEAKS.json)",
        "traffic": NCU_DIRECT_DRAM_BYTES_PER_PROBLEM * shard, "kernel": "il_admm_kernel",
        "kernel_ms_per_launch": ims, "algorithmic_bytes_per_launch": bytes_launch,
        "call_ms": kms, "call_frac_of_kernel": ims / kms, "a_plus_streamed": not ap_identity, "g_streamed": not g_select,
        "w_rows_read": n if w_rows is None else w_rows,
        "note": "one launch = the 30 ADMM iterations of one SQP iteration for the whole shard; algorithmic bytes = "
                "per ADMM iteration the block-Cholesky factor read in both sweeps, the QP rows (A-, A+, G, q, c, "
                "l, u) once and the updated state; traffic = measured DRAM bytes of that kernel (ncu, 8192 "
                "problems, scaled per problem); call_ms = the whole ADMM call including the layout conversion, "
                "assembly and factor"}


def pcg_variant(ocp, params, sp, batch, steps=2, warmup=1):
    """The headline workload with 30 PCG iterations per ADMM iteration
    (forward backend "b200"), device-timed, with the PCG kernel's roofline."""
    import torch

    from turbompc_b200 import ops
    from turbompc_b200.solver import TurboMPCSolver

    solver = TurboMPCSolver(ocp, sp, forward_backend="b200")
    guess = solver.initial_guess(params)
    for _ in range(warmup):
        solver.solve(guess, params)
    orig = ops.admm_solve
    launch = []

    def timed(*a, **k):
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        out = orig(*a, **k)
        e1.record()
        launch.append((e0, e1))
        return out

    import turbompc_b200.solver as solver_mod

    solver_mod.ops.admm_solve = timed
    try:
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(True), torch.cuda.Event(True)
        s0.record()
        for _ in range(steps):
            solver.solve(guess, params)
        s1.record()
        torch.cuda.synchronize()
    finally:
        solver_mod.ops.admm_solve = orig
    ms = s0.elapsed_time(s1) / steps
    kms = sum(a.elapsed_time(b) for a, b in launch) / len(launch)
    qp = solver._build_qp_data(guess.states, guess.controls, params)
    hbm, _ = peaks()
    return {"config": f"quadrotor N={N_HORIZON} batch {batch}, {SQP} SQP x {ADMM} ADMM x {PCG} PCG (forward "
                      "backend b200, drop-in for admm_fused_pcg)", "metric": "MPC solves/sec",
            "value": batch / (ms / 1e3), "unit": "solves/s", "ms_per_step": ms, "dtype": "f32", "n_gpus": 1,
            "roofline": pcg_roofline(qp.T, qp.n, qp.nx, qp.m, qp.n0, batch, kms, hbm)}


def cpu_baseline(target_s=8.0, seed=0, runs=3, backend="direct"):
    """CPU baseline: the C restatement of the reference's ADMM (oracle/c, the
    reference's own JAX CPU install is unavailable) on all host cores, on the
    QPs of the first SQP iteration of this workload (fp32, 30 ADMM iterations,
    each with the direct block-Cholesky solve or with 30 PCG iterations as the
    GPU arm), scaled by the 5 SQP iterations of a solve.  Linearisation is not
    timed on the CPU side, which flatters the CPU.  The sample is sized so one
    timed run takes about ``target_s`` seconds; the value is the median of
    ``runs`` timed runs on the same sample."""
    import torch

    from oracle import admm_ref as ref
    from oracle import c_oracle
    from turbompc_b200.problems.quadrotor import make_quadrotor_problem
    from turbompc_b200.solver import TurboMPCSolver

    threads = c_oracle.max_threads()

    def qp_sample(k):
        ocp, p = make_quadrotor_problem(k, N=N_HORIZON, seed=seed, dtype=torch.float32, device="cpu")
        s = TurboMPCSolver(ocp, {"num_sqp_iteration_max": SQP})
        g = s.initial_guess(p)
        t = {kk: v.numpy() for kk, v in s._build_qp_data(g.states, g.controls, p).tensors().items()}
        return ref.QP(D=t["D"], E=t["E"], q=t["q"], A0=t["A0"], Am=t["A_minus"], Ap=t["A_plus"], c0=t["c0"],
                      c=t["c"], G=t["G"], l=t["l"], u=t["u"])

    def timed(q):
        t0 = time.perf_counter()
        c_oracle.admm_fixed(q, 0.1, ADMM, -1 if backend == "direct" else PCG, threads=threads)
        return time.perf_counter() - t0

    k = threads
    dt = timed(qp_sample(k))
    k = int(min(65536, max(k, k * target_s / max(dt, 1e-3))))
    q = qp_sample(k)
    times = [timed(q) for _ in range(runs)]
    dt = statistics.median(times)
    return {"value": k / (dt * SQP), "unit": "solves/s", "cores": threads, "kind": "port",
            "sample": f"{k} quadrotor QPs x 1 SQP iteration (30 ADMM, {linsys_label(backend)}, fp32, C restatement "
                      "in oracle/c, "
                      f"{threads} host threads), scaled x{SQP} SQP iterations; median of {runs} runs "
                      f"({', '.join(f'{t:.1f}' for t in times)} s)"}


def linsys_label(backend):
    return ("direct block-Cholesky solve per ADMM iteration" if backend == "direct"
            else f"{PCG} PCG iterations per ADMM iteration")


def workload_config(batch, world, shard, backend="direct"):
    """The `config` object of both arms' JSON lines."""
    return {"workload": f"quadrotor-12 N={N_HORIZON} batch {batch}, {SQP} SQP x {ADMM} ADMM, "
                        f"{linsys_label(backend)} (fixed counts)",
            "backend": ("b200_direct (drop-in for admm_fused_cudss, the reference's default)" if backend == "direct"
                        else "b200 (drop-in for admm_fused_pcg)"),
            "global_batch": batch, "per_gpu_batch": shard, "horizon": N_HORIZON, "parallelism": f"batch-shard x{world}"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    cb = cpu_baseline(runs=max(3, args.steps), backend=args.backend)
    cfg = workload_config(args.batch, 1, args.batch, args.backend)
    cfg["l2"] = "CPU run (no GPU); sample in cpu_baseline.sample"
    line = {"metric": METRIC, "value": cb["value"], "unit": "solves/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": args.batch / cb["value"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": cfg, "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "solves/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def admm_only(nb, linsys="auto", reps=3, pcg=PCG, admm=ADMM):
    """One warm-up and `reps` timed fused ADMM launches (30 ADMM x 30 PCG, fp32)
    on nb quadrotor-shaped LTI QPs; prints ms per launch (CUDA events)."""
    import torch

    from turbompc_b200 import _ffi, ops
    from turbompc_b200.problems import synthetic

    b = synthetic.random_lti(nb, 12, 4, N_HORIZON, seed=0)
    qd = synthetic.to_qpdata(b, dtype=torch.float32, device="cuda")
    ls = {"auto": _ffi.LINSYS_PCG, "packed": _ffi.LINSYS_PCG_PACKED, "direct": _ffi.LINSYS_DIRECT}[linsys]
    cfg = ops.AdmmConfig(max_iter=admm, pcg_max_iter=pcg, check_every=0, adapt_rho_every=0, eps_abs=0.0,
                         eps_rel=0.0, pcg_eps=0.0, linsys=ls)
    s0 = ops.admm_initial_state(qd, 0.1)
    out, it, st = ops.admm_solve(qd, s0, cfg)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        ops.admm_solve(qd, s0, cfg, out=out)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    print(json.dumps({"admm_only": nb, "linsys": linsys, "admm_iters": admm, "pcg_iters": pcg, "ms_per_launch": round(ms, 3),
                      "us_per_problem": round(1e3 * ms / nb, 3), "status_nonzero": int((st != 0).sum())}))


def il_only(point, reps=2):
    """Profiling aid: the batch-interleaved factor and solve of one LTI point
    ('nx,nu,N,batch,dtype'), `reps` launches each after one warm-up, timed
    with CUDA events (one JSON line)."""
    import torch

    from turbompc_b200 import _ffi, ops
    from turbompc_b200.problems import synthetic

    f = point.split(",")
    nx, nu, N, batch, dt = int(f[0]), int(f[1]), int(f[2]), int(f[3]), f[4]
    tdt = torch.float32 if dt == "f32" else torch.float64
    n, T = nx + nu, N + 1
    small = synthetic.to_qpdata(synthetic.random_lti(64, nx, nu, N, seed=1000 + nx + N), dtype=tdt, device="cuda")
    S, _, _ = ops.schur_assemble(small, 0.1, 1e-6, 1000.0)
    S = S.repeat((batch + 63) // 64, 1, 1, 1)[:batch].contiguous()
    dims = _ffi.TmpcDims(batch, T, n, nx, 0, 0)
    ops_il = ops.schur_interleave(S)
    del S
    g = torch.Generator(device="cuda").manual_seed(7)
    rhs_il = ops.interleave(torch.randn(batch, T, n, generator=g, device="cuda", dtype=tdt))
    fac, st = ops.riccati_factor_il(ops_il, dims)
    x = ops.riccati_solve_il(fac, dims, rhs_il)
    torch.cuda.synchronize()
    e0, e1, e2 = torch.cuda.Event(True), torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record()
    for _ in range(reps):
        ops.riccati_factor_il(ops_il, dims, fac, st)
    e1.record()
    for _ in range(reps):
        ops.riccati_solve_il(fac, dims, rhs_il, x)
    e2.record()
    torch.cuda.synchronize()
    print(json.dumps({"il_only": point, "factor_ms": e0.elapsed_time(e1) / reps, "solve_ms": e1.elapsed_time(e2) / reps,
                      "status_nonzero": int((st != 0).sum())}))


def pcg_sweep(points, reps=5, pcg_iters=PCG, emit=None):
    """Config 2 (linear-system kernel sweep): standalone PCG (fixed iterations,
    tol 0) on assembled packed operators and the direct block-Cholesky solve,
    timed with CUDA events and reported against the HBM roofline with the
    streaming model B_pcg = 2(2T-1)n^2 w per PCG iteration (factor:
    read S + write the factor; solve: read the factor).  Operators of 64
    seeded LTI problems are tiled to the batch (same values, distinct memory)."""
    import torch

    from turbompc_b200 import _ffi, ops
    from turbompc_b200.problems import synthetic

    emit = emit or (lambda d: print(json.dumps(d), flush=True))
    peak, pk_kind = peaks()
    for (nx, nu, N, batch, dt) in points:
        tdt = torch.float32 if dt == "f32" else torch.float64
        w = 4 if dt == "f32" else 8
        n, T = nx + nu, N + 1
        small = synthetic.to_qpdata(synthetic.random_lti(64, nx, nu, N, seed=1000 + nx + N), dtype=tdt,
                                    device="cuda")
        dims = _ffi.TmpcDims(batch, T, n, nx, 0, 0)
        g = torch.Generator(device="cuda").manual_seed(7)
        rhs = torch.randn(batch, T, n, generator=g, device="cuda", dtype=tdt)
        x0 = torch.zeros_like(rhs)
        b_pcg = 2 * (2 * T - 1) * n * n * w
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        for kind in ("stream", "packed"):
            if kind == "stream":
                o64, st = ops.schur_assemble_stream(small, 0.1, 1e-6, 1000.0)
                solve = ops.pcg_solve_stream
            else:
                o64, st = ops.schur_assemble_packed(small, 0.1, 1e-6, 1000.0)
                solve = ops.pcg_solve_packed
            per = o64.numel() // 64
            opsb = o64[:64 * per].view(64, per).repeat((batch + 63) // 64, 1)[:batch].contiguous().view(-1)
            try:
                x, it = solve(opsb, dims, rhs, x0, 0.0, pcg_iters)
            except Exception as exc:  # e.g. the packed kernel's vectors exceed shared memory
                emit(({"sweep": "pcg_" + kind, "nx": nx, "nu": nu, "N": N, "batch": batch, "dtype": dt,
                                  "unavailable": str(exc)}))
                del opsb
                continue
            torch.cuda.synchronize()
            e0.record()
            for _ in range(reps):
                solve(opsb, dims, rhs, x0, 0.0, pcg_iters)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            gbs = batch * pcg_iters * b_pcg / (ms / 1e3) / 1e9
            line = {"sweep": "pcg_" + kind, "nx": nx, "nu": nu, "N": N, "batch": batch, "dtype": dt,
                    "pcg_iters": pcg_iters, "iters_ok": bool((it == pcg_iters).all()), "ms": round(ms, 3),
                    "solves_per_s": round(batch / (ms / 1e3), 1), "model_GBps": round(gbs, 1),
                    "frac_of_peak": round(gbs / peak, 3), "peak": peak, "peak_source": pk_kind}
            emit(line)
            del opsb
        # direct solve on reference-layout S
        S, P, _ = ops.schur_assemble(small, 0.1, 1e-6, 1000.0)
        Sb = S.repeat((batch + 63) // 64, 1, 1, 1)[:batch].contiguous()
        del P
        fac, fst = ops.riccati_factor(Sb)
        xr = ops.riccati_solve(fac, rhs)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):  # preallocated outputs: no allocation inside the timed region
            ops.riccati_factor(Sb, fac, fst)
        e1.record()
        torch.cuda.synchronize()
        ms_f = e0.elapsed_time(e1) / reps
        e0.record()
        for _ in range(reps):
            ops.riccati_solve(fac, rhs, xr)
        e1.record()
        torch.cuda.synchronize()
        ms_s = e0.elapsed_time(e1) / reps
        b_f = (T * n * 3 * n + (2 * T - 1) * n * n) * w  # read S (reference layout) + write the factor
        b_s = (2 * T - 1) * n * n * w + 2 * T * n * w
        emit(({"sweep": "riccati", "nx": nx, "nu": nu, "N": N, "batch": batch, "dtype": dt,
                          "factor_ms": round(ms_f, 3), "solve_ms": round(ms_s, 3),
                          "factor_model_GBps": round(batch * b_f / (ms_f / 1e3) / 1e9, 1),
                          "solve_model_GBps": round(batch * b_s / (ms_s / 1e3) / 1e9, 1),
                          "status_nonzero": int((fst != 0).sum())}))
        if n <= (16 if dt == "f32" else 12):
            # the same factor / solve on the batch-interleaved layout (one
            # problem per thread, coalesced across problems)
            ops_il = ops.schur_interleave(Sb)
            rhs_il = ops.interleave(rhs)
            fil, sil = ops.riccati_factor_il(ops_il, dims)
            xil = ops.riccati_solve_il(fil, dims, rhs_il)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(reps):
                ops.riccati_factor_il(ops_il, dims, fil, sil)
            e1.record()
            torch.cuda.synchronize()
            ms_fi = e0.elapsed_time(e1) / reps
            e0.record()
            for _ in range(reps):
                ops.riccati_solve_il(fil, dims, rhs_il, xil)
            e1.record()
            torch.cuda.synchronize()
            ms_si = e0.elapsed_time(e1) / reps
            eop = T * n * (n + 1) // 2 + N * n * n  # elements per problem of the operator and of the factor
            bf = 2 * eop * w  # read Theta / Phi, write L / W (W_{t-1} re-read from L2)
            bs = (2 * eop + 4 * T * n) * w  # factor read in both sweeps; rhs, y write + read, x write
            xd = ops.deinterleave(xil, (batch, T, n))
            emit(({"sweep": "riccati_interleaved", "nx": nx, "nu": nu, "N": N, "batch": batch, "dtype": dt,
                   "factor_ms": round(ms_fi, 3), "solve_ms": round(ms_si, 3),
                   "factor_GBps": round(batch * bf / (ms_fi / 1e3) / 1e9, 1),
                   "factor_frac_of_peak": round(batch * bf / (ms_fi / 1e3) / 1e9 / peak, 3),
                   "solve_GBps": round(batch * bs / (ms_si / 1e3) / 1e9, 1),
                   "solve_frac_of_peak": round(batch * bs / (ms_si / 1e3) / 1e9 / peak, 3),
                   "speedup_vs_reference_layout": [round(ms_f / ms_fi, 2), round(ms_s / ms_si, 2)],
                   "max_rel_diff_vs_reference_layout":
                       float(((xd - xr).abs().max() / xr.abs().max()).item()),
                   "status_nonzero": int((sil != 0).sum()),
                   "bytes": "factor 2 E w (E = T n(n+1)/2 + N n^2 per problem), solve (2 E + 4 T n) w"}))
            del ops_il, rhs_il, fil, xil, xd
        del Sb, fac


def run_config(name, steps=3, warmup=2, emit=True, backend="direct"):
    """Configs 4 and 5 on one GPU (one JSON line each; the default run above is
    config 3).  obstacles: quadrotor N=40 with 8 spheres per problem, batch
    8192, 10 SQP x 50 ADMM x 30 PCG, each step warm-started from the previous
    solution (states, controls and ADMM state).  cw_mlp: Clohessy-Wiltshire
    with the learned MLP stage cost, N=60, batch 16384, 3 SQP x 50 ADMM x 30
    PCG forward plus the VJP w.r.t. x0, the MLP parameters and A, B (adjoint
    KKT on the GPU).  backend "direct" (the default, as the headline) replaces
    the PCG iterations by the exact block-Cholesky solve of every ADMM linear
    system.  Device time with CUDA events."""
    import torch

    from turbompc_b200.problems.learned_cost import make_learned_cost_problem
    from turbompc_b200.problems.quadrotor import make_obstacle_problem
    from turbompc_b200.solver import TurboMPCSolver

    def fixed(sqp, admm, pcg):
        return {"num_sqp_iteration_max": sqp, "tol_convergence": 0.0,
                "admm": {"max_iter": admm, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": 0.0,
                         "eps_rel": 0.0, "pcg": {"max_iter": pcg, "tol_epsilon": 0.0}}}

    fb = "b200_direct" if backend == "direct" else "b200"
    lin = "direct solve" if backend == "direct" else "30 PCG"
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    if name == "obstacles":
        batch = 8192
        prog, params = make_obstacle_problem(batch, N=40, seed=4, dtype=torch.float32, device="cuda")
        solver = TurboMPCSolver(prog, fixed(10, 50, 30), forward_backend=fb)
        guess = solver.initial_guess(params)
        for _ in range(warmup):
            guess = solver.solve(guess, params)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            guess = solver.solve(guess, params)  # warm start from the previous solve
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        line = {"config": "obstacles (config 4)", "metric": "MPC solves/sec", "value": batch / (ms / 1e3),
                "unit": "solves/s", "ms_per_step": ms, "batch": batch, "horizon": 40, "m": 12,
                "iterations": f"10 SQP x 50 ADMM x {lin}, warm-started", "backend": fb, "dtype": "f32", "n_gpus": 1}
    else:
        batch = 16384
        prog, params = make_learned_cost_problem(batch, N=60, seed=0, dtype=torch.float32, device="cuda")
        solver = TurboMPCSolver(prog, fixed(3, 50, 30), use_full_hessian=True, forward_backend=fb)
        guess = solver.initial_guess(params)
        leaves = {"mlp_W1": params["mlp_W1"], "mlp_b1": params["mlp_b1"], "mlp_w2": params["mlp_w2"],
                  "dynamics_state_dot_params": dict(params["dynamics_state_dot_params"]),
                  "initial_state": params["initial_state"]}

        def fwd_bwd():
            w = {k: (v.detach().clone().requires_grad_(True) if isinstance(v, torch.Tensor) else
                     {kk: vv.detach().clone().requires_grad_(True) for kk, vv in v.items()})
                 for k, v in leaves.items()}
            sol = solver.solve(guess, params, w)
            loss = (sol.states ** 2).sum() + (sol.controls ** 2).sum()
            flat = [w["mlp_W1"], w["mlp_b1"], w["mlp_w2"], w["initial_state"],
                    w["dynamics_state_dot_params"]["A"], w["dynamics_state_dot_params"]["B"]]
            return torch.autograd.grad(loss, flat)

        for _ in range(warmup):
            fwd_bwd()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            with torch.no_grad():
                solver.solve(guess, params)
        e1.record()
        torch.cuda.synchronize()
        ms_f = e0.elapsed_time(e1) / steps
        e0.record()
        for _ in range(steps):
            fwd_bwd()
        e1.record()
        torch.cuda.synchronize()
        ms_fb = e0.elapsed_time(e1) / steps
        line = {"config": "cw_mlp (config 5)", "metric": "MPC solves/sec", "value": batch / (ms_f / 1e3),
                "unit": "solves/s", "forward_ms": ms_f, "forward_plus_vjp_ms": ms_fb,
                "forward_plus_vjp_solves_per_s": batch / (ms_fb / 1e3), "batch": batch, "horizon": 60,
                "iterations": f"3 SQP x 50 ADMM x {lin}; VJP w.r.t. x0, MLP W1 b1 w2, A, B", "backend": fb, "dtype": "f32",
                "n_gpus": 1}
    if emit:
        print(json.dumps(line), flush=True)
    return line


def other_configs():
    """Configurations 4 and 5 and a short configuration-2 sweep on one GPU,
    reported inside the headline line (one JSON line per run)."""
    out = {}
    for name in ("obstacles", "cw_mlp"):
        try:
            out[name] = run_config(name, emit=False)
        except Exception as exc:  # reported, not fatal
            out[name] = {"error": repr(exc)}
    sweep = []
    try:
        pcg_sweep([(6, 3, 32, 65536, "f32"), (12, 4, 64, 16384, "f32"), (24, 8, 128, 4096, "f32"),
                   (24, 8, 128, 2048, "f64")], reps=3, emit=sweep.append)
    except Exception as exc:
        sweep.append({"error": repr(exc)})
    out["lti_sweep"] = sweep
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--backend", default="direct", choices=["direct", "pcg"],
                    help="linear solve of each ADMM iteration: direct (block Cholesky) or 30 PCG iterations")
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="skip the one-GPU runs of configurations 2, 4 and 5 that the default run adds to its line")
    ap.add_argument("--admm-only", type=int, default=0, metavar="NB",
                    help="profiling aid: one fused ADMM launch (30 ADMM x 30 PCG, fp32) on NB quadrotor-shaped "
                         "synthetic QPs, then exit")
    ap.add_argument("--admm-linsys", default="auto", choices=["auto", "packed", "direct"],
                    help="with --admm-only: auto (register-resident kernel where it applies), the packed kernel, or the direct (block-Cholesky) solve")
    ap.add_argument("--admm-pcg", type=int, default=PCG, help="with --admm-only: PCG iterations per ADMM iteration")
    ap.add_argument("--admm-iters", type=int, default=ADMM, help="with --admm-only: ADMM iterations per launch")
    ap.add_argument("--il-only", default="", metavar="POINT",
                    help="profiling aid: interleaved factor + solve of one 'nx,nu,N,batch,dtype' point, then exit")
    ap.add_argument("--config", default="", choices=["", "obstacles", "cw_mlp"],
                    help="time config 4 (obstacles) or config 5 (cw_mlp) on one GPU instead of the default run")
    ap.add_argument("--pcg-sweep", default="", metavar="POINTS",
                    help="config-2 linear-system sweep: ';'-separated nx,nu,N,batch,dtype points "
                         "(e.g. '24,8,128,4096,f32'); 'default' runs a representative set")
    args = ap.parse_args()
    if args.config:
        return run_config(args.config, backend=args.backend)
    if args.pcg_sweep:
        spec = args.pcg_sweep
        if spec == "default":
            spec = ("6,3,32,65536,f32;12,4,64,16384,f32;24,8,128,4096,f32;"
                    "6,3,32,65536,f64;12,4,64,16384,f64;24,8,128,2048,f64")
        pts = []
        for item in spec.split(";"):
            a = item.split(",")
            pts.append((int(a[0]), int(a[1]), int(a[2]), int(a[3]), a[4]))
        return pcg_sweep(pts)
    if args.il_only:
        return il_only(args.il_only)
    if args.admm_only:
        return admm_only(args.admm_only, args.admm_linsys, pcg=args.admm_pcg, admm=args.admm_iters)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch

    from turbompc_b200 import _ffi, ops
    from turbompc_b200.dynamics import Quadrotor12Dynamics
    from turbompc_b200.problems.ocp import OptimalControlProblem
    from turbompc_b200.problems.quadrotor import quadrotor_params
    from turbompc_b200.sharding import gather_batch, shard_params, shard_range
    from turbompc_b200.solver import TurboMPCSolver

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=dev)
    _ffi.load(build_if_missing=False)
    lo, hi = shard_range(args.batch, world, rank)
    shard = hi - lo
    full = quadrotor_params(args.batch, N=N_HORIZON, seed=1000, dtype=torch.float32, device="cpu")
    params = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v)
              for k, v in shard_params(full, args.batch, lo, hi).items()}
    ocp = OptimalControlProblem(Quadrotor12Dynamics(), params)
    sp = {"num_sqp_iteration_max": SQP, "tol_convergence": 0.0,
          "admm": {"max_iter": ADMM, "check_termination_every": 0, "adapt_rho_every": 0, "eps_abs": 0.0,
                   "eps_rel": 0.0, "pcg": {"max_iter": PCG, "tol_epsilon": 0.0}}}
    direct = args.backend == "direct"
    solver = TurboMPCSolver(ocp, sp, forward_backend="b200_direct" if direct else "b200")
    guess = solver.initial_guess(params)
    lib = _ffi.load(build_if_missing=False)

    # ---- device-resident timing (value) with per-launch events for the ADMM kernel
    launch_ms = []
    n_lin = [0]
    orig = ops.admm_solve
    orig_lin = ops.linearize_dynamics
    orig_kkt = ops.first_order_error
    orig_ineq = ops.ineq_rows

    def timed_admm(*a, **k):
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record()
        out = orig(*a, **k)
        e1.record()
        launch_ms.append((e0, e1))
        return out

    def counted_lin(*a, **k):
        n_lin[0] += 1
        return orig_lin(*a, **k)

    def counted_kkt(*a, **k):
        n_lin[0] += 1
        return orig_kkt(*a, **k)

    def counted_ineq(*a, **k):
        n_lin[0] += 1
        return orig_ineq(*a, **k)

    def step():
        return solver.solve(guess, params)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.admm_solve = timed_admm
    ops.linearize_dynamics = counted_lin
    ops.first_order_error = counted_kkt
    ops.ineq_rows = counted_ineq
    import turbompc_b200.solver as solver_mod

    solver_mod.ops.admm_solve = timed_admm
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    if direct:
        lib.tmpc_admm_iteration_timing(1)  # events around the iteration kernel of each ADMM call
    with ClockSampler(local) as clk:
        s0, s1 = torch.cuda.Event(True), torch.cuda.Event(True)
        s0.record()
        for _ in range(args.steps):
            sol = step()
        s1.record()
        torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ops.admm_solve = orig
    ops.linearize_dynamics = orig_lin
    ops.first_order_error = orig_kkt
    ops.ineq_rows = orig_ineq
    solver_mod.ops.admm_solve = orig
    ms = s0.elapsed_time(s1) / args.steps
    kern_ms = [a.elapsed_time(b) for a, b in launch_ms]
    kms = sum(kern_ms) / len(kern_ms)  # one whole ADMM call (all its kernels)
    ims = kms
    if direct:
        import ctypes

        lib.tmpc_admm_iteration_timing(0)
        buf = (ctypes.c_float * 1024)()
        cnt = lib.tmpc_admm_iteration_timing_read(buf, 1024)
        ims = sum(buf[:cnt]) / max(cnt, 1)  # the iteration kernel alone
    if dist:
        t = torch.tensor([ms, kms, ims], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, kms, ims = t.tolist()
    value = args.batch / (ms / 1e3)

    # ---- end-to-end through the public API with host buffers
    x0_host = params["initial_state"].cpu().pin_memory()
    ref_host = params["reference_state_trajectory"].cpu().pin_memory()
    u0_host = torch.empty(args.batch if rank == 0 else 1, 4, dtype=torch.float32).pin_memory()
    e2e_steps = max(1, args.steps)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(True), torch.cuda.Event(True)
    a0.record()
    for _ in range(e2e_steps):
        p2 = dict(params)
        p2["initial_state"] = x0_host.to(dev, non_blocking=True)
        p2["reference_state_trajectory"] = ref_host.to(dev, non_blocking=True)
        g2 = solver.initial_guess(p2)
        s2 = solver.solve(g2, p2)
        u0 = s2.controls[:, 0].contiguous()
        if dist:
            u0 = gather_batch(u0, args.batch)  # the only collective: the final gather
        if rank == 0:
            u0_host.copy_(u0, non_blocking=True)
    a1.record()
    torch.cuda.synchronize()
    e2e_ms = a0.elapsed_time(a1) / e2e_steps
    if dist:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    h2d = (x0_host.numel() + ref_host.numel()) * 4 * world
    d2h = args.batch * 4 * 4

    if rank == 0:
        qp = solver._build_qp_data(guess.states, guess.controls, params)
        T, n, nx, m, n0 = qp.T, qp.n, qp.nx, qp.m, qp.n0
        hbm, pk_kind = peaks()
        if direct:
            ap = qp.eq.A_plus
            pat = torch.zeros(ap.shape[-2:], dtype=ap.dtype, device=ap.device)
            pat[:, :nx] = -torch.eye(nx, dtype=ap.dtype, device=ap.device)
            G = qp.ineq.G
            g0 = G[:1, :1]
            gsel = bool((G == g0).all()) and bool(((g0 == 1).sum(-1) == 1).all()) and bool(
                ((g0 == 0) | (g0 == 1)).all())
            # rows nx.. of Phi_t = E_t + rho_f A+_t^T A-_t vanish when A+'s control
            # columns and E's control rows are zero: W_t keeps nx rows
            wz = bool((ap[..., nx:] == 0).all()) and bool((qp.cost.E[..., nx:, :] == 0).all())
            roof = direct_roofline(T, n, nx, m, n0, shard, ims, kms, hbm, pk_kind, bool((ap == pat).all()), gsel,
                                   nx if wz else n)
            per_call = direct_launches_per_solve(n0, m)
        else:
            roof = pcg_roofline(T, n, nx, m, n0, shard, kms, hbm)
            per_call = 1
        # QP data one fused ADMM launch reads (one SQP iteration's D, E, q,
        # A_minus, A_plus, c, G, l, u for this GPU's shard, fp32).
        qp_gb = shard * 4 * (T * n * n * 2 + T * n + 2 * (T - 1) * nx * n + (T - 1) * nx
                                               + T * m * (n + 2)) / 1e9
        cb = None
        if world == 1 and not args.no_cpu_baseline:
            try:
                cb = cpu_baseline(backend=args.backend)
            except Exception as exc:  # reported, not fatal
                cb = {"error": repr(exc)}
        cfg = workload_config(args.batch, world, shard, args.backend)
        cfg["l2"] = (f"inputs > L2 (QP data ~{qp_gb:.1f} GB per SQP iteration)" if qp_gb > 0.126
                     else f"QP data {qp_gb:.3f} GB per SQP iteration (fits L2)")
        line = {
            "metric": METRIC, "value": value, "unit": "solves/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
            "e2e": {"value": args.batch / (e2e_ms / 1e3), "unit": "solves/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": roof,
            "gpu_launches": len(launch_ms) * per_call + n_lin[0],
            "clocks": clk.summary(),
            "cpu_baseline": cb,
        }
        if world == 1 and not args.headline_only:
            line["configs"] = other_configs()
            if direct:  # the same workload with 30 PCG iterations per ADMM iteration
                try:
                    line["configs"]["pcg_variant"] = pcg_variant(ocp, params, sp, args.batch)
                except Exception as exc:  # reported, not fatal
                    line["configs"]["pcg_variant"] = {"error": repr(exc)}
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
