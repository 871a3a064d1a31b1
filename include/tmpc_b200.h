/*
 * tmpc_b200.h - C ABI of the B200-native batched SQP+ADMM inner solve.
 *
 * Every entry point is `extern "C"`, takes plain device pointers, sizes and a
 * CUDA stream (passed as `void*`, i.e. a `cudaStream_t`), enqueues its work on
 * that stream and returns an int status:
 *      0              success
 *     <0              argument error (nothing was launched)
 *     >0              CUDA error code from the launch
 * No exception crosses the ABI, nothing is allocated behind the caller's back
 * (scratch space is a caller-owned workspace whose size a *_workspace_bytes
 * query reports), and no entry point keeps global state, so calls on
 * different streams are independent.
 *
 * Batched arrays are problem-major and contiguous, exactly the layout the
 * reference's XLA FFI handlers receive after `vmap_method="broadcast_all"`
 * (turbompc/solvers/admm/admm_ffi_backend.py:358-362):
 *     D       [Nb, T, n, n]      E        [Nb, N, n, n]     q  [Nb, T, n]
 *     A0      [Nb, n0, n]        A_minus  [Nb, N, nx, n]    A_plus [Nb, N, nx, n]
 *     c0      [Nb, n0]           c        [Nb, N, nx]
 *     G       [Nb, T, m, n]      l, u     [Nb, T, m]
 *     S, Phiinv (reference layout) [Nb, T, n, 3n]
 * with T = N + 1 and n = nx + nu.
 */
#ifndef TMPC_B200_H_
#define TMPC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TMPC_OK 0
#define TMPC_ERR_NULL_ARG (-1)
#define TMPC_ERR_BAD_DIMS (-2)
#define TMPC_ERR_UNSUPPORTED (-3)
#define TMPC_ERR_WORKSPACE (-4) /* workspace / factor buffer missing, too small or not 16-byte aligned */
#define TMPC_ERR_SMEM (-5)
#define TMPC_ERR_SCRATCH_LIMIT (-6) /* needs more scratch than the fixed device buffer holds */

/* Per-problem status bits written by solves (status_out[b]). */
#define TMPC_STATUS_SINGULAR_BLOCK 1 /* a Theta_t / Cholesky / LU pivot was zero or not finite */
#define TMPC_STATUS_NONFINITE 2      /* a non-finite value reached the output */

typedef void* tmpc_stream_t; /* a cudaStream_t */

typedef struct TmpcDims {
  int32_t Nb; /* batch size (independent problems) */
  int32_t T;  /* stages, N + 1 */
  int32_t n;  /* nx + nu */
  int32_t nx; /* states */
  int32_t n0; /* rows of A0 (nx, or nx + nu with a fixed initial control) */
  int32_t m;  /* inequality rows per stage (may be 0) */
} TmpcDims;

/* Stage-blocked QP (turbompc/solvers/qp_data.py:13-97). Device pointers of the
 * function's precision.  G, l, u may be NULL when m == 0. */
typedef struct TmpcQP {
  const void* D;
  const void* E;
  const void* q;
  const void* A0;
  const void* A_minus;
  const void* A_plus;
  const void* c0;
  const void* c;
  const void* G;
  const void* l;
  const void* u;
} TmpcQP;

/* ADMMState (turbompc/solvers/admm/admm.py:27-34), batched. */
typedef struct TmpcAdmmState {
  void* x;       /* [Nb, T, n] */
  void* y_g;     /* [Nb, T, m] */
  void* y_f0;    /* [Nb, n0]   */
  void* y_fdyn;  /* [Nb, N, nx] */
  void* z_g;     /* [Nb, T, m] */
  void* xi_g;    /* [Nb, T, m] */
  void* rho_bar; /* [Nb]       */
} TmpcAdmmState;

#define TMPC_LINSYS_PCG 0    /* preconditioned CG on the Schur system (admm_fused_pcg) */
#define TMPC_LINSYS_DIRECT 1 /* block-tridiagonal Cholesky (replaces admm_fused_cudss) */
/* PCG as TMPC_LINSYS_PCG, but always on the shared-memory packed-operator kernel
 * (TMPC_LINSYS_PCG picks the register-resident kernel for fp32, 8 < n <= 16, T <= 64). */
#define TMPC_LINSYS_PCG_PACKED 2

/* Mirrors ADMMConfig (turbompc/solvers/admm/csrc/admm_fused.cuh:6-22). */
typedef struct TmpcAdmmConfig {
  int32_t max_iter;
  int32_t pcg_max_iter;
  int32_t check_every;     /* <= 0 disables residual checks */
  int32_t adapt_rho_every; /* <= 0 disables rho adaptation */
  double eps_abs;
  double eps_rel;
  double sigma;
  double rho_f_factor;
  double alpha;
  double pcg_eps;
  double adaptive_rho_tolerance;
  double rho_min;
  double rho_max;
  int32_t use_slack;
  int32_t linsys; /* TMPC_LINSYS_* */
} TmpcAdmmConfig;

/* Library version (major*10000 + minor*100 + patch) and error strings. */
int32_t tmpc_version(void);
const char* tmpc_error_string(int32_t code);

/* Diagnostics hook, no counterpart in the reference.  Kernels that stage
 * their operators into shared memory with TMA bulk copies wait for them with
 * a bounded poll loop; if it runs out, the problem's iters_out is set to
 * 0xffffffff (a transfer time-out), the copies still in flight are drained,
 * and the CTA returns without hanging the GPU.  This sets that loop's poll
 * limit for subsequent launches (default 2^26) and returns the previous one;
 * a limit of 0 makes every such wait report a time-out, which lets a test
 * exercise the status path on copies that do complete. */
uint32_t tmpc_set_transfer_poll_limit(uint32_t polls);

/* Diagnostics hook, no counterpart in the reference.  While enabled, every
 * tmpc_admm_solve_* call that runs the batch-interleaved direct solve
 * (linsys = TMPC_LINSYS_DIRECT with n <= 16 in fp32, n <= 12 in fp64) records
 * a CUDA event pair on its stream around its ADMM iteration kernels (after
 * the layout conversion, assembly and factor; before the conversion back), at
 * most 1024 pairs.  _timing(enable) returns the previous setting; _read waits
 * for the recorded pairs, writes up to max_out elapsed times in ms (call
 * order), releases every pair and returns the number written. */
int32_t tmpc_admm_iteration_timing(int32_t enable);
int32_t tmpc_admm_iteration_timing_read(float* ms_out, int32_t max_out);

/* ---------------------------------------------------------------------------
 * Schur complement + preconditioner assembly.
 * Replaces compute_S_Phiinv (turbompc/solvers/admm/admm.py:71-154): writes the
 * reference-layout S and Phiinv [Nb, T, n, 3n] for rho_f = rho_bar[b] *
 * rho_f_factor and rho_ineq = rho_bar[b].
 * ------------------------------------------------------------------------- */
int32_t tmpc_schur_assemble_f32(const TmpcDims* dims, const TmpcQP* qp, const float* rho_bar,
                                double sigma, double rho_f_factor, float* S, float* Phiinv,
                                int32_t* status_out, tmpc_stream_t stream);
int32_t tmpc_schur_assemble_f64(const TmpcDims* dims, const TmpcQP* qp, const double* rho_bar,
                                double sigma, double rho_f_factor, double* S, double* Phiinv,
                                int32_t* status_out, tmpc_stream_t stream);

/* Packed operator format: per problem the unique blocks of S and Phiinv
 * (upper triangle of each diagonal block, the full sub-diagonal blocks),
 * zero-padded to the kernel block size.  Bytes for the whole batch: */
size_t tmpc_packed_operator_bytes(const TmpcDims* dims, int32_t dtype_bytes);
int32_t tmpc_schur_assemble_packed_f32(const TmpcDims* dims, const TmpcQP* qp, const float* rho_bar,
                                       double sigma, double rho_f_factor, void* ops,
                                       int32_t* status_out, tmpc_stream_t stream);
int32_t tmpc_schur_assemble_packed_f64(const TmpcDims* dims, const TmpcQP* qp, const double* rho_bar,
                                       double sigma, double rho_f_factor, void* ops,
                                       int32_t* status_out, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Batched block-tridiagonal PCG.
 * Replaces the `pcg_blktridi_cuda[_f64]` FFI target
 * (turbompc/solvers/linear_systems_solvers/csrc/pcg_ffi.cc:115-147;
 * LaunchPcgBlkTridiF32/F64 pcg_blktridi.cuh:7-32): solves S x = rhs from x0
 * with the preconditioner Phiinv, stopping when |eta| < 1e-12 + eps*|eta_0|
 * or after max_iters iterations; iters_out[b] is the iteration count.
 * Any T*n is accepted (no size cliff, no host synchronisation).
 * ------------------------------------------------------------------------- */
int32_t tmpc_pcg_solve_f32(const TmpcDims* dims, const float* S, const float* Phiinv,
                           const float* rhs, const float* x0, float* x_out, uint32_t* iters_out,
                           double eps, int32_t max_iters, tmpc_stream_t stream);
int32_t tmpc_pcg_solve_f64(const TmpcDims* dims, const double* S, const double* Phiinv,
                           const double* rhs, const double* x0, double* x_out, uint32_t* iters_out,
                           double eps, int32_t max_iters, tmpc_stream_t stream);
/* Same solve on operators in the packed format written by
 * tmpc_schur_assemble_packed_*. */
int32_t tmpc_pcg_solve_packed_f32(const TmpcDims* dims, const void* ops, const float* rhs,
                                  const float* x0, float* x_out, uint32_t* iters_out, double eps,
                                  int32_t max_iters, tmpc_stream_t stream);
int32_t tmpc_pcg_solve_packed_f64(const TmpcDims* dims, const void* ops, const double* rhs,
                                  const double* x0, double* x_out, uint32_t* iters_out, double eps,
                                  int32_t max_iters, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused ADMM solve (Schur assembly + ADMM iteration + linear solve in one
 * kernel, one CTA per problem).
 * Replaces the `admm_fused_cuda[_f64]` FFI target
 * (turbompc/solvers/admm/csrc/admm_ffi.cc:150-274; LaunchADMMFusedF32/F64,
 * admm_fused.cuh:25-124) and, with cfg->linsys == TMPC_LINSYS_DIRECT, the
 * cuDSS loop `admm_cudss_cuda[_f64]` (admm/csrc/admm_cudss_ffi.cc:142-256).
 * S / Phiinv are built on the device from the QP (no host-side
 * compute_S_Phiinv), so the reference's S, Phiinv, S_work and Phiinv_work
 * buffers have no counterpart.  state_out may alias state_in.
 * slack_weight [Nb] may be NULL (all zero).  x_out [Nb, T, n] may be NULL.
 * The workspace is needed only when the per-problem operators do not fit in
 * shared memory; query its size with tmpc_admm_workspace_bytes.
 * ------------------------------------------------------------------------- */
size_t tmpc_admm_workspace_bytes(const TmpcDims* dims, int32_t dtype_bytes, const TmpcAdmmConfig* cfg);
int32_t tmpc_admm_solve_f32(const TmpcDims* dims, const TmpcQP* qp, const TmpcAdmmState* state_in,
                            const TmpcAdmmState* state_out, const float* slack_weight,
                            const TmpcAdmmConfig* cfg, float* x_out, uint32_t* iters_out,
                            int32_t* status_out, void* workspace, size_t workspace_bytes,
                            tmpc_stream_t stream);
int32_t tmpc_admm_solve_f64(const TmpcDims* dims, const TmpcQP* qp, const TmpcAdmmState* state_in,
                            const TmpcAdmmState* state_out, const double* slack_weight,
                            const TmpcAdmmConfig* cfg, double* x_out, uint32_t* iters_out,
                            int32_t* status_out, void* workspace, size_t workspace_bytes,
                            tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Batched block-tridiagonal Cholesky (block Riccati recursion) of the
 * reference-layout S, written from scratch; replaces the cuDSS direct solve
 * `cudss_blktridi_cuda[_f64]` (linear_systems_solvers/csrc/cudss_ffi.cc:76-98,
 * cudss_blktridi.cu:60-184).  The factor occupies
 * tmpc_riccati_factor_bytes(dims, dtype_bytes) bytes (caller-owned);
 * status_out[b] = TMPC_STATUS_SINGULAR_BLOCK when S is not positive definite.
 * dims->nx, n0 and m are not used.
 * ------------------------------------------------------------------------- */
size_t tmpc_riccati_factor_bytes(const TmpcDims* dims, int32_t dtype_bytes);
int32_t tmpc_riccati_factor_f32(const TmpcDims* dims, const float* S, void* factor,
                                int32_t* status_out, tmpc_stream_t stream);
int32_t tmpc_riccati_factor_f64(const TmpcDims* dims, const double* S, void* factor,
                                int32_t* status_out, tmpc_stream_t stream);
int32_t tmpc_riccati_solve_f32(const TmpcDims* dims, const void* factor, const float* rhs,
                               float* x_out, tmpc_stream_t stream);
int32_t tmpc_riccati_solve_f64(const TmpcDims* dims, const void* factor, const double* rhs,
                               double* x_out, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Adjoint KKT solve of the backward pass.  Replaces the dense solve
 * solve_backward_kkt (turbompc/solvers/backward/backward_kkt_jax.py:177-211)
 * and the `cudss_sparse_kkt_f32/f64` target
 * (backward/backward_kkt_cudss_ffi.py:210-224): solves
 *     [P  C^T] [dz]   [-q]
 *     [C  R  ] [mu] = [ 0]
 * with C = [A0; A_minus/A_plus rows; G rows], R = -1e-12 on all-zero G rows.
 * The QP's G holds the active rows (sign * G, zero rows inactive); c0, c, l,
 * u are not read.  dz_out [Nb, T, n]; mult_out [Nb, n0 + N*nx + T*m] in the
 * reference order (A0 rows, dynamics rows, inequality rows).  The caller
 * provides tmpc_adjoint_kkt_workspace_bytes() bytes of workspace.
 * ------------------------------------------------------------------------- */
size_t tmpc_adjoint_kkt_workspace_bytes(const TmpcDims* dims, int32_t dtype_bytes);
int32_t tmpc_adjoint_kkt_solve_f32(const TmpcDims* dims, const TmpcQP* qp, float* dz_out,
                                   float* mult_out, int32_t* status_out, void* workspace,
                                   size_t workspace_bytes, tmpc_stream_t stream);
int32_t tmpc_adjoint_kkt_solve_f64(const TmpcDims* dims, const TmpcQP* qp, double* dz_out,
                                   double* mult_out, int32_t* status_out, void* workspace,
                                   size_t workspace_bytes, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Fused ADMM solve that allocates nothing.  No counterpart in the reference:
 * an addition for callers that cannot allocate device memory (a runtime that
 * owns all allocations, a handler that may only touch the buffers it is
 * handed, an embedded controller with a fixed memory plan).  Same arguments
 * and results as tmpc_admm_solve_f64 without the workspace: when the
 * operators do not fit in shared memory they go to a statically allocated
 * device buffer of 64 MiB that every GPU
 * loading the library holds until process exit.  Batches needing more
 * return TMPC_ERR_SCRATCH_LIMIT without launching.  The first call on a
 * device looks up the buffer's device address (make it before any stream
 * capture); the address is kept for the life of the device's primary
 * context, so no call may follow a cudaDeviceReset of that device.  All calls share the buffer: calls that can overlap on the GPU
 * (different streams, or different host threads, on one device) race and
 * must be serialised by the caller.
 * ------------------------------------------------------------------------- */
int32_t tmpc_admm_solve_fixed_scratch_f64(const TmpcDims* dims, const TmpcQP* qp,
                                          const TmpcAdmmState* state_in, const TmpcAdmmState* state_out,
                                          const double* slack_weight, const TmpcAdmmConfig* cfg,
                                          double* x_out, uint32_t* iters_out, int32_t* status_out,
                                          tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * HBM-streaming PCG for operators too large to stay on chip (long horizons,
 * large n).  Same math, arguments and results as tmpc_pcg_solve_* (the
 * pcg_blktridi_cuda target, pcg_ffi.cc:115-147), on operators in the stream
 * layout written by tmpc_schur_assemble_stream_*: per problem S then Phiinv,
 * each T full NB x NB diagonal blocks followed by N full NB x NB sub-diagonal
 * blocks, row-major (NB = the compiled block size >= n, zero padded).  Every
 * PCG iteration reads each operator once from HBM.
 * ------------------------------------------------------------------------- */
size_t tmpc_stream_operator_bytes(const TmpcDims* dims, int32_t dtype_bytes);
int32_t tmpc_schur_assemble_stream_f32(const TmpcDims* dims, const TmpcQP* qp, const float* rho_bar, double sigma,
                                       double rho_f_factor, float* ops, int32_t* status, tmpc_stream_t stream);
int32_t tmpc_schur_assemble_stream_f64(const TmpcDims* dims, const TmpcQP* qp, const double* rho_bar, double sigma,
                                       double rho_f_factor, double* ops, int32_t* status, tmpc_stream_t stream);
int32_t tmpc_pcg_solve_stream_f32(const TmpcDims* dims, const float* ops, const float* rhs, const float* x0,
                                  float* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                                  tmpc_stream_t stream);
int32_t tmpc_pcg_solve_stream_f64(const TmpcDims* dims, const double* ops, const double* rhs, const double* x0,
                                  double* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                                  tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * First-order (KKT) error of SQP iterates z [Nb][T][n] with multipliers
 * y_f0 [Nb][n0], y_fdyn [Nb][N][nx], y_g [Nb][T][m] against the QP linearised
 * there: the "first_order" convergence measure of the SQP loop
 * (turbompc/solvers/turbompc_solver.py:1158-1225).  Per problem:
 *   conv = max(stat, eq, ineq [, ||w_s slack + y_g||_inf when use_slack]),
 *   stat = ||P z + q + C^T y_f + G^T y_g||_inf, eq = ||C z - c||_inf,
 *   ineq = ||max(l - g, 0, g - u)||_inf with g = G z (+ slack) written to g_out.
 * slack [Nb][T][m] and slack_weight [Nb] only with use_slack.
 * ------------------------------------------------------------------------- */
int32_t tmpc_first_order_error_f32(const TmpcDims* dims, const TmpcQP* qp, const float* z, const float* y_f0,
                                   const float* y_fdyn, const float* y_g, const float* slack,
                                   const float* slack_weight, int32_t use_slack, float* conv_out, float* eq_out,
                                   float* ineq_out, float* g_out, tmpc_stream_t stream);
int32_t tmpc_first_order_error_f64(const TmpcDims* dims, const TmpcQP* qp, const double* z, const double* y_f0,
                                   const double* y_fdyn, const double* y_g, const double* slack,
                                   const double* slack_weight, int32_t use_slack, double* conv_out, double* eq_out,
                                   double* ineq_out, double* g_out, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Linearised discrete dynamics of a built-in model, batched over (problem,
 * stage t < N): the QP's dynamics rows, as produced in the reference by
 * get_dynamics_linearized_matrices (turbompc/problems/
 * optimal_control_problem.py:1217-1272, explicit schemes, forward-mode
 * Jacobian).  With F one step of `scheme` (turbompc/dynamics/integrators.py)
 * of the model's x_dot:
 *   A_minus[b][t] = [dF/dx, dF/du] at (x_t, u_t)        [Nb][N][nx][n]
 *   c[b][t]       = -F(x_t, u_t) + A_minus[b][t] [x_t; u_t]   [Nb][N][nx]
 * states [Nb][T][nx], controls [Nb][T][nu]; dims: Nb, T, n = nx + nu, nx
 * (n0, m unused).  params (host array):
 *   TMPC_MODEL_QUADROTOR12         {mass, Jx, Jy, Jz, arm_length, yaw_coefficient}
 *   TMPC_MODEL_CLOHESSY_WILTSHIRE  {mean_motion}
 * ------------------------------------------------------------------------- */
#define TMPC_MODEL_QUADROTOR12 1
#define TMPC_MODEL_CLOHESSY_WILTSHIRE 2
#define TMPC_SCHEME_EULER 0
#define TMPC_SCHEME_MIDPOINT 1
#define TMPC_SCHEME_RK4 2
int32_t tmpc_linearize_dynamics_f32(const TmpcDims* dims, int32_t model, int32_t scheme, double dt,
                                    const float* states, const float* controls, const double* params,
                                    int32_t n_params, float* A_minus, float* c, tmpc_stream_t stream);
int32_t tmpc_linearize_dynamics_f64(const TmpcDims* dims, int32_t model, int32_t scheme, double dt,
                                    const double* states, const double* controls, const double* params,
                                    int32_t n_params, double* A_minus, double* c, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * QP producers of the benchmark problems beyond the dynamics rows, batched
 * over (problem, stage); dims: Nb, T, n = nx + nu, nx (n0, m unused).
 *
 * Spherical obstacle rows (turbompc/problems/obstacle_avoidance.py:16-52,
 * linearised as get_inequalities_linearized_matrices does,
 * optimal_control_problem.py:580-626): for p = states[b][t][:dim],
 *   g_k = 1 - ||p - c_k|| / (r_k + 0.001), G_k = dg_k / dz,
 *   l_k = -1e9 - (g_k - G_k z), u_k = -(g_k - G_k z),  all times row_scale.
 * states [Nb][T][nx], centers [Nb][K][dim], radii [Nb][K];
 * outputs G [Nb][T][K][n], l, u [Nb][T][K].
 * ------------------------------------------------------------------------- */
int32_t tmpc_obstacle_rows_f32(const TmpcDims* dims, int32_t dim, int32_t n_obstacles, const float* states,
                               const float* centers, const float* radii, double row_scale, float* G, float* l,
                               float* u, tmpc_stream_t stream);
int32_t tmpc_obstacle_rows_f64(const TmpcDims* dims, int32_t dim, int32_t n_obstacles, const double* states,
                               const double* centers, const double* radii, double row_scale, double* G, double* l,
                               double* u, tmpc_stream_t stream);
/* Inequality rows at an iterate: g[b][t][k] = G_t[k] . z_t (+ slack[b][t][k]
 * when slack is non-null), clamped to [l, u] when l and u are given (both or
 * neither).  G [Nb][T][m][n], z [Nb][T][n], slack / l / u / g_out [Nb][T][m];
 * dims->nx and dims->n0 are not used.
 * Replaces the G z products of ADMM's initial state (z_g = clamp(G x, l, u),
 * turbompc/solvers/admm/admm.py:1051-1088) and of the SQP loop's active-set
 * identification (turbompc/solvers/turbompc_solver.py:1387-1439). */
int32_t tmpc_ineq_rows_f32(const TmpcDims* dims, const float* G, const float* z, const float* slack, const float* l,
                           const float* u, float* g_out, tmpc_stream_t stream);
int32_t tmpc_ineq_rows_f64(const TmpcDims* dims, const double* G, const double* z, const double* slack,
                           const double* l, const double* u, double* g_out, tmpc_stream_t stream);
/* A learned stage cost s * w2 . tanh(W1 z + b1) (z = [x, u], every stage)
 * quadratised exactly and added in place to the cost blocks (the
 * stage-separable case of get_cost_linearized_blocks,
 * optimal_control_problem.py:1068-1174):  D_t += H, q_t += grad - H z with
 * grad = s W1^T (w2 * (1 - th^2)), H = s W1^T diag(w2 * (-2 th (1 - th^2))) W1,
 * th = tanh(W1 z + b1).  W1 [hidden][n], b1, w2 [hidden] (shared by the
 * batch); D [Nb][T][n][n], q [Nb][T][n]; n <= 16.  No counterpart kernel in
 * the reference (its learned costs go through jax.grad / jax.hessian). */
int32_t tmpc_mlp_cost_blocks_f32(const TmpcDims* dims, int32_t hidden, const float* states, const float* controls,
                                 const float* W1, const float* b1, const float* w2, double scale, float* D, float* q,
                                 tmpc_stream_t stream);
int32_t tmpc_mlp_cost_blocks_f64(const TmpcDims* dims, int32_t hidden, const double* states,
                                 const double* controls, const double* W1, const double* b1, const double* w2,
                                 double scale, double* D, double* q, tmpc_stream_t stream);

/* ---------------------------------------------------------------------------
 * Batch-interleaved layout and the direct solve on it.
 *
 * TMPC_LAYOUT_REFERENCE is the problem-major layout every entry point above
 * takes (what the reference's FFI handlers receive).  TMPC_LAYOUT_INTERLEAVED
 * groups problems by 32 and stores each group element-major, problem-minor:
 *     element e of problem b  at  ((b / 32) * E + e) * 32 + b % 32
 * (E = elements per problem), so the 32 lanes of a warp, one problem each,
 * read and write every element with one coalesced transaction.  Interleaved
 * arrays hold tmpc_interleaved_elems(Nb, E) elements (ceil(Nb / 32) * 32
 * problem slots; the slots past Nb are padding the kernels may write).
 *
 * Interleaved operator / factor format, E = tmpc_riccati_il_elems_per_problem:
 *   T blocks Theta_t (factor: L_t), lower triangle packed row-major
 *     ((i, j <= i) at t n(n+1)/2 + i(i+1)/2 + j), then
 *   N blocks Phi_t = S(t+1, t) (factor: W_t = Phi_t L_t^-T), row-major n x n.
 * Vectors (rhs, x) are [T][n] per problem, interleaved.
 * The factor and solve replace the cuDSS direct solve `cudss_blktridi_cuda`
 * (linear_systems_solvers/csrc/cudss_ffi.cc:76-98) like tmpc_riccati_*, one
 * problem per thread; n <= 16 in fp32, n <= 12 in fp64 (TMPC_ERR_UNSUPPORTED
 * beyond: use tmpc_riccati_* on the reference layout).
 * ------------------------------------------------------------------------- */
#define TMPC_LAYOUT_REFERENCE 0
#define TMPC_LAYOUT_INTERLEAVED 1
size_t tmpc_interleaved_elems(int32_t Nb, int64_t elems_per_problem);
int64_t tmpc_riccati_il_elems_per_problem(const TmpcDims* dims);
/* [Nb][elems] problem-major <-> interleaved (any per-problem array). */
int32_t tmpc_interleave_f32(int32_t Nb, int64_t elems, const float* src, float* dst, tmpc_stream_t stream);
int32_t tmpc_interleave_f64(int32_t Nb, int64_t elems, const double* src, double* dst, tmpc_stream_t stream);
int32_t tmpc_deinterleave_f32(int32_t Nb, int64_t elems, const float* src, float* dst, tmpc_stream_t stream);
int32_t tmpc_deinterleave_f64(int32_t Nb, int64_t elems, const double* src, double* dst, tmpc_stream_t stream);
/* Reference-layout S [Nb, T, n, 3n] -> interleaved operator (Theta, Phi). */
int32_t tmpc_schur_interleave_f32(const TmpcDims* dims, const float* S, float* ops, tmpc_stream_t stream);
int32_t tmpc_schur_interleave_f64(const TmpcDims* dims, const double* S, double* ops, tmpc_stream_t stream);
/* status_out [Nb] (problem-major) as tmpc_riccati_factor_*. */
int32_t tmpc_riccati_factor_il_f32(const TmpcDims* dims, const float* ops, float* factor, int32_t* status_out,
                                   tmpc_stream_t stream);
int32_t tmpc_riccati_factor_il_f64(const TmpcDims* dims, const double* ops, double* factor, int32_t* status_out,
                                   tmpc_stream_t stream);
int32_t tmpc_riccati_solve_il_f32(const TmpcDims* dims, const float* factor, const float* rhs, float* x_out,
                                  tmpc_stream_t stream);
int32_t tmpc_riccati_solve_il_f64(const TmpcDims* dims, const double* factor, const double* rhs, double* x_out,
                                  tmpc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TMPC_B200_H_ */
