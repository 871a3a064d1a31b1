// C-ABI shim over the reference's own CUDA launchers, compiled together with
// the unmodified reference sources by oracle/build_ref.sh into
// oracle/_ref/libtmpc_refcuda.so.  TEST INFRASTRUCTURE ONLY: used to produce
// the golden vectors in tests/golden/ and as a second GPU-side oracle.
//   LaunchADMMFusedF32/F64   turbompc/solvers/admm/csrc/admm_fused.cuh:25,74
//   LaunchPcgBlkTridiF32/F64 turbompc/solvers/linear_systems_solvers/csrc/pcg_blktridi.cuh:7,21
#include <cuda_runtime.h>
#include <stdint.h>

#include "admm_fused.cuh"
#include "pcg_blktridi.cuh"

extern "C" {

struct RefAdmmArgs {
  void *x_out, *iters_out, *x_blocks_out, *z_g_out, *y_g_out, *y_f_0_out, *y_f_dyn_out, *xi_g_out, *rho_bar_out,
      *kernel_ns_out, *S_work, *Phiinv_work;
  const void *S, *Phiinv, *D, *E, *q, *A0, *A_minus, *A_plus, *G, *l, *u, *c0, *c, *x0, *z_g0, *y_g0, *y_f_0,
      *y_f_dyn, *xi_g0, *rho_bar, *slack_weight;
  int32_t T, n, nx, n0, m, Nb;
  int32_t max_iter, pcg_max_iter, check_every, adapt_rho_every, use_slack;
  double eps_abs, eps_rel, sigma, rho_f_factor, alpha, pcg_eps, adaptive_rho_tolerance, rho_min, rho_max;
};

static ADMMConfig cfg_of(const RefAdmmArgs* a) {
  ADMMConfig c;
  c.max_iter = a->max_iter;
  c.pcg_max_iter = a->pcg_max_iter;
  c.check_every = a->check_every;
  c.eps_abs = a->eps_abs;
  c.eps_rel = a->eps_rel;
  c.sigma = a->sigma;
  c.rho_f_factor = a->rho_f_factor;
  c.alpha = a->alpha;
  c.pcg_eps = a->pcg_eps;
  c.adapt_rho = a->adapt_rho_every > 0;
  c.use_slack = a->use_slack != 0;
  c.adapt_rho_every = a->adapt_rho_every;
  c.adaptive_rho_tolerance = a->adaptive_rho_tolerance;
  c.rho_min = a->rho_min;
  c.rho_max = a->rho_max;
  return c;
}

#define REF_ADMM(NAME, LAUNCH, R)                                                                               \
  int NAME(const RefAdmmArgs* a, void* stream) {                                                                \
    cudaError_t e = LAUNCH(                                                                                     \
        (cudaStream_t)stream, (R*)a->x_out, (uint32_t*)a->iters_out, (R*)a->x_blocks_out, (R*)a->z_g_out,      \
        (R*)a->y_g_out, (R*)a->y_f_0_out, (R*)a->y_f_dyn_out, (R*)a->xi_g_out, (R*)a->rho_bar_out,             \
        (R*)a->kernel_ns_out, (R*)a->S_work, (R*)a->Phiinv_work, (const R*)a->S, (const R*)a->Phiinv,         \
        (const R*)a->D, (const R*)a->E, (const R*)a->q, (const R*)a->A0, (const R*)a->A_minus,                \
        (const R*)a->A_plus, (const R*)a->G, (const R*)a->l, (const R*)a->u, (const R*)a->c0, (const R*)a->c,  \
        (const R*)a->x0, (const R*)a->z_g0, (const R*)a->y_g0, (const R*)a->y_f_0, (const R*)a->y_f_dyn,      \
        (const R*)a->xi_g0, (const R*)a->rho_bar, (const R*)a->slack_weight, a->T, a->n, a->nx, a->n0, a->m,  \
        a->Nb, cfg_of(a));                                                                                      \
    return (int)e;                                                                                              \
  }
REF_ADMM(ref_admm_fused_f32, LaunchADMMFusedF32, float)
REF_ADMM(ref_admm_fused_f64, LaunchADMMFusedF64, double)

int ref_pcg_f32(void* stream, float* x_out, uint32_t* iters, const float* S, const float* P, const float* rhs,
                const float* x0, double eps, int max_iters, int T, int n, int Nb) {
  LaunchPcgBlkTridiF32((cudaStream_t)stream, x_out, iters, S, P, rhs, x0, (float)eps, max_iters, T, n, Nb);
  return (int)cudaPeekAtLastError();
}
int ref_pcg_f64(void* stream, double* x_out, uint32_t* iters, const double* S, const double* P, const double* rhs,
                const double* x0, double eps, int max_iters, int T, int n, int Nb) {
  LaunchPcgBlkTridiF64((cudaStream_t)stream, x_out, iters, S, P, rhs, x0, eps, max_iters, T, n, Nb);
  return (int)cudaPeekAtLastError();
}

}  // extern "C"
