// Fused ADMM: size queries, argument checks and dispatch to the per-block-size
// kernels (instantiated in inst_nb*.cu).
#include "launchers.cuh"

namespace tmpc {

template <typename R>
size_t admm_ws_bytes(const TmpcDims& d) {
  if (d.n > 32) return admm_generic_ws_bytes<R>(d);
  size_t out = 0;
  dispatch_nb(d.n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    const size_t s_res = admm_smem_bytes<NB, R>(d.T, d.nx, d.n0, d.m, true);
    out = ((long)s_res <= max_dyn_smem()) ? 0 : (size_t)d.Nb * 2 * Geo<NB, R>::op_elems(d.T) * sizeof(R);
    return 0;
  });
  return out;
}

// Workspace for cfg: the direct solve always keeps its factor in HBM.
template <typename R>
size_t admm_ws_bytes_cfg(const TmpcDims& d, const TmpcAdmmConfig* cfg) {
  if (!cfg || cfg->linsys != TMPC_LINSYS_DIRECT) return admm_ws_bytes<R>(d);
  if (d.n > 32) return 0;  // the direct solve is compiled for n <= 32
  const size_t il = admm_il_ws_bytes<R>(d);  // the batch-interleaved path where it applies
  if (il > 0) return il;
  size_t out = 0;
  dispatch_nb(d.n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    out = (size_t)d.Nb * Geo<NB, R>::op_elems(d.T) * sizeof(R);
    return 0;
  });
  return out;
}

template <typename R>
int admm_solve(const TmpcDims* d, const TmpcQP* qp, const TmpcAdmmState* in, const TmpcAdmmState* out,
               const R* slack_weight, const TmpcAdmmConfig* cfg, R* x_out, uint32_t* iters_out, int32_t* status_out,
               void* ws, size_t ws_bytes, cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!qp || !in || !out || !cfg) return TMPC_ERR_NULL_ARG;
  if (!qp->D || !qp->E || !qp->q || !qp->A_minus || !qp->A_plus || !qp->c) return TMPC_ERR_NULL_ARG;
  if (d->n0 > 0 && (!qp->A0 || !qp->c0)) return TMPC_ERR_NULL_ARG;
  if (d->m > 0 && (!qp->G || !qp->l || !qp->u || !in->z_g || !in->y_g || !in->xi_g || !out->z_g || !out->y_g ||
                   !out->xi_g))
    return TMPC_ERR_NULL_ARG;
  if (!in->x || !in->y_fdyn || !in->rho_bar || !out->x || !out->y_fdyn || !out->rho_bar) return TMPC_ERR_NULL_ARG;
  if (d->n0 > 0 && (!in->y_f0 || !out->y_f0)) return TMPC_ERR_NULL_ARG;
  if (cfg->linsys != TMPC_LINSYS_PCG && cfg->linsys != TMPC_LINSYS_DIRECT && cfg->linsys != TMPC_LINSYS_PCG_PACKED)
    return TMPC_ERR_UNSUPPORTED;
  AdmmParams<R> P;
  P.qp = *qp;
  P.in = *in;
  P.out = *out;
  P.slack_weight = slack_weight;
  P.x_out = x_out;
  P.iters_out = iters_out;
  P.status_out = status_out;
  P.ws = static_cast<R*>(ws);
  P.T = d->T; P.n = d->n; P.nx = d->nx; P.n0 = d->n0; P.m = d->m; P.Nb = d->Nb;
  P.max_iter = cfg->max_iter; P.pcg_max_iter = cfg->pcg_max_iter; P.check_every = cfg->check_every;
  P.adapt_every = cfg->adapt_rho_every; P.use_slack = cfg->use_slack;
  P.eps_abs = (R)cfg->eps_abs; P.eps_rel = (R)cfg->eps_rel; P.sigma = (R)cfg->sigma;
  P.rho_f_factor = (R)cfg->rho_f_factor; P.alpha = (R)cfg->alpha; P.pcg_eps = (R)cfg->pcg_eps;
  P.adapt_tol = (R)cfg->adaptive_rho_tolerance; P.rho_min = (R)cfg->rho_min; P.rho_max = (R)cfg->rho_max;
  if constexpr (std::is_same<R, float>::value) {
    if (cfg->linsys == TMPC_LINSYS_PCG && admm_rows_ok(d->T, d->n, d->nx, d->n0, d->m))
      return launch_admm_rows(P, st);
  }
  if (d->n > 32) {  // stage blocks wider than 32: operators in the workspace (admm_generic.cu)
    if (cfg->linsys == TMPC_LINSYS_DIRECT) return TMPC_ERR_UNSUPPORTED;
    return launch_admm_generic<R>(P, ws_bytes, st);
  }
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    if (cfg->linsys == TMPC_LINSYS_DIRECT) {
      if (admm_il_ws_bytes<R>(*d) > 0) return launch_admm_direct_il<R>(P, ws_bytes, st);
      return launch_admm_direct_nb<NB, R>(P, ws_bytes, st);
    }
    return launch_admm_nb<NB, R>(P, ws_bytes, st);
  });
}

template int admm_solve<double>(const TmpcDims*, const TmpcQP*, const TmpcAdmmState*, const TmpcAdmmState*,
                                const double*, const TmpcAdmmConfig*, double*, uint32_t*, int32_t*, void*, size_t,
                                cudaStream_t);
template size_t admm_ws_bytes<double>(const TmpcDims&);
template size_t admm_ws_bytes_cfg<double>(const TmpcDims&, const TmpcAdmmConfig*);

}  // namespace tmpc

extern "C" {

size_t tmpc_admm_workspace_bytes(const TmpcDims* dims, int32_t dtype_bytes, const TmpcAdmmConfig* cfg) {
  if (tmpc::check_dims(dims)) return 0;
  return dtype_bytes == 8 ? tmpc::admm_ws_bytes_cfg<double>(*dims, cfg) : tmpc::admm_ws_bytes_cfg<float>(*dims, cfg);
}

int32_t tmpc_admm_solve_f32(const TmpcDims* dims, const TmpcQP* qp, const TmpcAdmmState* state_in,
                            const TmpcAdmmState* state_out, const float* slack_weight, const TmpcAdmmConfig* cfg,
                            float* x_out, uint32_t* iters_out, int32_t* status_out, void* workspace,
                            size_t workspace_bytes, tmpc_stream_t stream) {
  return tmpc::admm_solve<float>(dims, qp, state_in, state_out, slack_weight, cfg, x_out, iters_out, status_out,
                                 workspace, workspace_bytes, (cudaStream_t)stream);
}

int32_t tmpc_admm_solve_f64(const TmpcDims* dims, const TmpcQP* qp, const TmpcAdmmState* state_in,
                            const TmpcAdmmState* state_out, const double* slack_weight, const TmpcAdmmConfig* cfg,
                            double* x_out, uint32_t* iters_out, int32_t* status_out, void* workspace,
                            size_t workspace_bytes, tmpc_stream_t stream) {
  return tmpc::admm_solve<double>(dims, qp, state_in, state_out, slack_weight, cfg, x_out, iters_out, status_out,
                                  workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
