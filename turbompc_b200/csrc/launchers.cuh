// Declarations of the per-block-size launchers.  Each is defined in a kernel
// header and explicitly instantiated once per NB in inst_nb*.cu, so that the
// heavy kernels compile in parallel translation units.
#pragma once

#include "tmpc_common.cuh"

namespace tmpc {

template <typename R>
struct AdmmParams;

template <int NB, typename R>
int launch_admm_direct_nb(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st);
template <int NB, typename R>
int launch_admm_nb(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st);
template <int NB, typename R>
size_t admm_smem_bytes(int T, int nx, int n0, int m, bool ops_smem);
template <int NB, typename R>
int launch_assemble_ref(const TmpcDims* d, const TmpcQP* qp, const R* rho, R sigma, R rff, R* S, R* P,
                        int32_t* status, cudaStream_t st);
template <int NB, typename R>
int launch_assemble_packed(const TmpcDims* d, const TmpcQP* qp, const R* rho, R sigma, R rff, R* ops,
                           int32_t* status, cudaStream_t st);
template <int NB, typename R>
int launch_pcg_packed(const TmpcDims* d, const R* o, const R* rhs, const R* x0, R* xo, uint32_t* it, R eps,
                      int max_iter, cudaStream_t st);

// Stage blocks wider than 32 (32 < n <= 96; admm_generic.cu).
template <typename R>
size_t admm_generic_ws_bytes(const TmpcDims& d);
template <typename R>
int launch_admm_generic(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st);
template <typename R>
int assemble_generic(const TmpcDims* d, const TmpcQP* qp, const R* rho, R sigma, R rff, R* S, R* P, int32_t* status,
                     cudaStream_t st);

// Direct solve on the batch-interleaved layout (admm_il.cu): workspace bytes
// (0 where it does not apply) and the launch (TMPC_ERR_UNSUPPORTED where it
// does not apply).
template <typename R>
size_t admm_il_ws_bytes(const TmpcDims& d);
template <typename R>
int launch_admm_direct_il(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st);

// Register-resident kernel for 8 < n <= 16, T <= 64, fp32 (admm_rows.cu).
bool admm_rows_ok(int T, int n, int nx, int n0, int m);
int launch_admm_rows(const AdmmParams<float>& P, cudaStream_t st);

template <typename R>
struct AdmmParams {
  TmpcQP qp;
  TmpcAdmmState in, out;
  const R* slack_weight;
  R* x_out;
  uint32_t* iters_out;
  int32_t* status_out;
  R* ws;  // operators in HBM when they do not fit on chip
  int T, n, nx, n0, m, Nb;
  int max_iter, pcg_max_iter, check_every, adapt_every, use_slack;
  R eps_abs, eps_rel, sigma, rho_f_factor, alpha, pcg_eps, adapt_tol, rho_min, rho_max;
};

}  // namespace tmpc
