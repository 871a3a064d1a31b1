// Standalone Schur assembly (compute_S_Phiinv) and batched block-tridiagonal
// PCG (pcg_blktridi_cuda) entry points.
#include "launchers.cuh"

namespace tmpc {

// ---------------------------------------------------------------------------
// PCG on the reference layout: one CTA per problem, vectors in shared memory,
// one thread per row of S/Phiinv reading the row's entries from HBM through
// the read-only path.  Semantics of pcgBlkTridiSingleBlock
// (pcg_blktridi.cu:96-229), for every T*n.
// ---------------------------------------------------------------------------
template <typename R>
__device__ __forceinline__ void ref_matvec(R* y, const R* __restrict__ M, const R* v, int T, int n) {
  const int tot = T * n;
  const int n3 = 3 * n;
  for (int row = threadIdx.x; row < tot; row += blockDim.x) {
    const int t = row / n;
    const R* mr = M + (size_t)row * n3;
    R s = R(0);
    const int j0 = t > 0 ? 0 : n;
    const int j1 = t < T - 1 ? n3 : 2 * n;
    for (int j = j0; j < j1; ++j) s = fma(__ldg(mr + j), v[(t - 1) * n + j], s);
    y[row] = s;
  }
}

template <typename R>
__global__ void __launch_bounds__(512) pcg_ref_kernel(const R* __restrict__ S, const R* __restrict__ Pm,
                                                      const R* __restrict__ rhs, const R* __restrict__ x0, R* x_out,
                                                      uint32_t* iters_out, R eps, int max_iter, int Nb, int T,
                                                      int n) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  const int b = blockIdx.x;
  if (b >= Nb) return;
  const int tot = T * n;
  R* x = sm;
  R* r = x + tot;
  R* z = r + tot;
  R* p = z + tot;
  R* sp = p + tot;
  R* red = sp + tot;
  const size_t mo = (size_t)b * tot * 3 * n;
  const R* Sb = S + mo;
  const R* Pb = Pm + mo;
  for (int i = threadIdx.x; i < tot; i += blockDim.x) x[i] = x0[(size_t)b * tot + i];
  __syncthreads();
  ref_matvec(sp, Sb, x, T, n);
  __syncthreads();
  for (int i = threadIdx.x; i < tot; i += blockDim.x) r[i] = rhs[(size_t)b * tot + i] - sp[i];
  __syncthreads();
  ref_matvec(z, Pb, r, T, n);
  __syncthreads();
  R part = R(0);
  for (int i = threadIdx.x; i < tot; i += blockDim.x) {
    p[i] = z[i];
    part = fma(r[i], z[i], part);
  }
  R eta = block_sum(part, red);
  const R eta0 = fabs(eta);
  int it = 0;
  for (; it < max_iter; ++it) {
    if (fabs(eta) < R(1e-12) + eps * eta0) break;
    __syncthreads();
    ref_matvec(sp, Sb, p, T, n);
    __syncthreads();
    part = R(0);
    for (int i = threadIdx.x; i < tot; i += blockDim.x) part = fma(p[i], sp[i], part);
    R den = block_sum(part, red + 32);
    if (fabs(den) < R(1e-30)) den = R(1e-30);
    const R a = eta / den;
    for (int i = threadIdx.x; i < tot; i += blockDim.x) {
      x[i] = fma(a, p[i], x[i]);
      r[i] = fma(-a, sp[i], r[i]);
    }
    __syncthreads();
    ref_matvec(z, Pb, r, T, n);
    __syncthreads();
    part = R(0);
    for (int i = threadIdx.x; i < tot; i += blockDim.x) part = fma(r[i], z[i], part);
    const R en = block_sum(part, red);
    const R beta = en / eta;
    eta = en;
    for (int i = threadIdx.x; i < tot; i += blockDim.x) p[i] = fma(beta, p[i], z[i]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < tot; i += blockDim.x) x_out[(size_t)b * tot + i] = x[i];
  if (threadIdx.x == 0) iters_out[b] = (uint32_t)it;
}

template <typename R>
int schur_assemble(const TmpcDims* d, const TmpcQP* qp, const R* rho, double sigma, double rff, R* S, R* P,
                   int32_t* status, cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!qp || !rho || !S || !P || !qp->D || !qp->E || !qp->A_minus || !qp->A_plus) return TMPC_ERR_NULL_ARG;
  if (d->n0 > 0 && !qp->A0) return TMPC_ERR_NULL_ARG;
  if (d->m > 0 && !qp->G) return TMPC_ERR_NULL_ARG;
  if (d->Nb == 0) return TMPC_OK;
  if (d->n > 32) return assemble_generic<R>(d, qp, rho, (R)sigma, (R)rff, S, P, status, st);
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    return launch_assemble_ref<NB, R>(d, qp, rho, (R)sigma, (R)rff, S, P, status, st);
  });
}

template <typename R>
int schur_assemble_packed(const TmpcDims* d, const TmpcQP* qp, const R* rho, double sigma, double rff, void* ops,
                          int32_t* status, cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!qp || !rho || !ops || !qp->D || !qp->E || !qp->A_minus || !qp->A_plus) return TMPC_ERR_NULL_ARG;
  if (d->n0 > 0 && !qp->A0) return TMPC_ERR_NULL_ARG;
  if (d->m > 0 && !qp->G) return TMPC_ERR_NULL_ARG;
  if (d->Nb == 0) return TMPC_OK;
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    return launch_assemble_packed<NB, R>(d, qp, rho, (R)sigma, (R)rff, static_cast<R*>(ops), status, st);
  });
}

template <typename R>
int pcg_ref(const TmpcDims* d, const R* S, const R* P, const R* rhs, const R* x0, R* xo, uint32_t* it, double eps,
            int max_iter, cudaStream_t st) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 1 || d->n < 1) return TMPC_ERR_BAD_DIMS;
  if (!S || !P || !rhs || !x0 || !xo || !it) return TMPC_ERR_NULL_ARG;
  if (d->Nb == 0) return TMPC_OK;
  const int tot = d->T * d->n;
  int th = (tot + 31) / 32 * 32;
  if (th > 512) th = 512;
  if (th < 32) th = 32;
  const size_t smem = (5 * (size_t)tot + 64) * sizeof(R);
  if ((long)smem > max_dyn_smem()) return TMPC_ERR_SMEM;
  cudaError_t e = cudaFuncSetAttribute(pcg_ref_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  pcg_ref_kernel<R><<<d->Nb, th, smem, st>>>(S, P, rhs, x0, xo, it, (R)eps, max_iter, d->Nb, d->T, d->n);
  return (int)cudaPeekAtLastError();
}

template <typename R>
int pcg_packed(const TmpcDims* d, const void* ops, const R* rhs, const R* x0, R* xo, uint32_t* it, double eps,
               int max_iter, cudaStream_t st) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 2 || d->n < 1) return TMPC_ERR_BAD_DIMS;
  if (!ops || !rhs || !x0 || !xo || !it) return TMPC_ERR_NULL_ARG;
  if (d->Nb == 0) return TMPC_OK;
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    return launch_pcg_packed<NB, R>(d, static_cast<const R*>(ops), rhs, x0, xo, it, (R)eps, max_iter, st);
  });
}

}  // namespace tmpc

extern "C" {

size_t tmpc_packed_operator_bytes(const TmpcDims* d, int32_t dtype_bytes) {
  if (tmpc::check_dims(d)) return 0;
  size_t out = 0;
  tmpc::dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    out = dtype_bytes == 8 ? (size_t)d->Nb * 2 * tmpc::Geo<NB, double>::op_elems(d->T) * sizeof(double)
                           : (size_t)d->Nb * 2 * tmpc::Geo<NB, float>::op_elems(d->T) * sizeof(float);
    return 0;
  });
  return out;
}

int32_t tmpc_schur_assemble_f32(const TmpcDims* dims, const TmpcQP* qp, const float* rho_bar, double sigma,
                                double rho_f_factor, float* S, float* Phiinv, int32_t* status_out,
                                tmpc_stream_t stream) {
  return tmpc::schur_assemble<float>(dims, qp, rho_bar, sigma, rho_f_factor, S, Phiinv, status_out,
                                     (cudaStream_t)stream);
}
int32_t tmpc_schur_assemble_f64(const TmpcDims* dims, const TmpcQP* qp, const double* rho_bar, double sigma,
                                double rho_f_factor, double* S, double* Phiinv, int32_t* status_out,
                                tmpc_stream_t stream) {
  return tmpc::schur_assemble<double>(dims, qp, rho_bar, sigma, rho_f_factor, S, Phiinv, status_out,
                                      (cudaStream_t)stream);
}
int32_t tmpc_schur_assemble_packed_f32(const TmpcDims* dims, const TmpcQP* qp, const float* rho_bar, double sigma,
                                       double rho_f_factor, void* ops, int32_t* status_out, tmpc_stream_t stream) {
  return tmpc::schur_assemble_packed<float>(dims, qp, rho_bar, sigma, rho_f_factor, ops, status_out,
                                            (cudaStream_t)stream);
}
int32_t tmpc_schur_assemble_packed_f64(const TmpcDims* dims, const TmpcQP* qp, const double* rho_bar, double sigma,
                                       double rho_f_factor, void* ops, int32_t* status_out, tmpc_stream_t stream) {
  return tmpc::schur_assemble_packed<double>(dims, qp, rho_bar, sigma, rho_f_factor, ops, status_out,
                                             (cudaStream_t)stream);
}
int32_t tmpc_pcg_solve_f32(const TmpcDims* dims, const float* S, const float* Phiinv, const float* rhs,
                           const float* x0, float* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                           tmpc_stream_t stream) {
  return tmpc::pcg_ref<float>(dims, S, Phiinv, rhs, x0, x_out, iters_out, eps, max_iters, (cudaStream_t)stream);
}
int32_t tmpc_pcg_solve_f64(const TmpcDims* dims, const double* S, const double* Phiinv, const double* rhs,
                           const double* x0, double* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                           tmpc_stream_t stream) {
  return tmpc::pcg_ref<double>(dims, S, Phiinv, rhs, x0, x_out, iters_out, eps, max_iters, (cudaStream_t)stream);
}
int32_t tmpc_pcg_solve_packed_f32(const TmpcDims* dims, const void* ops, const float* rhs, const float* x0,
                                  float* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                                  tmpc_stream_t stream) {
  return tmpc::pcg_packed<float>(dims, ops, rhs, x0, x_out, iters_out, eps, max_iters, (cudaStream_t)stream);
}
int32_t tmpc_pcg_solve_packed_f64(const TmpcDims* dims, const void* ops, const double* rhs, const double* x0,
                                  double* x_out, uint32_t* iters_out, double eps, int32_t max_iters,
                                  tmpc_stream_t stream) {
  return tmpc::pcg_packed<double>(dims, ops, rhs, x0, x_out, iters_out, eps, max_iters, (cudaStream_t)stream);
}

}  // extern "C"
