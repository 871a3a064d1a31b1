// Per-block-size kernels of the standalone Schur assembly and packed PCG.
#pragma once

#include "assemble.cuh"
#include "pcg_core.cuh"
#include "tma.cuh"
#include "tmpc_common.cuh"

namespace tmpc {

template <int NB, typename R>
__global__ void __launch_bounds__(256) assemble_packed_kernel(TmpcQP qpa, const R* rho, R sigma, R rho_f_factor,
                                                              R* ops, int32_t* status, int Nb, int T, int n, int nx,
                                                              int n0, int m) {
  const int b = blockIdx.x;
  if (b >= Nb) return;
  __shared__ int flag;
  if (threadIdx.x == 0) flag = 0;
  __syncthreads();
  const size_t opn = Geo<NB, R>::op_elems(T);
  const PackedAcc<NB, R> acc{ops + (size_t)b * 2 * opn, ops + (size_t)b * 2 * opn + opn, T};
  const QPView<R> qp = qp_view<R>(qpa, b, T, n, nx, n0, m);
  const R r = rho[b];
  assemble_ops<NB>(acc, qp, r * rho_f_factor, r, sigma, T, n, nx, n0, m, &flag);
  if (threadIdx.x == 0 && status) status[b] = flag;
}

template <int NB, typename R>
__global__ void __launch_bounds__(256) assemble_ref_kernel(TmpcQP qpa, const R* rho, R sigma, R rho_f_factor, R* S,
                                                           R* P, int32_t* status, int Nb, int T, int n, int nx,
                                                           int n0, int m) {
  const int b = blockIdx.x;
  if (b >= Nb) return;
  __shared__ int flag;
  if (threadIdx.x == 0) flag = 0;
  __syncthreads();
  const size_t per = (size_t)T * n * 3 * n;
  const RefAcc<R> acc{S + (size_t)b * per, P + (size_t)b * per, T, n};
  const QPView<R> qp = qp_view<R>(qpa, b, T, n, nx, n0, m);
  const R r = rho[b];
  assemble_ops<NB>(acc, qp, r * rho_f_factor, r, sigma, T, n, nx, n0, m, &flag);
  if (threadIdx.x == 0 && status) status[b] = flag;
}

// ---------------------------------------------------------------------------
// PCG on packed operators.  OPS_SMEM: the problem's operators are staged into
// shared memory by TMA bulk copies, then all iterations run on chip;
// otherwise they are streamed from HBM/L2 every iteration.
// ---------------------------------------------------------------------------
template <int NB, typename R, bool OPS_SMEM>
__global__ void __launch_bounds__(max_threads_for(NB)) pcg_packed_kernel(const R* __restrict__ ops,
                                                                 const R* __restrict__ rhs,
                                                                 const R* __restrict__ x0, R* x_out,
                                                                 uint32_t* iters_out, R eps, int max_iter, int Nb,
                                                                 int T, int n, uint32_t max_polls) {
  using Gm = Geo<NB, R>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  __shared__ __align__(8) uint64_t bar;
  __shared__ int tma_ok;
  const int b = blockIdx.x;
  if (b >= Nb) return;
  const size_t opn = Gm::op_elems(T);
  const R* gS = ops + (size_t)b * 2 * opn;
  const R* opS = gS;
  const R* opP = gS + opn;
  R* vb = sm;
  if constexpr (OPS_SMEM) {
    R* s_ops = sm;
    vb = sm + 2 * opn;
    if (threadIdx.x == 0) {
      tma_ok = 1;
      mbar_init(&bar, 1);
      const uint32_t bytes = (uint32_t)(2 * opn * sizeof(R));
      mbar_expect_tx(&bar, bytes);
      for (uint32_t off = 0; off < bytes; off += 65536u) {
        const uint32_t len = bytes - off < 65536u ? bytes - off : 65536u;
        bulk_g2s(reinterpret_cast<unsigned char*>(s_ops) + off, reinterpret_cast<const unsigned char*>(gS) + off,
                 len, &bar);
      }
    }
    opS = s_ops;
    opP = s_ops + opn;
  }
  const size_t VS = (size_t)T * Gm::VSTR;
  BlockVecs<NB, R> w{vb, vb + VS, vb + 2 * VS, vb + 3 * VS, vb + 4 * VS, vb + 5 * VS,
                     vb + 6 * VS, (int)VS};
  R* g = vb + 10 * VS;
  R* red = vb + 11 * VS;
  for (size_t e = threadIdx.x; e < 11 * VS; e += blockDim.x) vb[e] = R(0);
  __syncthreads();
  const int tot = T * n;
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    const int t = e / n, j = e - t * n;
    w.x[t * Gm::VSTR + j] = x0[(size_t)b * tot + e];
    g[t * Gm::VSTR + j] = rhs[(size_t)b * tot + e];
  }
  if constexpr (OPS_SMEM) {
    if (threadIdx.x == 0) {
      if (!mbar_wait_bounded(&bar, 0, max_polls)) {
        tma_ok = 0;
        // The CTA must not retire with bulk copies into its shared memory
        // still in flight: drain them (again with a bounded wait) first.
        mbar_wait_bounded(&bar, 0, kTransferDrainPolls);
      }
    }
  }
  __syncthreads();
  if constexpr (OPS_SMEM) {
    if (!tma_ok) {
      if (threadIdx.x == 0) iters_out[b] = 0xffffffffu;  // transfer timed out
      return;
    }
  }
  const int it = pcg_solve<NB, OPS_SMEM>(opS, opP, T, g, w, red, max_iter, eps);
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    const int t = e / n, j = e - t * n;
    x_out[(size_t)b * tot + e] = w.x[t * Gm::VSTR + j];
  }
  if (threadIdx.x == 0) iters_out[b] = (uint32_t)it;
}


template <int NB, typename R>
int launch_assemble_ref(const TmpcDims* d, const TmpcQP* qp, const R* rho, R sigma, R rff, R* S, R* P,
                        int32_t* status, cudaStream_t st) {
  assemble_ref_kernel<NB, R><<<d->Nb, 256, 0, st>>>(*qp, rho, sigma, rff, S, P, status, d->Nb, d->T, d->n, d->nx,
                                                    d->n0, d->m);
  return (int)cudaPeekAtLastError();
}

template <int NB, typename R>
int launch_assemble_packed(const TmpcDims* d, const TmpcQP* qp, const R* rho, R sigma, R rff, R* ops,
                           int32_t* status, cudaStream_t st) {
  assemble_packed_kernel<NB, R><<<d->Nb, 256, 0, st>>>(*qp, rho, sigma, rff, ops, status, d->Nb, d->T, d->n, d->nx,
                                                       d->n0, d->m);
  return (int)cudaPeekAtLastError();
}

template <int NB, typename R>
int launch_pcg_packed(const TmpcDims* d, const R* o, const R* rhs, const R* x0, R* xo, uint32_t* it, R eps,
                      int max_iter, cudaStream_t st) {
  using Gm = Geo<NB, R>;
  const int th = cta_threads(d->T, max_threads_for(NB));
  const int smax = max_dyn_smem();
  const size_t vec_bytes = (11 * (size_t)d->T * Gm::VSTR + 64) * sizeof(R);
  const size_t op_bytes = 2 * Gm::op_elems(d->T) * sizeof(R);
  if ((reinterpret_cast<uintptr_t>(o) & 15) != 0) return TMPC_ERR_WORKSPACE;  // 128-bit / bulk copies of the operators
  if ((long)(vec_bytes + op_bytes) <= smax) {
    auto k = pcg_packed_kernel<NB, R, true>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(vec_bytes + op_bytes));
    if (e != cudaSuccess) return (int)e;
    k<<<d->Nb, th, vec_bytes + op_bytes, st>>>(o, rhs, x0, xo, it, eps, max_iter, d->Nb, d->T, d->n,
                                                transfer_poll_limit().load());
  } else {
    if ((long)vec_bytes > smax) return (int)TMPC_ERR_SMEM;
    auto k = pcg_packed_kernel<NB, R, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)vec_bytes);
    if (e != cudaSuccess) return (int)e;
    k<<<d->Nb, th, vec_bytes, st>>>(o, rhs, x0, xo, it, eps, max_iter, d->Nb, d->T, d->n, 0u);
  }
  return (int)cudaPeekAtLastError();
}

}  // namespace tmpc
