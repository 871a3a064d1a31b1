// First-order (KKT) error of an SQP iterate against the QP linearised there,
// the convergence measure of the SQP loop (turbompc/solvers/
// turbompc_solver.py:1158-1225, "first_order" criterion), fused into one
// kernel per batch (one CTA per problem):
//   stat = || P z + q + C^T y_f + G^T y_g ||_inf
//          (P z)_t = D_t z_t + E_{t-1} z_{t-1} + E_t^T z_{t+1}
//          C^T y_f at t: A0^T y_f0 (t = 0) + Am_t^T y_t (t < N) + Ap_{t-1}^T y_{t-1} (t >= 1)
//   eq   = max(|| A0 z_0 - c0 ||_inf, || Am_t z_t + Ap_t z_{t+1} - c_t ||_inf)
//   g    = G_t z_t (+ slack, written to g_out), ineq = || max(l - g, 0, g - u) ||_inf
//   conv = max(stat, eq, ineq [, || w_s * slack + y_g ||_inf with soft constraints])
#include "tmpc_common.cuh"

namespace tmpc {

constexpr int kKktThreads = 128;

template <typename R>
__global__ void __launch_bounds__(kKktThreads) kkt_residual_kernel(TmpcQP qpa, const R* __restrict__ z,
                                                                   const R* __restrict__ yf0,
                                                                   const R* __restrict__ yfd,
                                                                   const R* __restrict__ yg,
                                                                   const R* __restrict__ slack,
                                                                   const R* __restrict__ sw, int use_slack,
                                                                   R* conv_out, R* eq_out, R* ineq_out, R* g_out,
                                                                   int Nb, int T, int n, int nx, int n0, int m) {
  const int b = blockIdx.x;
  if (b >= Nb) return;
  __shared__ R red[3][kKktThreads / 32];
  const int N = T - 1;
  const QPView<R> qp = qp_view<R>(qpa, b, T, n, nx, n0, m);
  const R* x = z + (size_t)b * T * n;
  const R* y0 = n0 > 0 ? yf0 + (size_t)b * n0 : nullptr;
  const R* yd = yfd + (size_t)b * N * nx;
  const R* ygb = m > 0 ? yg + (size_t)b * T * m : nullptr;
  const R* sl = (use_slack && m > 0) ? slack + (size_t)b * T * m : nullptr;
  R stat = R(0), eq = R(0), ineq = R(0);
  // stationarity, entry (t, j): each term's products in their own partial
  // sum (independent FMA chains whose loads can be in flight together),
  // added in the order of the formula
  constexpr int V = 16 / sizeof(R);
  const bool vec = n % V == 0 && (reinterpret_cast<uintptr_t>(qp.D) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(qp.E) & 15) == 0;
  for (int e = threadIdx.x; e < T * n; e += blockDim.x) {
    const int t = e / n, j = e - t * n;
    const R* xt = x + (size_t)t * n;
    R sd = R(0), se0 = R(0), se1 = R(0), s0 = R(0), sm = R(0), sp = R(0), sg = R(0);
    const R* Dt = qp.D + (size_t)t * n * n + (size_t)j * n;
    const R* Em = t > 0 ? qp.E + (size_t)(t - 1) * n * n + (size_t)j * n : nullptr;  // E_{t-1}[j][:]
    // rows of D_t and E_{t-1} are contiguous per thread: 128-bit loads where aligned
    if (vec) {
#pragma unroll 2
      for (int k = 0; k < n; k += V) {
        R w[V];
        ld128(w, Dt + k);
#pragma unroll
        for (int v = 0; v < V; ++v) sd = fma(w[v], xt[k + v], sd);
      }
      if (Em) {
#pragma unroll 2
        for (int k = 0; k < n; k += V) {
          R w[V];
          ld128(w, Em + k);
#pragma unroll
          for (int v = 0; v < V; ++v) se0 = fma(w[v], xt[k + v - n], se0);
        }
      }
    } else {
#pragma unroll 4
      for (int k = 0; k < n; ++k) sd = fma(Dt[k], xt[k], sd);
      if (Em) {
#pragma unroll 4
        for (int k = 0; k < n; ++k) se0 = fma(Em[k], xt[k - n], se0);
      }
    }
    if (t < N) {
      const R* Et = qp.E + (size_t)t * n * n;  // E_t[:][j]
#pragma unroll 4
      for (int k = 0; k < n; ++k) se1 = fma(Et[(size_t)k * n + j], xt[n + k], se1);
    }
    if (t == 0)
      for (int k = 0; k < n0; ++k) s0 = fma(qp.A0[(size_t)k * n + j], y0[k], s0);
    if (t < N) {
      const R* am = qp.Am + (size_t)t * nx * n;
#pragma unroll 4
      for (int k = 0; k < nx; ++k) sm = fma(am[(size_t)k * n + j], yd[(size_t)t * nx + k], sm);
    }
    if (t > 0) {
      const R* ap = qp.Ap + (size_t)(t - 1) * nx * n;
#pragma unroll 4
      for (int k = 0; k < nx; ++k) sp = fma(ap[(size_t)k * n + j], yd[(size_t)(t - 1) * nx + k], sp);
    }
#pragma unroll 4
    for (int k = 0; k < m; ++k) sg = fma(qp.G[((size_t)t * m + k) * n + j], ygb[(size_t)t * m + k], sg);
    const R s = (((((qp.q[e] + sd) + se0) + se1) + s0) + (sm + sp)) + sg;
    stat = fmax(stat, fabs(s));
  }
  // equality rows
  for (int e = threadIdx.x; e < n0 + N * nx; e += blockDim.x) {
    R s;
    if (e < n0) {
      s = -qp.c0[e];
      for (int k = 0; k < n; ++k) s = fma(qp.A0[(size_t)e * n + k], x[k], s);
    } else {
      const int r = e - n0, t = r / nx, i = r - t * nx;
      const R* am = qp.Am + ((size_t)t * nx + i) * n;
      const R* ap = qp.Ap + ((size_t)t * nx + i) * n;
      R sa = R(0), sb = R(0);
#pragma unroll 4
      for (int k = 0; k < n; ++k) sa = fma(am[k], x[(size_t)t * n + k], sa);
#pragma unroll 4
      for (int k = 0; k < n; ++k) sb = fma(ap[k], x[(size_t)(t + 1) * n + k], sb);
      s = (sa + sb) - qp.c[r];
    }
    eq = fmax(eq, fabs(s));
  }
  // inequality rows
  for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
    const int t = e / m;
    const R* gr = qp.G + (size_t)e * n;
    R s = R(0);
#pragma unroll 4
    for (int k = 0; k < n; ++k) s = fma(gr[k], x[(size_t)t * n + k], s);
    const R gb = sl ? s + sl[e] : s;
    g_out[(size_t)b * T * m + e] = gb;
    const R v = fmax(fmax(qp.l[e] - gb, R(0)), gb - qp.u[e]);
    ineq = fmax(ineq, v);
  }
  R slk = R(0);
  if (sl) {
    const R w = sw ? sw[b] : R(0);
    for (int e = threadIdx.x; e < T * m; e += blockDim.x) slk = fmax(slk, fabs(fma(w, sl[e], ygb[e])));
  }
  stat = warp_max(stat);
  eq = warp_max(eq);
  ineq = warp_max(fmax(ineq, R(0)));
  slk = warp_max(slk);
  __shared__ R rs[kKktThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    red[0][wid] = stat;
    red[1][wid] = eq;
    red[2][wid] = ineq;
    rs[wid] = slk;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    R a = R(0), c = R(0), d = R(0), f = R(0);
    for (int w = 0; w < kKktThreads / 32; ++w) {
      a = fmax(a, red[0][w]);
      c = fmax(c, red[1][w]);
      d = fmax(d, red[2][w]);
      f = fmax(f, rs[w]);
    }
    R conv = fmax(a, fmax(c, d));
    if (sl) conv = fmax(conv, f);
    conv_out[b] = conv;
    eq_out[b] = c;
    ineq_out[b] = d;
  }
}

template <typename R>
int kkt_residual(const TmpcDims* d, const TmpcQP* qp, const R* z, const R* yf0, const R* yfd, const R* yg,
                 const R* slack, const R* sw, int use_slack, R* conv, R* eq, R* ineq, R* g, cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!qp || !z || !yfd || !conv || !eq || !ineq) return TMPC_ERR_NULL_ARG;
  if (!qp->D || !qp->E || !qp->q || !qp->A_minus || !qp->A_plus || !qp->c) return TMPC_ERR_NULL_ARG;
  if (d->n0 > 0 && (!qp->A0 || !qp->c0 || !yf0)) return TMPC_ERR_NULL_ARG;
  if (d->m > 0 && (!qp->G || !qp->l || !qp->u || !yg || !g)) return TMPC_ERR_NULL_ARG;
  if (use_slack && d->m > 0 && !slack) return TMPC_ERR_NULL_ARG;
  kkt_residual_kernel<R><<<d->Nb, kKktThreads, 0, st>>>(*qp, z, yf0, yfd, yg, slack, sw, use_slack, conv, eq, ineq,
                                                        g, d->Nb, d->T, d->n, d->nx, d->n0, d->m);
  return (int)cudaPeekAtLastError();
}

}  // namespace tmpc

extern "C" {

int32_t tmpc_first_order_error_f32(const TmpcDims* dims, const TmpcQP* qp, const float* z, const float* y_f0,
                                   const float* y_fdyn, const float* y_g, const float* slack,
                                   const float* slack_weight, int32_t use_slack, float* conv_out, float* eq_out,
                                   float* ineq_out, float* g_out, tmpc_stream_t stream) {
  return tmpc::kkt_residual<float>(dims, qp, z, y_f0, y_fdyn, y_g, slack, slack_weight, use_slack, conv_out, eq_out,
                                   ineq_out, g_out, (cudaStream_t)stream);
}

int32_t tmpc_first_order_error_f64(const TmpcDims* dims, const TmpcQP* qp, const double* z, const double* y_f0,
                                   const double* y_fdyn, const double* y_g, const double* slack,
                                   const double* slack_weight, int32_t use_slack, double* conv_out, double* eq_out,
                                   double* ineq_out, double* g_out, tmpc_stream_t stream) {
  return tmpc::kkt_residual<double>(dims, qp, z, y_f0, y_fdyn, y_g, slack, slack_weight, use_slack, conv_out,
                                    eq_out, ineq_out, g_out, (cudaStream_t)stream);
}

}  // extern "C"
