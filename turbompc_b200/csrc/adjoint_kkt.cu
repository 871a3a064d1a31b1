// Adjoint (backward) KKT solve, one CTA per problem.
//
// Solves  [P  C^T] [dz]   [-q]
//         [C  R  ] [mu] = [ 0]        (turbompc/solvers/backward/backward_kkt_jax.py:10-211)
// with P = blocktridiag(E_{t-1}, D_t, E_t^T), C = [A0 rows; dynamics rows
// Am_t z_t + Ap_t z_{t+1}; G_t rows] and R = -1e-12 on the diagonal of G rows
// that are entirely zero (inactive inequalities).
//
// The unknowns are grouped by stage, v_t = [lam_t, z_t, mu_t], where lam_0 is
// the multiplier of the A0 rows and lam_{t+1} the multiplier of dynamics
// row-block t (so every stage block carries exactly one equality block that
// touches z_t with full row rank for explicit integrators).  The KKT matrix is
// then block tridiagonal and symmetric:
//   K_tt     = [[0, Ap_{t-1} (or A0)], [.^T, D_t, G_t^T], [0, G_t, R_t]]
//   K_{t,t+1} has nonzeros only in the z_t rows: [Am_t^T (lam_{t+1} cols), E_t^T (z_{t+1} cols)] =: U_t
// Block elimination forward in t:
//   K'_t = K_tt - U_{t-1}^T [K'_{t-1}^-1]_zz U_{t-1}   (on the (lam_t, z_t) block)
//   [X_t | w_t] = K'_t^-1 [B_t | y_t],  B_t = U_t in the z rows, 0 elsewhere
//   y_{t+1}     = b_{t+1} - U_t^T w_t[z]
// and back substitution v_N = w_N, v_t = w_t - X_t v_{t+1}[lam, z].
// Each K'_t is inverted (applied) by Gauss-Jordan elimination with partial
// pivoting on the augmented block [K'_t | B_t | y_t] in shared memory; a zero
// pivot sets TMPC_STATUS_SINGULAR_BLOCK (no trap).  X_t and w_t are kept in
// the caller's workspace for the back substitution.
#include "tmpc_common.cuh"

namespace tmpc {

constexpr int kKktThreads = 256;

template <typename R>
__global__ void __launch_bounds__(kKktThreads) adjoint_kkt_kernel(TmpcQP qpa, R* dz_out, R* mult_out,
                                                                  int32_t* status, R* ws, int Nb, int T, int n,
                                                                  int nx, int n0, int m) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  const int b = blockIdx.x;
  if (b >= Nb) return;
  const int N = T - 1;
  const int c = nx + n;                       // coupling columns (lam_{t+1}, z_{t+1})
  const int smax = (n0 > nx ? n0 : nx) + n + m;
  const int W = smax + c + 1;                 // augmented row length
  R* A = sm;                                  // [smax][W]
  R* Xz = A + (size_t)smax * W;               // previous stage's X[z rows] (n x c) and w[z] (n)
  R* wz = Xz + (size_t)n * c;
  R* fac = wz + n;                            // elimination factors (smax)
  int* piv = reinterpret_cast<int*>(fac + smax);
  __shared__ int flag;
  if (threadIdx.x == 0) flag = 0;
  const QPView<R> qp = qp_view<R>(qpa, b, T, n, nx, n0, m);
  const size_t stage_ws = (size_t)smax * (c + 1);
  R* wsb = ws + (size_t)b * T * stage_ws;
  __syncthreads();

  for (int t = 0; t < T; ++t) {
    const int nl = (t == 0) ? n0 : nx;  // lam rows of this stage
    const int s = nl + n + m;
    // ---- assemble [K'_t | B_t | y_t]
    for (int e = threadIdx.x; e < s * W; e += blockDim.x) {
      const int i = e / W, j = e - i * W;
      R v = R(0);
      if (j < s) {
        // K_tt (symmetric), rows/cols ordered [lam (nl), z (n), mu (m)]
        const int ir = i < nl ? 0 : (i < nl + n ? 1 : 2), jr = j < nl ? 0 : (j < nl + n ? 1 : 2);
        const int ii = i - (ir == 0 ? 0 : (ir == 1 ? nl : nl + n));
        const int jj = j - (jr == 0 ? 0 : (jr == 1 ? nl : nl + n));
        if (ir == 1 && jr == 1) {
          v = qp.D[((size_t)t * n + ii) * n + jj];
        } else if (ir == 0 && jr == 1) {
          v = (t == 0) ? qp.A0[ii * n + jj] : qp.Ap[((size_t)(t - 1) * nx + ii) * n + jj];
        } else if (ir == 1 && jr == 0) {
          v = (t == 0) ? qp.A0[jj * n + ii] : qp.Ap[((size_t)(t - 1) * nx + jj) * n + ii];
        } else if (ir == 2 && jr == 1) {
          v = qp.G[((size_t)t * m + ii) * n + jj];
        } else if (ir == 1 && jr == 2) {
          v = qp.G[((size_t)t * m + jj) * n + ii];
        } else if (ir == 2 && jr == 2 && ii == jj) {
          R g2 = R(0);
          for (int k = 0; k < n; ++k) {
            const R gv = qp.G[((size_t)t * m + ii) * n + k];
            g2 += gv * gv;
          }
          v = (g2 == R(0)) ? R(-1e-12) : R(0);
        }
        // Schur correction on the (lam, z) block: - U_{t-1}^T Xz_{t-1}
        if (t > 0 && ir <= 1 && jr <= 1) {
          const int a = (ir == 0 ? ii : nx + ii), bcol = (jr == 0 ? jj : nx + jj);  // index into c
          R s2 = R(0);
          for (int k = 0; k < n; ++k) {
            // U_{t-1}[k][a]: a < nx -> Am_{t-1}[a][k]; else E_{t-1}[a-nx][k]
            const R u = a < nx ? qp.Am[((size_t)(t - 1) * nx + a) * n + k] : qp.E[((size_t)(t - 1) * n + (a - nx)) * n + k];
            s2 += u * Xz[k * c + bcol];
          }
          v -= s2;
        }
      } else if (j < s + c) {
        // B_t: z rows hold U_t = [Am_t^T, E_t^T] (only for t < N)
        const int jc = j - s;
        if (t < N && i >= nl && i < nl + n) {
          const int k = i - nl;
          v = jc < nx ? qp.Am[((size_t)t * nx + jc) * n + k] : qp.E[((size_t)t * n + (jc - nx)) * n + k];
        }
      } else {
        // y_t = b_t - U_{t-1}^T w_{t-1}[z]; b_t = [0, -q_t, 0]
        if (i >= nl && i < nl + n) v = -qp.q[t * n + (i - nl)];
        if (t > 0 && i < nl + n) {
          const int a = (i < nl ? i : nx + (i - nl));
          R s2 = R(0);
          for (int k = 0; k < n; ++k) {
            const R u = a < nx ? qp.Am[((size_t)(t - 1) * nx + a) * n + k] : qp.E[((size_t)(t - 1) * n + (a - nx)) * n + k];
            s2 += u * wz[k];
          }
          v -= s2;
        }
      }
      A[i * W + j] = v;
    }
    __syncthreads();
    // ---- Gauss-Jordan with partial pivoting on the first s columns
    for (int k = 0; k < s; ++k) {
      if (threadIdx.x < 32) {
        R best = R(-1);
        int bi = k;
        for (int i = k + threadIdx.x; i < s; i += 32) {
          const R a = fabs(A[i * W + k]);
          if (a > best) {
            best = a;
            bi = i;
          }
        }
        for (int o = 16; o > 0; o >>= 1) {
          const R ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ob > best || (ob == best && oi < bi)) {
            best = ob;
            bi = oi;
          }
        }
        if (threadIdx.x == 0) {
          piv[0] = bi;
          if (!(best > R(0)) || !isfinite(best)) flag |= TMPC_STATUS_SINGULAR_BLOCK;
        }
      }
      __syncthreads();
      const int p = piv[0];
      if (p != k) {
        for (int j = k + threadIdx.x; j < W; j += blockDim.x) {
          const R tmp = A[k * W + j];
          A[k * W + j] = A[p * W + j];
          A[p * W + j] = tmp;
        }
        __syncthreads();
      }
      const R inv = R(1) / A[k * W + k];
      for (int i = threadIdx.x; i < s; i += blockDim.x) fac[i] = A[i * W + k];
      __syncthreads();
      for (int j = k + 1 + threadIdx.x; j < W; j += blockDim.x) A[k * W + j] *= inv;
      __syncthreads();
      const int wcols = W - (k + 1);
      for (int e = threadIdx.x; e < s * wcols; e += blockDim.x) {
        const int i = e / wcols, j = k + 1 + e % wcols;
        if (i != k) A[i * W + j] -= fac[i] * A[k * W + j];
      }
      __syncthreads();
    }
    // ---- keep X_t, w_t (rows 0..s) in the workspace; X[z], w[z] on chip
    R* st = wsb + (size_t)t * stage_ws;
    for (int e = threadIdx.x; e < s * (c + 1); e += blockDim.x) {
      const int i = e / (c + 1), j = e - i * (c + 1);
      st[e] = A[i * W + s + j];  // columns s .. s + c (X then w)
    }
    for (int e = threadIdx.x; e < n * (c + 1); e += blockDim.x) {
      const int k = e / (c + 1), j = e - k * (c + 1);
      const R v = A[(nl + k) * W + s + j];
      if (j < c) Xz[k * c + j] = v;
      else wz[k] = v;
    }
    __syncthreads();
  }
  // ---- back substitution: v_N = w_N, v_t = w_t - X_t v_{t+1}[lam, z]
  // A's first row holds v_{t+1}[lam, z] (length c) between steps.
  R* vnext = A;
  R* vcur = A + smax + c;
  for (int t = N; t >= 0; --t) {
    const int nl = (t == 0) ? n0 : nx;
    const int s = nl + n + m;
    const R* stg = wsb + (size_t)t * stage_ws;
    for (int i = threadIdx.x; i < s; i += blockDim.x) {
      R v = stg[i * (c + 1) + c];
      if (t < N) {
        R s2 = R(0);
        for (int j = 0; j < c; ++j) s2 += stg[i * (c + 1) + j] * vnext[j];
        v -= s2;
      }
      vcur[i] = v;
    }
    __syncthreads();
    // outputs
    for (int i = threadIdx.x; i < s; i += blockDim.x) {
      const R v = vcur[i];
      if (i < nl) {
        if (t == 0) mult_out[(size_t)b * (n0 + N * nx + T * m) + i] = v;
        else mult_out[(size_t)b * (n0 + N * nx + T * m) + n0 + (t - 1) * nx + i] = v;
      } else if (i < nl + n) {
        dz_out[((size_t)b * T + t) * n + (i - nl)] = v;
      } else {
        mult_out[(size_t)b * (n0 + N * nx + T * m) + n0 + N * nx + t * m + (i - nl - n)] = v;
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nl + n; i += blockDim.x) vnext[i] = vcur[i];  // [lam_t, z_t] for stage t-1
    __syncthreads();
  }
  if (threadIdx.x == 0 && status) status[b] = flag;
}

template <typename R>
size_t kkt_ws_bytes(const TmpcDims& d) {
  const int smax = (d.n0 > d.nx ? d.n0 : d.nx) + d.n + d.m;
  return (size_t)d.Nb * d.T * smax * (d.nx + d.n + 1) * sizeof(R);
}

template <typename R>
size_t kkt_smem_bytes(const TmpcDims& d) {
  const int smax = (d.n0 > d.nx ? d.n0 : d.nx) + d.n + d.m;
  const int c = d.nx + d.n;
  const size_t W = smax + c + 1;
  return ((size_t)smax * W + (size_t)d.n * c + d.n + smax) * sizeof(R) + 16;
}

template <typename R>
int adjoint_kkt(const TmpcDims* d, const TmpcQP* qp, R* dz, R* mult, int32_t* status, void* ws, size_t ws_bytes,
                cudaStream_t st) {
  int rc = check_dims(d);
  if (rc) return rc;
  if (d->Nb == 0) return TMPC_OK;
  if (!qp || !dz || !mult || !qp->D || !qp->E || !qp->q || !qp->A0 || !qp->A_minus || !qp->A_plus)
    return TMPC_ERR_NULL_ARG;
  if (d->m > 0 && !qp->G) return TMPC_ERR_NULL_ARG;
  if (!ws || ws_bytes < kkt_ws_bytes<R>(*d)) return TMPC_ERR_WORKSPACE;
  const size_t smem = kkt_smem_bytes<R>(*d);
  if ((long)smem > max_dyn_smem()) return TMPC_ERR_SMEM;
  cudaError_t e =
      cudaFuncSetAttribute(adjoint_kkt_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  adjoint_kkt_kernel<R><<<d->Nb, kKktThreads, smem, st>>>(*qp, dz, mult, status, static_cast<R*>(ws), d->Nb, d->T,
                                                          d->n, d->nx, d->n0, d->m);
  return (int)cudaPeekAtLastError();
}

}  // namespace tmpc

extern "C" {

size_t tmpc_adjoint_kkt_workspace_bytes(const TmpcDims* dims, int32_t dtype_bytes) {
  if (tmpc::check_dims(dims)) return 0;
  return dtype_bytes == 8 ? tmpc::kkt_ws_bytes<double>(*dims) : tmpc::kkt_ws_bytes<float>(*dims);
}

int32_t tmpc_adjoint_kkt_solve_f32(const TmpcDims* dims, const TmpcQP* qp, float* dz_out, float* mult_out,
                                   int32_t* status_out, void* workspace, size_t workspace_bytes,
                                   tmpc_stream_t stream) {
  return tmpc::adjoint_kkt<float>(dims, qp, dz_out, mult_out, status_out, workspace, workspace_bytes,
                                  (cudaStream_t)stream);
}
int32_t tmpc_adjoint_kkt_solve_f64(const TmpcDims* dims, const TmpcQP* qp, double* dz_out, double* mult_out,
                                   int32_t* status_out, void* workspace, size_t workspace_bytes,
                                   tmpc_stream_t stream) {
  return tmpc::adjoint_kkt<double>(dims, qp, dz_out, mult_out, status_out, workspace, workspace_bytes,
                                   (cudaStream_t)stream);
}

}  // extern "C"
