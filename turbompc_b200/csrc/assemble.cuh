// CTA-level assembly of the Schur operator S and the preconditioner Phiinv of
// one problem.
//
// Math (turbompc/solvers/admm/admm.py:71-154):
//   Theta_t = D_t + sigma I + rho_ineq G_t^T G_t
//             + rho_f (A0^T A0 + Am_0^T Am_0)                 t = 0
//             + rho_f (Ap_{t-1}^T Ap_{t-1} + Am_t^T Am_t)      0 < t < N
//             + rho_f  Ap_{N-1}^T Ap_{N-1}                     t = N
//   Phi_t   = E_t + rho_f Ap_t^T Am_t                          (block (t+1, t))
//   S       = blocktridiag(Phi_{t-1}, Theta_t, Phi_t^T)
//   Phiinv  = blocktridiag(Theta_t^-1 Phi_{t-1} Theta_{t-1}^-1, -Theta_t^-1,
//                          Theta_t^-1 Phi_t^T Theta_{t+1}^-1)
// Theta_t^-1 comes from Gauss-Jordan elimination with partial pivoting (the
// reference inverts with jnp.linalg.inv and, on device, with Gauss-Jordan,
// admm/csrc/admm_math.cuh:248-310), done here by one warp per block entirely
// in registers: lane c owns column c of [Theta | I].
//
// The destination is abstracted by an accessor:
//   PackedAcc  packed on-chip/HBM format (tmpc_common.cuh)
//   RefAcc     the reference layout S, Phiinv [T][n][3n]
#pragma once

#include "tmpc_common.cuh"

namespace tmpc {

template <int NB, typename R>
struct PackedAcc {
  R* opS;
  R* opP;
  int T;
  using Gm = Geo<NB, R>;
  __device__ R* sd(int t) const { return opS + (size_t)t * Gm::DSTR; }
  __device__ R* so(int t) const { return opS + (size_t)T * Gm::DSTR + (size_t)t * Gm::OSTR; }
  __device__ R* pd(int t) const { return opP + (size_t)t * Gm::DSTR; }
  __device__ R* po(int t) const { return opP + (size_t)T * Gm::DSTR + (size_t)t * Gm::OSTR; }
  __device__ void set_theta(int t, int i, int j, R v) const { sd(t)[tri_index(i, j, NB)] = v; }  // i <= j
  __device__ R get_theta(int t, int i, int j) const { return sd(t)[tri_index(i, j, NB)]; }      // i <= j
  __device__ void set_phi(int t, int i, int j, R v) const { so(t)[i * NB + j] = v; }
  __device__ R get_phi(int t, int i, int j) const { return so(t)[i * NB + j]; }
  __device__ void set_ntinv(int t, int i, int j, R v) const { pd(t)[tri_index(i, j, NB)] = v; }  // i <= j
  __device__ R get_ntinv(int t, int i, int j) const {
    return i <= j ? pd(t)[tri_index(i, j, NB)] : pd(t)[tri_index(j, i, NB)];
  }
  __device__ void set_m(int t, int i, int j, R v) const { po(t)[i * NB + j] = v; }
  // Zero the 128-bit-load tails of the diagonal blocks.
  __device__ void init() const {
    constexpr int TL = Gm::DSTR - Gm::TRI;
    for (int e = threadIdx.x; e < T * TL; e += blockDim.x) {
      const int t = e / TL, k = e - t * TL;
      sd(t)[Gm::TRI + k] = R(0);
      pd(t)[Gm::TRI + k] = R(0);
    }
  }
};

template <typename R>
struct RefAcc {
  R* S;  // [T][n][3n]
  R* P;  // [T][n][3n]
  int T, n;
  __device__ R* srow(int t, int i) const { return S + ((size_t)t * n + i) * 3 * n; }
  __device__ R* prow(int t, int i) const { return P + ((size_t)t * n + i) * 3 * n; }
  __device__ void set_theta(int t, int i, int j, R v) const {
    if (i < n && j < n) {
      srow(t, i)[n + j] = v;
      srow(t, j)[n + i] = v;
    }
  }
  __device__ R get_theta(int t, int i, int j) const { return (i < n && j < n) ? srow(t, i)[n + j] : R(0); }
  __device__ void set_phi(int t, int i, int j, R v) const {
    if (i < n && j < n) {
      srow(t + 1, i)[j] = v;      // S(t+1, t) = Phi_t
      srow(t, j)[2 * n + i] = v;  // S(t, t+1) = Phi_t^T
    }
  }
  __device__ R get_phi(int t, int i, int j) const { return (i < n && j < n) ? srow(t + 1, i)[j] : R(0); }
  __device__ void set_ntinv(int t, int i, int j, R v) const {
    if (i < n && j < n) {
      prow(t, i)[n + j] = v;
      prow(t, j)[n + i] = v;
    }
  }
  __device__ R get_ntinv(int t, int i, int j) const { return (i < n && j < n) ? prow(t, i)[n + j] : R(0); }
  __device__ void set_m(int t, int i, int j, R v) const {
    if (i < n && j < n) {
      prow(t + 1, i)[j] = v;
      prow(t, j)[2 * n + i] = v;
    }
  }
  // Zero the boundary blocks S(0, -1), S(N, N+1) (and Phiinv's).
  __device__ void init() const {
    const int N = T - 1;
    for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
      const int i = e / n, j = e - i * n;
      srow(0, i)[j] = R(0);
      prow(0, i)[j] = R(0);
      srow(N, i)[2 * n + j] = R(0);
      prow(N, i)[2 * n + j] = R(0);
    }
  }
};

// Phase 1: Theta (upper) and Phi of every stage.
template <int NB, typename R, class Acc>
__device__ void assemble_theta_phi(const Acc& acc, const QPView<R>& qp, R rho_f, R rho_i, R sigma, int T, int n,
                                   int nx, int n0, int m) {
  constexpr int TRI = tri_size(NB);
  const int N = T - 1;
  for (int e = threadIdx.x; e < T * TRI; e += blockDim.x) {
    const int t = e / TRI, idx = e - t * TRI;
    const int i = tri_row(idx, NB), j = tri_col(idx, NB);
    R val = R(0);
    if (i < n && j < n) {
      val = qp.D[((size_t)t * n + i) * n + j];
      if (i == j) val += sigma;
      R gtg = R(0);
      for (int k = 0; k < m; ++k) gtg += qp.G[((size_t)t * m + k) * n + i] * qp.G[((size_t)t * m + k) * n + j];
      val += rho_i * gtg;
      R ata = R(0);
      if (t == 0) {
        for (int k = 0; k < n0; ++k) ata += qp.A0[k * n + i] * qp.A0[k * n + j];
        if (N > 0)
          for (int k = 0; k < nx; ++k) ata += qp.Am[k * n + i] * qp.Am[k * n + j];
      } else {
        const R* ap = qp.Ap + (size_t)(t - 1) * nx * n;
        for (int k = 0; k < nx; ++k) ata += ap[k * n + i] * ap[k * n + j];
        if (t < N) {
          const R* am = qp.Am + (size_t)t * nx * n;
          for (int k = 0; k < nx; ++k) ata += am[k * n + i] * am[k * n + j];
        }
      }
      val += rho_f * ata;
    }
    acc.set_theta(t, i, j, val);
  }
  for (int e = threadIdx.x; e < N * NB * NB; e += blockDim.x) {
    const int t = e / (NB * NB), ij = e - t * NB * NB;
    const int i = ij / NB, j = ij - i * NB;
    R val = R(0);
    if (i < n && j < n) {
      val = qp.E[((size_t)t * n + i) * n + j];
      const R* ap = qp.Ap + (size_t)t * nx * n;
      const R* am = qp.Am + (size_t)t * nx * n;
      R s = R(0);
      for (int k = 0; k < nx; ++k) s += ap[k * n + i] * am[k * n + j];
      val += rho_f * s;
    }
    acc.set_phi(t, i, j, val);
  }
}

// Phase 2: one warp inverts Theta_t for t = t0 + warp, t0 + warp + nwarps,
// ... < t1 and stores -Theta_t^-1.  Sets *flag when a pivot is zero or not
// finite.
template <int NB, typename R, class Acc>
__device__ void invert_thetas(const Acc& acc, int T, int n, int* flag, int t0 = 0, int t1 = -1) {
  constexpr int CPL = (2 * NB + 31) / 32;  // augmented columns per lane
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  if (t1 < 0) t1 = T;
  for (int t = t0 + wid; t < t1; t += nw) {
    R a[CPL][NB];
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = lane + 32 * k;
#pragma unroll
      for (int r = 0; r < NB; ++r) {
        R v = R(0);
        if (c < NB) {
          if (r < n && c < n) v = r <= c ? acc.get_theta(t, r, c) : acc.get_theta(t, c, r);
        } else if (c < 2 * NB) {
          v = (r == c - NB && r < n) ? R(1) : R(0);
        }
        a[k][r] = v;
      }
    }
    bool bad = false;
#pragma unroll
    for (int col = 0; col < NB; ++col) {
      if (col < n) {
        // Broadcast the pivot column (slot 0 of lane `col`).
        R pv[NB];
#pragma unroll
        for (int r = 0; r < NB; ++r) pv[r] = __shfl_sync(0xffffffffu, a[0][r], col);
        int p = col;
        R best = fabs(pv[col]);
#pragma unroll
        for (int r = col + 1; r < NB; ++r) {
          if (r < n && fabs(pv[r]) > best) {
            best = fabs(pv[r]);
            p = r;
          }
        }
        // Swap rows col <-> p (select chains; p is warp-uniform).
        R pvp = pv[col];
#pragma unroll
        for (int r = col + 1; r < NB; ++r) pvp = (r == p) ? pv[r] : pvp;
#pragma unroll
        for (int r = col + 1; r < NB; ++r) pv[r] = (r == p) ? pv[col] : pv[r];
        pv[col] = pvp;
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          R ap = a[k][col];
#pragma unroll
          for (int r = col + 1; r < NB; ++r) ap = (r == p) ? a[k][r] : ap;
#pragma unroll
          for (int r = col + 1; r < NB; ++r) a[k][r] = (r == p) ? a[k][col] : a[k][r];
          a[k][col] = ap;
        }
        const R piv = pv[col];
        if (!(fabs(piv) > R(0)) || !isfinite(piv)) bad = true;
        const R inv = R(1) / piv;
#pragma unroll
        for (int k = 0; k < CPL; ++k) {
          a[k][col] *= inv;
#pragma unroll
          for (int r = 0; r < NB; ++r)
            if (r != col) a[k][r] -= pv[r] * a[k][col];
        }
      }
    }
    // Lane NB + j holds column j of the inverse; store its upper part negated.
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = lane + 32 * k - NB;
      if (c >= 0 && c < NB) {
#pragma unroll
        for (int r = 0; r < NB; ++r)
          if (r <= c) acc.set_ntinv(t, r, c, -a[k][r]);
      }
    }
    if (bad && lane == 0) atomicOr(flag, TMPC_STATUS_SINGULAR_BLOCK);
  }
}

// Phase 3: M_t = Theta_{t+1}^-1 Phi_t Theta_t^-1, one thread per (t, row i):
//   V = Theta_{t+1}^-1[i, :] Phi_t ;  M[i, :] = V Theta_t^-1.
template <int NB, typename R, class Acc>
__device__ void assemble_precond_offdiag(const Acc& acc, int T) {
  const int N = T - 1;
  for (int e = threadIdx.x; e < N * NB; e += blockDim.x) {
    const int t = e / NB, i = e - t * NB;
    R v[NB];
#pragma unroll
    for (int l = 0; l < NB; ++l) v[l] = R(0);
#pragma unroll 1
    for (int k = 0; k < NB; ++k) {
      const R w = acc.get_ntinv(t + 1, i, k);
#pragma unroll
      for (int l = 0; l < NB; ++l) v[l] += w * acc.get_phi(t, k, l);
    }
#pragma unroll 1
    for (int j = 0; j < NB; ++j) {
      R s = R(0);
#pragma unroll
      for (int l = 0; l < NB; ++l) s += v[l] * acc.get_ntinv(t, l, j);
      acc.set_m(t, i, j, s);  // (-A)(-B) = AB: the two negations cancel
    }
  }
}

// Full assembly; all threads of the CTA must call it.  Ends with a barrier.
template <int NB, typename R, class Acc>
__device__ __noinline__ void assemble_ops(const Acc& acc, const QPView<R>& qp, R rho_f, R rho_i, R sigma, int T, int n, int nx,
                             int n0, int m, int* flag) {
  acc.init();
  assemble_theta_phi<NB>(acc, qp, rho_f, rho_i, sigma, T, n, nx, n0, m);
  __syncthreads();
  invert_thetas<NB, R>(acc, T, n, flag);
  __syncthreads();
  assemble_precond_offdiag<NB, R>(acc, T);
  __syncthreads();
}

}  // namespace tmpc
