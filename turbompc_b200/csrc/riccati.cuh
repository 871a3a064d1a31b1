// Block-tridiagonal Cholesky (block Riccati recursion) of the symmetric
// positive definite Schur matrix S = blocktridiag(Phi_{t-1}, Theta_t, Phi_t^T),
// written from scratch as the direct replacement of the reference's cuDSS
// solve (turbompc/solvers/linear_systems_solvers/csrc/cudss_blktridi.cu,
// admm/csrc/admm_cudss.cu):
//
//   L_0 L_0^T = Theta_0
//   W_{t-1}   = Phi_{t-1} L_{t-1}^-T          (so S = L L^T with block-bidiagonal L)
//   L_t L_t^T = Theta_t - W_{t-1} W_{t-1}^T
//
//   solve S x = b:  y_t = L_t^-1 (b_t - W_{t-1} y_{t-1})        t = 0..N
//                   x_t = L_t^-T (y_t - W_t^T x_{t+1})          t = N..0
//
// One warp per problem.  The factor uses the packed operator layout
// (tmpc_common.cuh): diagonal slot t holds L_t^T as a packed upper triangle
// (entry (a, b), a <= b, is L_t[b][a]); sub-diagonal slot t holds W_t
// row-major.  NB padding is handled by an identity diagonal in the padded
// rows, which keeps the padded solution components exactly zero.
#pragma once

#include "tmpc_common.cuh"

namespace tmpc {

template <int NB, typename R>
struct FactorView {
  R* base;  // one problem's factor
  int T;
  using Gm = Geo<NB, R>;
  __device__ R* lt(int t) const { return base + (size_t)t * Gm::DSTR; }
  __device__ R* w(int t) const { return base + (size_t)T * Gm::DSTR + (size_t)t * Gm::OSTR; }
};

// Per-warp shared scratch of riccati_factor_warp (elements): the working
// block M (NB x (NB+1)) and a copy of the previous W (NB x NB).
template <int NB>
__host__ __device__ constexpr int riccati_scratch_elems() {
  return NB * (NB + 1) + NB * NB;
}

// Factor one problem in place.  On entry slot t holds Theta_t (packed upper,
// as written by assemble_theta_phi) and sub-diagonal slot t holds Phi_t; on
// exit they hold L_t^T and W_t.  M is per-warp shared scratch of
// riccati_scratch_elems<NB>() elements (W_{t-1} is kept there for the Schur
// update, so it is not re-read from global memory).  Called by all 32 lanes
// of one warp; returns false (all lanes) when a pivot is not positive and
// finite.
template <int NB, typename R>
__device__ bool riccati_factor_warp(const FactorView<NB, R>& F, R* M, int n) {
  constexpr int LD = NB + 1;
  const int lane = threadIdx.x & 31;
  const int T = F.T;
  R* Wsh = M + NB * LD;  // W_{t-1}, row-major
  bool ok = true;
  for (int t = 0; t < T; ++t) {
    const R* th = F.lt(t);
    for (int e = lane; e < NB * NB; e += 32) {
      const int r = e / NB, c = e - r * NB;
      R v;
      if (r < n && c < n) {
        v = r <= c ? th[tri_index(r, c, NB)] : th[tri_index(c, r, NB)];
        if (t > 0) {
          R s = R(0);
#pragma unroll 8
          for (int k = 0; k < NB; ++k) s = fma(Wsh[r * NB + k], Wsh[c * NB + k], s);
          v -= s;
        }
      } else {
        v = (r == c) ? R(1) : R(0);
      }
      M[r * LD + c] = v;
    }
    __syncwarp();
    // Right-looking Cholesky on the lower triangle of M.
    for (int k = 0; k < NB; ++k) {
      const R d = M[k * LD + k];
      if (!(d > R(0)) || !isfinite(d)) ok = false;
      const R s = sqrt(d);
      __syncwarp();
      for (int r = k + 1 + lane; r < NB; r += 32) M[r * LD + k] /= s;
      if (lane == 0) M[k * LD + k] = s;
      __syncwarp();
      const int m = NB - 1 - k;  // trailing size
      for (int e = lane; e < m * m; e += 32) {
        const int r = k + 1 + e / m, c = k + 1 + e % m;
        if (c <= r) M[r * LD + c] -= M[r * LD + k] * M[c * LD + k];
      }
      __syncwarp();
    }
    // Store L_t^T packed (entry (a, b), a <= b, is L[b][a]).
    R* lt = F.lt(t);
    for (int e = lane; e < NB * NB; e += 32) {
      const int b = e / NB, a = e - b * NB;
      if (a <= b) lt[tri_index(a, b, NB)] = M[b * LD + a];
    }
    // W_t = Phi_t L_t^-T: lane i solves L w = Phi_t[i, :]^T by forward substitution.
    if (t < T - 1) {
      R* W = F.w(t);
      if (lane < NB) {
        R wv[NB];
#pragma unroll
        for (int k = 0; k < NB; ++k) wv[k] = W[lane * NB + k];
#pragma unroll
        for (int k = 0; k < NB; ++k) {
          R s = wv[k];
#pragma unroll
          for (int m2 = 0; m2 < k; ++m2) s -= M[k * LD + m2] * wv[m2];
          wv[k] = s / M[k * LD + k];
        }
#pragma unroll
        for (int k = 0; k < NB; ++k) {
          W[lane * NB + k] = wv[k];
          Wsh[lane * NB + k] = wv[k];
        }
      }
    }
    __syncwarp();
  }
  return __all_sync(0xffffffffu, ok);
}

// Solve S x = b with the factor; b, x, y are this problem's [T][VSTR] vectors
// (shared or global, padded entries of b must be zero).  All 32 lanes.
template <int NB, typename R>
__device__ void riccati_solve_warp(const FactorView<NB, R>& F, const R* b, R* y, R* x) {
  using Gm = Geo<NB, R>;
  const int lane = threadIdx.x & 31;
  const int T = F.T;
  const bool act = lane < NB;
  const int li = act ? lane : 0;
  // forward: y_t = L_t^-1 (b_t - W_{t-1} y_{t-1})
  for (int t = 0; t < T; ++t) {
    R u = act ? b[t * Gm::VSTR + li] : R(0);
    if (t > 0) {
      const R* W = F.w(t - 1) + li * NB;
      const R* yp = y + (t - 1) * Gm::VSTR;
      R s = R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) s = fma(W[k], yp[k], s);
      u -= s;
    }
    const R* lt = F.lt(t);
    R lcol[NB];  // L[li][k] = L^T packed (k, li) for k <= li
#pragma unroll
    for (int k = 0; k < NB; ++k) lcol[k] = (k <= li) ? lt[tri_index(k, li, NB)] : R(0);
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const R yk = __shfl_sync(0xffffffffu, u / lcol[k], k);  // valid in lane k: lcol[k] = L[k][k]
      if (li > k) u = fma(-lcol[k], yk, u);
      if (li == k) u = yk;
    }
    if (act) y[t * Gm::VSTR + li] = u;
    __syncwarp();
  }
  // backward: x_t = L_t^-T (y_t - W_t^T x_{t+1})
  for (int t = T - 1; t >= 0; --t) {
    R u = act ? y[t * Gm::VSTR + li] : R(0);
    if (t < T - 1) {
      const R* W = F.w(t);
      const R* xn = x + (t + 1) * Gm::VSTR;
      R s = R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) s = fma(W[k * NB + li], xn[k], s);
      u -= s;
    }
    const R* lt = F.lt(t);
    R lrow[NB];  // L^T[li][k] = L[k][li] = packed (li, k) for k >= li
#pragma unroll
    for (int k = 0; k < NB; ++k) lrow[k] = (k >= li) ? lt[tri_index(li, k, NB)] : R(0);
#pragma unroll
    for (int k = NB - 1; k >= 0; --k) {
      const R xk = __shfl_sync(0xffffffffu, u / lrow[k], k);  // lane k: lrow[k] = L[k][k]
      if (li < k) u = fma(-lrow[k], xk, u);
      if (li == k) u = xk;
    }
    if (act) x[t * Gm::VSTR + li] = u;
    __syncwarp();
  }
}

}  // namespace tmpc
