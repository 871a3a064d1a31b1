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

// Where the factor reads Theta_t and Phi_t (indices inside the n x n blocks).
//   PackedSrc: the factor's own slots (Theta_t packed upper in slot t, Phi_t in
//              sub-diagonal slot t), as written by assemble_theta_phi.
//   RefSrc:    the reference-layout S [T][n][3n] directly (no copy-in pass):
//              Theta_t[r][j] = S[t][r][n + j], Phi_t[i][k] = S[t+1][i][k].
template <int NB, typename R>
struct PackedSrc {
  FactorView<NB, R> F;
  __device__ R theta(int t, int r, int j) const {
    const R* th = F.lt(t);
    return r <= j ? th[tri_index(r, j, NB)] : th[tri_index(j, r, NB)];
  }
  __device__ R phi(int t, int i, int k) const { return F.w(t)[i * NB + k]; }
};
template <typename R>
struct RefSrc {
  const R* S;
  int n;
  __device__ R theta(int t, int r, int j) const { return __ldg(S + ((size_t)t * n + r) * 3 * n + n + j); }
  __device__ R phi(int t, int i, int k) const { return __ldg(S + ((size_t)(t + 1) * n + i) * 3 * n + k); }
};

// Per-warp shared scratch of riccati_factor_warp (elements): W_{t-1}
// (row-major) and L_t (column-major), NB x NB each.
template <int NB>
__host__ __device__ constexpr int riccati_scratch_elems() {
  return 2 * NB * NB;
}

// Factor one problem.  Theta_t and Phi_t come from `src` (the factor's own
// slots, filled by assemble_theta_phi, or the reference-layout S); on exit
// diagonal slot t holds L_t^T and sub-diagonal slot t holds W_t.  M is per-warp shared scratch of
// riccati_scratch_elems<NB>() elements, 16-byte aligned.  Called by all 32
// lanes of one warp; returns false (all lanes) when a pivot is not positive
// and finite.
//
// Lane j keeps column j of the stage's working matrix in registers:
//   M_t = Theta_t - W_{t-1} W_{t-1}^T     (rows of W_{t-1} broadcast from shared memory)
//   right-looking Cholesky: at step k lane k scales its column and publishes
//   it (column k of L_t) in shared memory; lanes j > k update their columns
//   W_t = Phi_t L_t^-T: lane i runs the forward substitution L w = Phi_t[i, :]^T
//   column by column (column m of L broadcast from shared memory).
//
// G = 32: the whole warp works on one problem.  G = 16 (NB <= 16): each
// half-warp factors its own problem (two problems per warp; both halves run
// the same T and n, so they stay in step through the warp-wide __syncwarp);
// `store` = false runs a half without writing the factor (the spare half of
// the last warp).
template <int NB, typename R, class Src, int G = 32>
__device__ bool riccati_factor_warp(const FactorView<NB, R>& F, R* M, int n, const Src& src, bool store = true) {
  static_assert(NB % 4 == 0, "128-bit shared-memory broadcasts");
  static_assert(G == 32 || (G == 16 && NB <= 16), "half-warp groups need NB <= 16");
  constexpr int VEC = 16 / (int)sizeof(R);  // elements per 128-bit access
  const int lane = threadIdx.x & (G - 1);
  const int T = F.T;
  R* Wsh = M;            // W_{t-1}: Wsh[r * NB + k]
  R* Lsh = M + NB * NB;  // L_t:     Lsh[k * NB + r] = L[r][k]
  const bool act = lane < NB;
  const int j = act ? lane : 0;
  auto load_theta = [&](int t, R(&dst)[NB]) {
#pragma unroll
    for (int r = 0; r < NB; ++r) {
      R v = (r == j) ? R(1) : R(0);  // identity in the padded rows / columns
      if (r < n && j < n) v = src.theta(t, r, j);
      dst[r] = v;
    }
  };
  auto load_phi = [&](int t, R(&dst)[NB]) {
#pragma unroll
    for (int k = 0; k < NB; ++k) dst[k] = (act && j < n && k < n) ? src.phi(t, j, k) : R(0);
  };
  // Where Theta_{t+1} is loaded: right after stage t's stores (EARLY_THETA: early
  // issue) or at the top of stage t + 1.  Measured per block size (B200,
  // factor of reference-layout S): the early issue is 19 % faster for NB * w = 256
  // bytes and 7 % for 48 bytes, 4-20 % slower for 64-128 bytes.  (Issuing
  // Phi_t and Theta_{t+1} at the start of stage t, to overlap the Cholesky,
  // measured no faster at any size.)
  constexpr int BW = NB * (int)sizeof(R);
  constexpr bool EARLY_THETA = BW >= 256 || BW <= 48;
  bool ok = true;
  R a[NB];
  if constexpr (EARLY_THETA) load_theta(0, a);
  for (int t = 0; t < T; ++t) {
    if constexpr (!EARLY_THETA) load_theta(t, a);
    if (t > 0 && j < n) {
      R wj[NB];
#pragma unroll
      for (int k = 0; k < NB; k += VEC) ld128(&wj[k], Wsh + j * NB + k);
#pragma unroll
      for (int r = 0; r < NB; ++r) {
        R sacc = R(0);
#pragma unroll
        for (int k = 0; k < NB; k += VEC) {
          R wv[VEC];
          ld128(wv, Wsh + r * NB + k);
#pragma unroll
          for (int e = 0; e < VEC; ++e) sacc = fma(wv[e], wj[k + e], sacc);
        }
        if (r < n) a[r] -= sacc;
      }
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      if (lane == k) {
        const R d = a[k];
        if (!(d > R(0)) || !isfinite(d)) ok = false;
        const R sq = sqrt(d);
        const R inv = R(1) / sq;
        a[k] = sq;
#pragma unroll
        for (int r = k + 1; r < NB; ++r) a[r] *= inv;
#pragma unroll
        for (int r = 0; r < NB; r += VEC) {
          R cv[VEC];
#pragma unroll
          for (int e = 0; e < VEC; ++e) cv[e] = (r + e >= k) ? a[r + e] : R(0);
          st128(Lsh + k * NB + r, cv);
        }
      }
      __syncwarp();
      if (act && lane > k) {
        const R ljk = Lsh[k * NB + j];
#pragma unroll
        for (int r0 = ((k + 1) / VEC) * VEC; r0 < NB; r0 += VEC) {
          R lv[VEC];
          ld128(lv, Lsh + k * NB + r0);
#pragma unroll
          for (int e = 0; e < VEC; ++e) {
            const int r = r0 + e;
            if (r > k && r >= j) a[r] = fma(-lv[e], ljk, a[r]);
          }
        }
      }
    }
    __syncwarp();
    // Store L_t^T packed (entry (a, b), a <= b, is L[b][a] = Lsh[a * NB + b]).
    R* lt = F.lt(t);
    for (int e = lane; e < NB * NB; e += G) {
      const int bb = e / NB, aa = e - bb * NB;
      if (aa <= bb && store) lt[tri_index(aa, bb, NB)] = Lsh[aa * NB + bb];
    }
    // W_t = Phi_t L_t^-T, row i = lane.
    if (t < T - 1) {
      R* W = F.w(t);
      R x[NB];
      load_phi(t, x);
#pragma unroll
      for (int m = 0; m < NB; ++m) {
        x[m] = x[m] / Lsh[m * NB + m];
#pragma unroll
        for (int r0 = ((m + 1) / VEC) * VEC; r0 < NB; r0 += VEC) {
          R lv[VEC];
          ld128(lv, Lsh + m * NB + r0);
#pragma unroll
          for (int e = 0; e < VEC; ++e)
            if (r0 + e > m) x[r0 + e] = fma(-lv[e], x[m], x[r0 + e]);
        }
      }
      __syncwarp();  // every lane is done reading W_{t-1} in this stage
      if (act) {
#pragma unroll
        for (int k = 0; k < NB; k += VEC) {
          if (store) st128(W + j * NB + k, &x[k]);
          st128(Wsh + j * NB + k, &x[k]);
        }
      }
    }
    __syncwarp();
    if constexpr (EARLY_THETA) {
      if (t < T - 1) load_theta(t + 1, a);
    }
  }
  if constexpr (G == 32) {
    return __all_sync(0xffffffffu, ok);
  } else {
    const unsigned bad = __ballot_sync(0xffffffffu, !ok);
    return ((bad >> (threadIdx.x & 16)) & 0xffffu) == 0;  // this half's lanes only
  }
}

// Solve S x = b with the factor; b, x, y are this problem's [T][VSTR] vectors
// (shared or global, padded entries of b must be zero).  All 32 lanes.
// The factor blocks a stage needs (a row / column of W and of L) do not
// depend on the vectors, so with PF the next stage's blocks are loaded while
// the current stage's substitution runs (the substitution chain is
// sequential in t, and a warp-synchronous step would otherwise wait a full
// memory latency per stage).  PIPE = false keeps the register footprint of
// the unpipelined solve (for register-capped callers).
// G = 16 (NB <= 16): one problem per half-warp, as in riccati_factor_warp
// (shuffles stay inside the half; b, y, x are the half's own vectors).
template <int NB, typename R, bool PIPE = true, int G = 32>
__device__ void riccati_solve_warp(const FactorView<NB, R>& F, const R* b, R* y, R* x) {
  using Gm = Geo<NB, R>;
  static_assert(G == 32 || (G == 16 && NB <= 16), "half-warp groups need NB <= 16");
  constexpr bool PF = PIPE && NB * (int)sizeof(R) <= 128;
  const int lane = threadIdx.x & (G - 1);
  const int T = F.T;
  const bool act = lane < NB;
  const int li = act ? lane : 0;
  // forward stage t reads W_{t-1} row li and L_t row li (packed (k, li), k <= li)
  auto load_fwd = [&](int t, R(&w)[NB], R(&l)[NB], R& dv) {
    const R* W = F.w(t > 0 ? t - 1 : 0) + li * NB;
#pragma unroll
    for (int k = 0; k < NB; ++k) w[k] = t > 0 ? W[k] : R(0);
    const R* lt = F.lt(t);
#pragma unroll
    for (int k = 0; k < NB; ++k) l[k] = (k <= li) ? lt[tri_index(k, li, NB)] : R(0);
    dv = lt[tri_index(li, li, NB)];
  };
  // backward stage t reads W_t column li and L_t^T row li (packed (li, k), k >= li)
  auto load_bwd = [&](int t, R(&w)[NB], R(&l)[NB], R& dv) {
    const R* W = F.w(t < T - 1 ? t : 0);
#pragma unroll
    for (int k = 0; k < NB; ++k) w[k] = t < T - 1 ? W[k * NB + li] : R(0);
    const R* lt = F.lt(t);
#pragma unroll
    for (int k = 0; k < NB; ++k) l[k] = (k >= li) ? lt[tri_index(li, k, NB)] : R(0);
    dv = lt[tri_index(li, li, NB)];
  };
  R wv[NB], lv[NB], dv;
  // forward: y_t = L_t^-1 (b_t - W_{t-1} y_{t-1})
  load_fwd(0, wv, lv, dv);
  for (int t = 0; t < T; ++t) {
    R wn[NB], ln[NB], dn = R(1);
    if constexpr (PF) {
      if (t + 1 < T) load_fwd(t + 1, wn, ln, dn);
    }
    R u = act ? b[t * Gm::VSTR + li] : R(0);
    if (t > 0) {
      const R* yp = y + (t - 1) * Gm::VSTR;
      R s = R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) s = fma(wv[k], yp[k], s);
      u -= s;
    }
    const R dinv = R(1) / dv;  // 1 / L[li][li]
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const R yk = __shfl_sync(0xffffffffu, u * dinv, k, G);  // lane k's scaled value
      if (li > k) u = fma(-lv[k], yk, u);
      if (li == k) u = yk;
    }
    if (act) y[t * Gm::VSTR + li] = u;
    __syncwarp();
    if (t + 1 < T) {
      if constexpr (PF) {
#pragma unroll
        for (int k = 0; k < NB; ++k) {
          wv[k] = wn[k];
          lv[k] = ln[k];
        }
        dv = dn;
      } else {
        load_fwd(t + 1, wv, lv, dv);
      }
    }
  }
  // backward: x_t = L_t^-T (y_t - W_t^T x_{t+1})
  load_bwd(T - 1, wv, lv, dv);
  for (int t = T - 1; t >= 0; --t) {
    R wn[NB], ln[NB], dn = R(1);
    if constexpr (PF) {
      if (t > 0) load_bwd(t - 1, wn, ln, dn);
    }
    R u = act ? y[t * Gm::VSTR + li] : R(0);
    if (t < T - 1) {
      const R* xn = x + (t + 1) * Gm::VSTR;
      R s = R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) s = fma(wv[k], xn[k], s);
      u -= s;
    }
    const R dinv = R(1) / dv;
#pragma unroll
    for (int k = NB - 1; k >= 0; --k) {
      const R xk = __shfl_sync(0xffffffffu, u * dinv, k, G);  // lane k's scaled value
      if (li < k) u = fma(-lv[k], xk, u);
      if (li == k) u = xk;
    }
    if (act) x[t * Gm::VSTR + li] = u;
    __syncwarp();
    if (t > 0) {
      if constexpr (PF) {
#pragma unroll
        for (int k = 0; k < NB; ++k) {
          wv[k] = wn[k];
          lv[k] = ln[k];
        }
        dv = dn;
      } else {
        load_bwd(t - 1, wv, lv, dv);
      }
    }
  }
}

}  // namespace tmpc
