// Block-tridiagonal matvec and PCG on packed operators, one CTA per problem.
//
// Matvec y = M v for a symmetric block-tridiagonal M in packed form
// (diagonal blocks Dg_t, sub-diagonal blocks L_t = M(t+1, t)):
//     y_t = L_{t-1} v_{t-1} + Dg_t v_t + L_t^T v_{t+1}
// is split into T + 2N independent tasks, one thread each:
//   diag task t          d[t]      = Dg_t v_t       (each packed entry used twice)
//   half task (t, h)     lo[t+1]  |= L_t[rows_h] v_t
//                        up_h[t]   = L_t[rows_h]^T v_{t+1}[rows_h]
// A task reads its whole block once with 128-bit loads and keeps the
// partial results in registers, so every stored entry is read once per
// matvec and feeds two FMAs.  y = d + lo + up0 + up1 after a barrier.
//
// The PCG recurrences and the stopping rule follow
// turbompc/solvers/admm/csrc/admm_fused.cu:54-161 (the fused kernel's PCG):
//   r = g - S x ; z = Phiinv r ; p = z ; eta = r.z ; eta0 = |eta|
//   for k < max_iter:  stop if |eta| < 1e-12 + eps*eta0
//     Sp = S p ; a = eta / max_abs(p.Sp, 1e-30) ; x += a p ; r -= a Sp
//     z = Phiinv r ; eta' = r.z ; beta = eta'/eta ; p = z + beta p
#pragma once

#include "tmpc_common.cuh"

namespace tmpc {

template <int NB, typename R>
struct BlockVecs {
  R* x;
  R* r;
  R* z;
  R* p;
  R* d;
  R* lo;
  R* up0;
  R* up1;
};

template <int NB, bool OPS_SMEM, typename R>
__device__ __forceinline__ void diag_task(const R* __restrict__ blk, const R* __restrict__ v, R* __restrict__ out) {
  using Gm = Geo<NB, R>;
  constexpr int VEC = Gm::VEC;
  R vv[NB], acc[NB], w[VEC];
#pragma unroll
  for (int c = 0; c < NB / VEC; ++c) ld128(&vv[c * VEC], v + c * VEC);
#pragma unroll
  for (int i = 0; i < NB; ++i) acc[i] = R(0);
  // Walk the packed upper triangle in storage order; a new 128-bit chunk is
  // loaded whenever the packed index crosses a chunk boundary.
#pragma unroll
  for (int i = 0; i < NB; ++i) {
#pragma unroll
    for (int j = i; j < NB; ++j) {
      const int idx = i * NB - (i * (i - 1)) / 2 + (j - i);
      if (idx % VEC == 0) ldop<OPS_SMEM>(w, blk + idx);
      const R a = w[idx % VEC];
      acc[i] = fma(a, vv[j], acc[i]);
      if (i != j) acc[j] = fma(a, vv[i], acc[j]);
    }
  }
#pragma unroll
  for (int c = 0; c < NB / VEC; ++c) st128(out + c * VEC, &acc[c * VEC]);
}

// Half h of sub-diagonal block L_t: rows [h*NB/2, (h+1)*NB/2).
template <int NB, bool OPS_SMEM, typename R>
__device__ __forceinline__ void half_task(const R* __restrict__ blk, const R* __restrict__ vt,
                                          const R* __restrict__ vt1, R* __restrict__ lo_out,
                                          R* __restrict__ up_out, int h) {
  using Gm = Geo<NB, R>;
  constexpr int VEC = Gm::VEC;
  constexpr int HR = NB / 2;
  R a[NB], b[HR], up[NB];
#pragma unroll
  for (int c = 0; c < NB / VEC; ++c) ld128(&a[c * VEC], vt + c * VEC);
  const int r0 = h * HR;
  if constexpr (HR % VEC == 0) {
#pragma unroll
    for (int c = 0; c < HR / VEC; ++c) ld128(&b[c * VEC], vt1 + r0 + c * VEC);
  } else {
#pragma unroll
    for (int k = 0; k < HR; ++k) b[k] = vt1[r0 + k];
  }
#pragma unroll
  for (int j = 0; j < NB; ++j) up[j] = R(0);
  const R* base = blk + (size_t)r0 * NB;
  R lo[HR];
#pragma unroll
  for (int i = 0; i < HR; ++i) {
    R s = R(0);
#pragma unroll
    for (int c = 0; c < NB / VEC; ++c) {
      R w[VEC];
      ldop<OPS_SMEM>(w, base + i * NB + c * VEC);
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        s = fma(w[e], a[c * VEC + e], s);
        up[c * VEC + e] = fma(w[e], b[i], up[c * VEC + e]);
      }
    }
    lo[i] = s;
  }
  if constexpr (HR % VEC == 0) {
#pragma unroll
    for (int c = 0; c < HR / VEC; ++c) st128(lo_out + r0 + c * VEC, &lo[c * VEC]);
  } else {
#pragma unroll
    for (int k = 0; k < HR; ++k) lo_out[r0 + k] = lo[k];
  }
#pragma unroll
  for (int c = 0; c < NB / VEC; ++c) st128(up_out + c * VEC, &up[c * VEC]);
}

// Partial results of y = M v; caller syncs before reading d/lo/up0/up1.
// lo[0], up0[N], up1[N] are never written and must hold zeros.
template <int NB, bool OPS_SMEM, typename R>
__device__ __forceinline__ void matvec_partials(const R* op, int T, const R* v, R* d, R* lo, R* up0, R* up1) {
  using Gm = Geo<NB, R>;
  const int N = T - 1;
  const R* Dg = op;
  const R* L = op + (size_t)T * Gm::DSTR;
  const int ntask = T + 2 * N;
  for (int task = threadIdx.x; task < ntask; task += blockDim.x) {
    if (task < T) {
      diag_task<NB, OPS_SMEM>(Dg + (size_t)task * Gm::DSTR, v + task * Gm::VSTR, d + task * Gm::VSTR);
    } else {
      const int k = task - T;
      const int h = k >= N ? 1 : 0;
      const int t = k - h * N;
      half_task<NB, OPS_SMEM>(L + (size_t)t * Gm::OSTR, v + t * Gm::VSTR, v + (t + 1) * Gm::VSTR,
                              lo + (t + 1) * Gm::VSTR, (h ? up1 : up0) + t * Gm::VSTR, h);
    }
  }
}

// Elementwise loop over the T*NB padded entries of a block vector: e is the
// dense index, off the on-chip offset t*VSTR + j.
#define TMPC_FOR_ENTRIES(e, off, T, NB, VSTR)                                                       \
  for (int e = threadIdx.x, off = 0; e < (T) * (NB) && ((off = (e / (NB)) * (VSTR) + e % (NB)), true); \
       e += blockDim.x)

// PCG on packed operators with all vectors on chip.  x (in: guess, out:
// solution) and g (rhs) are [T][VSTR] block vectors.  Returns the iteration
// count (identical in all threads).
template <int NB, bool OPS_SMEM, typename R>
__device__ int pcg_solve(const R* opS, const R* opP, int T, const R* g, const BlockVecs<NB, R>& w, R* red,
                         int max_iter, R eps) {
  using Gm = Geo<NB, R>;
  matvec_partials<NB, OPS_SMEM>(opS, T, w.x, w.d, w.lo, w.up0, w.up1);
  __syncthreads();
  TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) { w.r[o] = g[o] - (w.d[o] + w.lo[o] + w.up0[o] + w.up1[o]); }
  __syncthreads();
  matvec_partials<NB, OPS_SMEM>(opP, T, w.r, w.d, w.lo, w.up0, w.up1);
  __syncthreads();
  R part = R(0);
  TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) {
    const R zz = w.d[o] + w.lo[o] + w.up0[o] + w.up1[o];
    w.z[o] = zz;
    w.p[o] = zz;
    part = fma(w.r[o], zz, part);
  }
  R eta = block_sum(part, red);
  const R eta0 = fabs(eta);
  int it = 0;
  for (; it < max_iter; ++it) {
    if (fabs(eta) < R(1e-12) + eps * eta0) break;
    __syncthreads();  // p complete; reduction slots free
    matvec_partials<NB, OPS_SMEM>(opS, T, w.p, w.d, w.lo, w.up0, w.up1);
    __syncthreads();
    part = R(0);
    TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) {
      const R sp = w.d[o] + w.lo[o] + w.up0[o] + w.up1[o];
      w.d[o] = sp;
      part = fma(w.p[o], sp, part);
    }
    R den = block_sum(part, red + 32);
    if (fabs(den) < R(1e-30)) den = R(1e-30);
    const R alpha = eta / den;
    TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) {
      w.x[o] = fma(alpha, w.p[o], w.x[o]);
      w.r[o] = fma(-alpha, w.d[o], w.r[o]);
    }
    __syncthreads();
    matvec_partials<NB, OPS_SMEM>(opP, T, w.r, w.d, w.lo, w.up0, w.up1);
    __syncthreads();
    part = R(0);
    TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) {
      const R zz = w.d[o] + w.lo[o] + w.up0[o] + w.up1[o];
      w.z[o] = zz;
      part = fma(w.r[o], zz, part);
    }
    const R eta_new = block_sum(part, red);
    const R beta = eta_new / eta;
    eta = eta_new;
    TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) { w.p[o] = fma(beta, w.p[o], w.z[o]); }
  }
  __syncthreads();
  return it;
}

}  // namespace tmpc
