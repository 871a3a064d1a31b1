// Block-tridiagonal matvec and PCG on packed operators, one CTA per problem.
//
// Matvec y = M v for a symmetric block-tridiagonal M in packed form
// (diagonal blocks Dg_t, sub-diagonal blocks L_t = M(t+1, t)):
//     y_t = L_{t-1} v_{t-1} + Dg_t v_t + L_t^T v_{t+1}
// is split into T + 4N independent tasks, one thread each:
//   diag task t           d[t]      = Dg_t v_t       (each packed entry used twice)
//   quarter task (t, q)   lo[t+1]  |= L_t[rows_q] v_t
//                         up_q[t]   = L_t[rows_q]^T v_{t+1}[rows_q]
// A task reads its part of the block once with 128-bit loads and keeps the
// partial results in registers, so every stored entry is read once per
// matvec and feeds two FMAs.  y = d + lo + up0 + up1 + up2 + up3 after a
// barrier (fixed summation order: deterministic).
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

// On-chip block vectors (each T*VSTR elements) of one problem.  The four
// partial buffers up0..up3 are contiguous and selected by pointer arithmetic:
// indexing an array of pointers with a runtime index would force the struct
// into local memory.
template <int NB, typename R>
struct BlockVecs {
  R* x;
  R* r;
  R* z;
  R* p;
  R* d;
  R* lo;
  R* up0;  // up_q = up0 + q * vs
  int vs;
  __device__ R* up(int q) const { return up0 + q * vs; }
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

// Quarter h of sub-diagonal block L_t: rows [h*NB/4, (h+1)*NB/4).
template <int NB, bool OPS_SMEM, typename R>
__device__ __forceinline__ void quarter_task(const R* __restrict__ blk, const R* __restrict__ vt,
                                          const R* __restrict__ vt1, R* __restrict__ lo_out,
                                          R* __restrict__ up_out, int h) {
  using Gm = Geo<NB, R>;
  constexpr int VEC = Gm::VEC;
  constexpr int HR = NB / 4;
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

// Partial results of y = M v; caller syncs before reading d/lo/up[].
// lo[0] and up[q][N] are never written and must hold zeros.
template <int NB, bool OPS_SMEM, typename R>
__device__ __forceinline__ void matvec_partials(const R* op, int T, const R* v, const BlockVecs<NB, R>& w) {
  using Gm = Geo<NB, R>;
  const int N = T - 1;
  const R* Dg = op;
  const R* L = op + (size_t)T * Gm::DSTR;
  const int ntask = T + 4 * N;
  for (int task = threadIdx.x; task < ntask; task += blockDim.x) {
    if (task < T) {
      diag_task<NB, OPS_SMEM>(Dg + (size_t)task * Gm::DSTR, v + task * Gm::VSTR, w.d + task * Gm::VSTR);
    } else {
      const int k = task - T;
      const int q = k / N;  // consecutive threads take consecutive blocks of the same quarter
      const int t = k - q * N;
      quarter_task<NB, OPS_SMEM>(L + (size_t)t * Gm::OSTR, v + t * Gm::VSTR, v + (t + 1) * Gm::VSTR,
                                 w.lo + (t + 1) * Gm::VSTR, w.up(q) + t * Gm::VSTR, q);
    }
  }
}

// y = d + lo + up0 + up1 + up2 + up3 for the VEC entries at offset o.
template <int NB, typename R>
__device__ __forceinline__ void gather_y(R* y, const BlockVecs<NB, R>& w, int o) {
  constexpr int VEC = Geo<NB, R>::VEC;
  R a[VEC], b[VEC];
  ld128(y, w.d + o);
  ld128(a, w.lo + o);
#pragma unroll
  for (int k = 0; k < VEC; ++k) y[k] += a[k];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    ld128(b, w.up(q) + o);
#pragma unroll
    for (int k = 0; k < VEC; ++k) y[k] += b[k];
  }
}

// Vectorised elementwise loop over the T*NB padded entries of a block
// vector: each iteration handles VEC consecutive entries at on-chip offset
// `off` (16-byte aligned).
#define TMPC_FOR_CHUNKS(off, T, NB, VSTR, VEC)                                                            \
  for (int c_ = threadIdx.x, off = 0;                                                                    \
       c_ < (T) * ((NB) / (VEC)) && ((off = (c_ / ((NB) / (VEC))) * (VSTR) + (c_ % ((NB) / (VEC))) * (VEC)), true); \
       c_ += blockDim.x)

// Scalar elementwise loop (e: dense index t*NB + j, off: on-chip offset).
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
  constexpr int VEC = Gm::VEC;
  matvec_partials<NB, OPS_SMEM>(opS, T, w.x, w);
  __syncthreads();
  TMPC_FOR_CHUNKS(o, T, NB, Gm::VSTR, VEC) {
    R y[VEC], gg[VEC];
    gather_y<NB>(y, w, o);
    ld128(gg, g + o);
#pragma unroll
    for (int k = 0; k < VEC; ++k) y[k] = gg[k] - y[k];
    st128(w.r + o, y);
  }
  __syncthreads();
  matvec_partials<NB, OPS_SMEM>(opP, T, w.r, w);
  __syncthreads();
  R part = R(0);
  TMPC_FOR_CHUNKS(o, T, NB, Gm::VSTR, VEC) {
    R zz[VEC], rr[VEC];
    gather_y<NB>(zz, w, o);
    ld128(rr, w.r + o);
    st128(w.z + o, zz);
    st128(w.p + o, zz);
#pragma unroll
    for (int k = 0; k < VEC; ++k) part = fma(rr[k], zz[k], part);
  }
  R eta = block_sum(part, red);
  const R eta0 = fabs(eta);
  int it = 0;
  for (; it < max_iter; ++it) {
    if (fabs(eta) < R(1e-12) + eps * eta0) break;
    __syncthreads();  // p complete; reduction slots free
    matvec_partials<NB, OPS_SMEM>(opS, T, w.p, w);
    __syncthreads();
    part = R(0);
    TMPC_FOR_CHUNKS(o, T, NB, Gm::VSTR, VEC) {
      R sp[VEC], pp[VEC];
      gather_y<NB>(sp, w, o);
      ld128(pp, w.p + o);
      st128(w.d + o, sp);
#pragma unroll
      for (int k = 0; k < VEC; ++k) part = fma(pp[k], sp[k], part);
    }
    R den = block_sum(part, red + 32);
    if (fabs(den) < R(1e-30)) den = R(1e-30);
    const R alpha = eta / den;
    TMPC_FOR_CHUNKS(o, T, NB, Gm::VSTR, VEC) {
      R sp[VEC], pp[VEC], xx[VEC], rr[VEC];
      ld128(sp, w.d + o);
      ld128(pp, w.p + o);
      ld128(xx, w.x + o);
      ld128(rr, w.r + o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) {
        xx[k] = fma(alpha, pp[k], xx[k]);
        rr[k] = fma(-alpha, sp[k], rr[k]);
      }
      st128(w.x + o, xx);
      st128(w.r + o, rr);
    }
    __syncthreads();
    matvec_partials<NB, OPS_SMEM>(opP, T, w.r, w);
    __syncthreads();
    part = R(0);
    TMPC_FOR_CHUNKS(o, T, NB, Gm::VSTR, VEC) {
      R zz[VEC], rr[VEC];
      gather_y<NB>(zz, w, o);
      ld128(rr, w.r + o);
      st128(w.z + o, zz);
#pragma unroll
      for (int k = 0; k < VEC; ++k) part = fma(rr[k], zz[k], part);
    }
    const R eta_new = block_sum(part, red);
    const R beta = eta_new / eta;
    eta = eta_new;
    TMPC_FOR_CHUNKS(o, T, NB, Gm::VSTR, VEC) {
      R zz[VEC], pp[VEC];
      ld128(zz, w.z + o);
      ld128(pp, w.p + o);
#pragma unroll
      for (int k = 0; k < VEC; ++k) pp[k] = fma(beta, pp[k], zz[k]);
      st128(w.p + o, pp);
    }
  }
  __syncthreads();
  return it;
}

}  // namespace tmpc
