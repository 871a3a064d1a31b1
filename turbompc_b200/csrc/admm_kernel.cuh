// Fused ADMM solve: Schur/preconditioner assembly + the whole ADMM loop with
// the PCG linear solve, one CTA per problem, operators resident in shared
// memory when they fit (else in a caller workspace in HBM).
//
// Per ADMM iteration (order of turbompc/solvers/admm/csrc/admm_fused.cu:701-925):
//   gamma = sigma x - q + C^T(rho_f c - y_f) + G^T(rho z_g - y_g)   (admm.py:157-174)
//   x_old = x ; x = PCG(S, Phiinv, gamma, x)
//   Cx0, Cx, Gx on the pre-relaxation x                             (admm.py:884-887)
//   x = alpha x + (1 - alpha) x_old
//   z~ = alpha Gx + (1 - alpha) z_old + y_g / rho ; z = clamp(z~, l, u)  (+ slack form)
//   y_f0 += rho_f alpha (Cx0 - c0) ; y_fdyn += rho_f alpha (Cx - c)
//   y_g  += rho (alpha Gx + (1 - alpha) z_old - z)
//   every check_every: residuals, convergence, OSQP rho adaptation with an
//   on-chip rebuild of S and Phiinv.
#pragma once
#include "assemble.cuh"
#include "pcg_core.cuh"
#include "riccati.cuh"
#include "launchers.cuh"
#include "tmpc_common.cuh"

namespace tmpc {


// Element offsets inside the dynamic shared-memory arena.
template <int NB, typename R>
struct AdmmSmem {
  size_t opS, opP, vec0, yf0, yfd, zg, yg, xig, cx0, cx, gx, ct, gt, red, fm, nelem;
  __host__ __device__ AdmmSmem(int T, int nx, int n0, int m, bool ops_smem, int nvec = 12) {
    using Gm = Geo<NB, R>;
    const int N = T - 1;
    auto a4 = [](size_t v) { return (v + 3) & ~size_t(3); };  // 16-byte alignment for both precisions
    size_t o = 0;
    const size_t opn = Gm::op_elems(T);
    opS = o;
    if (ops_smem) o += opn;
    opP = o;
    if (ops_smem) o += opn;
    vec0 = o;
    o += (size_t)nvec * T * Gm::VSTR;  // PCG: x r z p d lo up0..3 gam xold; direct: x y gam xold
    yf0 = a4(o); o = yf0 + n0;
    yfd = a4(o); o = yfd + (size_t)N * nx;
    zg = a4(o); o = zg + (size_t)T * m;
    yg = a4(o); o = yg + (size_t)T * m;
    xig = a4(o); o = xig + (size_t)T * m;
    cx0 = a4(o); o = cx0 + n0;
    cx = a4(o); o = cx + (size_t)N * nx;
    gx = a4(o); o = gx + (size_t)T * m;
    ct = a4(o); o = ct + n0 + (size_t)N * nx;
    gt = a4(o); o = gt + (size_t)T * m;
    red = a4(o); o = red + kRedSize;
    fm = a4(o); o = fm + (nvec == 4 ? (size_t)riccati_scratch_elems<NB>() : 0);  // Cholesky scratch (direct)
    nelem = a4(o);
  }
};

// gamma_t[j] (padded to NB) from the on-chip duals; ct = rho_f c - y_f, gt = rho z - y_g.
template <int NB, typename R>
__device__ void compute_gamma(R* gam, const R* x, const QPView<R>& qp, const R* ct, const R* gt, R sigma, int T,
                              int n, int nx, int n0, int m) {
  using Gm = Geo<NB, R>;
  const int N = T - 1;
  TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) {
    const int t = e / NB, j = e - t * NB;
    R val = R(0);
    if (j < n) {
      val = sigma * x[o] - qp.q[t * n + j];
      R eq = R(0);
      // Loops unrolled by 4 so that four independent global loads are in
      // flight per thread (the QP blocks are read from L2 every iteration).
      if (t == 0) {
#pragma unroll 4
        for (int k = 0; k < n0; ++k) eq += qp.A0[k * n + j] * ct[k];
        if (N > 0) {
#pragma unroll 4
          for (int k = 0; k < nx; ++k) eq += qp.Am[k * n + j] * ct[n0 + k];
        }
      } else {
        const R* ap = qp.Ap + (size_t)(t - 1) * nx * n;
#pragma unroll 4
        for (int k = 0; k < nx; ++k) eq += ap[k * n + j] * ct[n0 + (t - 1) * nx + k];
        if (t < N) {
          const R* am = qp.Am + (size_t)t * nx * n;
#pragma unroll 4
          for (int k = 0; k < nx; ++k) eq += am[k * n + j] * ct[n0 + t * nx + k];
        }
      }
      val += eq;
      R iq = R(0);
#pragma unroll 4
      for (int k = 0; k < m; ++k) iq += qp.G[((size_t)t * m + k) * n + j] * gt[t * m + k];
      val += iq;
    }
    gam[o] = val;
  }
}

// s += a . v over n entries: 128-bit loads of the row a when n is a
// multiple of the vector width and the row starts 16-byte aligned, else a
// scalar loop unrolled by 4.  v is an on-chip block-vector row (aligned).
template <typename R>
__device__ __forceinline__ R row_dot(const R* __restrict__ a, const R* __restrict__ v, int n) {
  constexpr int VEC = 16 / (int)sizeof(R);
  R s = R(0);
  if (n % VEC == 0 && (reinterpret_cast<uintptr_t>(a) & 15) == 0) {
#pragma unroll 4
    for (int c = 0; c < n; c += VEC) {
      R w[VEC], x[VEC];
      ld128(w, a + c);  // generic load: a is global or a shared-memory copy
      ld128(x, v + c);
#pragma unroll
      for (int e = 0; e < VEC; ++e) s = fma(w[e], x[e], s);
    }
  } else {
#pragma unroll 4
    for (int j = 0; j < n; ++j) s = fma(a[j], v[j], s);
  }
  return s;
}

// Cx0 = A0 x_0, Cx_t = Am_t x_t + Ap_t x_{t+1}, Gx_t = G_t x_t.
template <int NB, typename R>
__device__ void apply_constraints(R* cx0, R* cx, R* gx, const R* x, const QPView<R>& qp, int T, int n, int nx,
                                  int n0, int m) {
  using Gm = Geo<NB, R>;
  const int N = T - 1;
  const int tot = n0 + N * nx + T * m;
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    if (e < n0) {
      cx0[e] = row_dot(qp.A0 + (size_t)e * n, x, n);
    } else if (e < n0 + N * nx) {
      const int k = e - n0, t = k / nx, i = k - t * nx;
      const R* am = qp.Am + ((size_t)t * nx + i) * n;
      const R* ap = qp.Ap + ((size_t)t * nx + i) * n;
      cx[k] = row_dot(am, x + t * Gm::VSTR, n) + row_dot(ap, x + (t + 1) * Gm::VSTR, n);
    } else {
      const int k = e - n0 - N * nx, t = k / m, i = k - t * m;
      gx[k] = row_dot(qp.G + ((size_t)t * m + i) * n, x + t * Gm::VSTR, n);
    }
  }
}

// Residuals of admm.py:266-331 (primal, dual, normalised), written to sc[0..5].
template <int NB, typename R>
__device__ __noinline__ void compute_residuals(R* sc, R* red, const R* x, const R* zg, const R* yg, const R* xig, const R* yf0,
                                  const R* yfd, const QPView<R>& qp, R slack_w, bool use_slack, int T, int n, int nx,
                                  int n0, int m) {
  using Gm = Geo<NB, R>;
  const int N = T - 1;
  R pr = R(0), ncx = R(0), nc = R(0), ngx = R(0), nz = R(0);
  const int tot = n0 + N * nx + T * m;
  for (int e = threadIdx.x; e < tot; e += blockDim.x) {
    if (e < n0) {
      R s = R(0);
      for (int j = 0; j < n; ++j) s += qp.A0[e * n + j] * x[j];
      pr = fmax(pr, fabs(s - qp.c0[e]));
      ncx = fmax(ncx, fabs(s));
      nc = fmax(nc, fabs(qp.c0[e]));
    } else if (e < n0 + N * nx) {
      const int k = e - n0, t = k / nx, i = k - t * nx;
      const R* am = qp.Am + ((size_t)t * nx + i) * n;
      const R* ap = qp.Ap + ((size_t)t * nx + i) * n;
      R s = R(0);
      for (int j = 0; j < n; ++j) s += am[j] * x[t * Gm::VSTR + j] + ap[j] * x[(t + 1) * Gm::VSTR + j];
      pr = fmax(pr, fabs(s - qp.c[k]));
      ncx = fmax(ncx, fabs(s));
      nc = fmax(nc, fabs(qp.c[k]));
    } else {
      const int k = e - n0 - N * nx, t = k / m, i = k - t * m;
      const R* g = qp.G + ((size_t)t * m + i) * n;
      R s = R(0);
      for (int j = 0; j < n; ++j) s += g[j] * x[t * Gm::VSTR + j];
      pr = fmax(pr, fabs(s - zg[k]));
      ngx = fmax(ngx, fabs(s));
      nz = fmax(nz, fabs(zg[k]));
    }
  }
  R du = R(0), npx = R(0), naty = R(0), nq = R(0);
  for (int e = threadIdx.x; e < T * n; e += blockDim.x) {
    const int t = e / n, j = e - t * n;
    R px = R(0);
    const R* Dt = qp.D + (size_t)t * n * n;
    for (int k = 0; k < n; ++k) px += Dt[j * n + k] * x[t * Gm::VSTR + k];
    if (t > 0) {
      const R* Et = qp.E + (size_t)(t - 1) * n * n;
      for (int k = 0; k < n; ++k) px += Et[j * n + k] * x[(t - 1) * Gm::VSTR + k];
    }
    if (t < N) {
      const R* Et = qp.E + (size_t)t * n * n;
      for (int k = 0; k < n; ++k) px += Et[k * n + j] * x[(t + 1) * Gm::VSTR + k];
    }
    R cty = R(0);
    if (t == 0) {
      for (int k = 0; k < n0; ++k) cty += qp.A0[k * n + j] * yf0[k];
      if (N > 0)
        for (int k = 0; k < nx; ++k) cty += qp.Am[k * n + j] * yfd[k];
    } else {
      const R* ap = qp.Ap + (size_t)(t - 1) * nx * n;
      for (int k = 0; k < nx; ++k) cty += ap[k * n + j] * yfd[(t - 1) * nx + k];
      if (t < N) {
        const R* am = qp.Am + (size_t)t * nx * n;
        for (int k = 0; k < nx; ++k) cty += am[k * n + j] * yfd[t * nx + k];
      }
    }
    for (int k = 0; k < m; ++k) cty += qp.G[((size_t)t * m + k) * n + j] * yg[t * m + k];
    const R qq = qp.q[t * n + j];
    du = fmax(du, fabs(px + qq + cty));
    npx = fmax(npx, fabs(px));
    naty = fmax(naty, fabs(cty));
    nq = fmax(nq, fabs(qq));
  }
  R nxi = R(0), nyg = R(0);
  if (use_slack && m > 0) {
    for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
      du = fmax(du, fabs(slack_w * xig[e] + yg[e]));
      nxi = fmax(nxi, fabs(xig[e]));
      nyg = fmax(nyg, fabs(yg[e]));
    }
  }
  // Per-warp maxima into the 11 x 32 table, one barrier, thread 0 finishes.
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  auto put = [&](int k, R v) {
    v = warp_max(v);
    if (lane == 0) red[k * 32 + wid] = v;
  };
  put(0, pr); put(1, ncx); put(2, nc); put(3, ngx); put(4, nz);
  put(5, du); put(6, npx); put(7, naty); put(8, nq); put(9, nxi); put(10, nyg);
  __syncthreads();
  R outv[11];
  if (threadIdx.x == 0) {
    for (int k = 0; k < 11; ++k) {
      R v = R(0);
      for (int w = 0; w < nw; ++w) v = fmax(v, red[k * 32 + w]);
      outv[k] = v;
    }
  }
  if (threadIdx.x == 0) {
    const R prim = outv[0];
    const R pterm = fmax(fmax(outv[1], outv[3]), fmax(outv[2], outv[4]));
    const R dual = outv[5];
    R dterm = fmax(fmax(outv[6], outv[7]), outv[8]);
    if (use_slack && m > 0) dterm = fmax(dterm, fmax(slack_w * outv[9], outv[10]));
    sc[0] = prim;
    sc[1] = dual;
    sc[2] = prim / (R(1e-10) + pterm);
    sc[3] = dual / (R(1e-10) + dterm);
    sc[4] = pterm;
    sc[5] = dterm;
  }
  __syncthreads();
}

// ct = rho_f c - y_f (equality rows, c0 first), gt = rho z_g - y_g.
template <typename R>
__device__ __forceinline__ void admm_targets(R* ct, R* gt, const QPView<R>& qp, const R* yf0, const R* yfd,
                                             const R* zg, const R* yg, R rho, R rho_f, int T, int nx, int n0, int m) {
  const int N = T - 1;
  for (int e = threadIdx.x; e < n0 + N * nx + T * m; e += blockDim.x) {
    if (e < n0) ct[e] = rho_f * qp.c0[e] - yf0[e];
    else if (e < n0 + N * nx) ct[e] = rho_f * qp.c[e - n0] - yfd[e - n0];
    else gt[e - n0 - N * nx] = rho * zg[e - n0 - N * nx] - yg[e - n0 - N * nx];
  }
}

// Over-relaxation of x and the slack / dual updates (admm.py:884-930, in the
// order of admm_fused.cu:760-860).  Caller syncs before and after.
template <int NB, typename R>
__device__ __forceinline__ void admm_relax_duals(R* x, const R* xold, R* yf0, R* yfd, R* zg, R* yg, R* xig,
                                                 const R* cx0, const R* cx, const R* gx, const QPView<R>& qp, R rho,
                                                 R rho_f, R al, R sw, bool use_slack, int T, int nx, int n0, int m) {
  using Gm = Geo<NB, R>;
  const int N = T - 1;
  TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) { x[o] = al * x[o] + (R(1) - al) * xold[o]; }
  for (int e = threadIdx.x; e < n0 + N * nx + T * m; e += blockDim.x) {
    if (e < n0) {
      yf0[e] += rho_f * al * (cx0[e] - qp.c0[e]);
    } else if (e < n0 + N * nx) {
      const int k = e - n0;
      yfd[k] += rho_f * al * (cx[k] - qp.c[k]);
    } else {
      const int k = e - n0 - N * nx;
      const R zold = zg[k];
      const R zt = al * gx[k] + (R(1) - al) * zold + yg[k] / rho;
      R cl = zt;
      const R lb = qp.l[k], ub = qp.u[k];
      if (cl < lb) cl = lb;
      if (cl > ub) cl = ub;
      R znew;
      if (use_slack) {
        const R f = sw / (sw + rho);
        znew = (R(1) - f) * zt + f * cl;
        xig[k] = (rho / (sw + rho)) * (cl - zt);
      } else {
        znew = cl;
      }
      zg[k] = znew;
      yg[k] += rho * (al * gx[k] + (R(1) - al) * zold - znew);
    }
  }
}

// Residual check every check_every iterations (admm.py:266-331 and the OSQP
// rho rule of admm_fused.cu:870-925).  Returns 1 when converged, 2 when rho
// should change to *rho_new, 0 otherwise.  All threads call it.
template <int NB, typename R>
__device__ __forceinline__ int admm_check(R* sc, R* red, const R* x, const R* zg, const R* yg, const R* xig,
                                          const R* yf0, const R* yfd, const QPView<R>& qp, R sw,
                                          const AdmmParams<R>& P, int it, R rho, R* rho_new, int T, int n, int nx,
                                          int n0, int m) {
  compute_residuals<NB>(sc, red, x, zg, yg, xig, yf0, yfd, qp, sw, P.use_slack != 0, T, n, nx, n0, m);
  const bool conv = (sc[0] < P.eps_abs + P.eps_rel * sc[4]) && (sc[1] < P.eps_abs + P.eps_rel * sc[5]);
  if (conv) return 1;
  if (P.adapt_every > 0 && it >= 2 && (it % P.adapt_every) == 0) {
    R cand = rho * sqrt(sc[2] / (sc[3] + R(1e-30)));
    if (cand < P.rho_min) cand = P.rho_min;
    if (cand > P.rho_max) cand = P.rho_max;
    R ratio = cand / rho;
    if (ratio < R(1)) ratio = R(1) / ratio;
    if (ratio >= P.adapt_tol) {
      *rho_new = cand;
      return 2;
    }
  }
  return 0;
}

// LINSYS: TMPC_LINSYS_PCG (operators on chip or in the workspace, one CTA per
// problem) or TMPC_LINSYS_DIRECT (block Cholesky factor in the workspace, one
// warp = one CTA per problem; requires OPS_SMEM == false).
template <int NB, typename R, bool OPS_SMEM, int LINSYS = TMPC_LINSYS_PCG>
__global__ void __launch_bounds__(max_threads_for(NB)) admm_fused_kernel(const AdmmParams<R> P) {
  using Gm = Geo<NB, R>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  const int b = blockIdx.x;
  if (b >= P.Nb) return;
  const int T = P.T, N = T - 1, n = P.n, nx = P.nx, n0 = P.n0, m = P.m;
  constexpr bool DIRECT = LINSYS == TMPC_LINSYS_DIRECT;
  constexpr int NVEC = DIRECT ? 4 : 12;
  const AdmmSmem<NB, R> L(T, nx, n0, m, OPS_SMEM, NVEC);
  const size_t opn = Gm::op_elems(T);
  R* opS = OPS_SMEM ? sm + L.opS : P.ws + (size_t)b * (DIRECT ? 1 : 2) * opn;
  R* opP = DIRECT ? nullptr : (OPS_SMEM ? sm + L.opP : P.ws + (size_t)b * 2 * opn + opn);
  const size_t VS = (size_t)T * Gm::VSTR;
  R* vbase = sm + L.vec0;
  BlockVecs<NB, R> w{vbase,          vbase + VS,     vbase + 2 * VS,
                     vbase + 3 * VS, vbase + 4 * VS, vbase + 5 * VS,
                     vbase + 6 * VS, (int)VS};
  R* gam = vbase + (DIRECT ? 2 : 10) * VS;
  R* xold = vbase + (DIRECT ? 3 : 11) * VS;
  R* ysolve = vbase + VS;  // direct solve scratch (aliases w.r, unused then)
  R* yf0 = sm + L.yf0;
  R* yfd = sm + L.yfd;
  R* zg = sm + L.zg;
  R* yg = sm + L.yg;
  R* xig = sm + L.xig;
  R* cx0 = sm + L.cx0;
  R* cx = sm + L.cx;
  R* gx = sm + L.gx;
  R* ct = sm + L.ct;
  R* gt = sm + L.gt;
  R* red = sm + L.red;
  R* sc = red + kRedSc;
  __shared__ int flag;
  if (threadIdx.x == 0) flag = 0;

  const QPView<R> qp = qp_view<R>(P.qp, b, T, n, nx, n0, m);

  // ---- load the warm-start state; zero all block vectors (keeps padding 0)
  for (size_t e = threadIdx.x; e < NVEC * VS; e += blockDim.x) vbase[e] = R(0);
  __syncthreads();
  {
    const R* x_in = static_cast<const R*>(P.in.x) + (size_t)b * T * n;
    for (int e = threadIdx.x; e < T * n; e += blockDim.x) {
      const int t = e / n, j = e - t * n;
      w.x[t * Gm::VSTR + j] = x_in[e];
    }
    if (n0 > 0) {
      const R* a = static_cast<const R*>(P.in.y_f0) + (size_t)b * n0;
      for (int e = threadIdx.x; e < n0; e += blockDim.x) yf0[e] = a[e];
    }
    const R* a = static_cast<const R*>(P.in.y_fdyn) + (size_t)b * N * nx;
    for (int e = threadIdx.x; e < N * nx; e += blockDim.x) yfd[e] = a[e];
    if (m > 0) {
      const R* z = static_cast<const R*>(P.in.z_g) + (size_t)b * T * m;
      const R* y = static_cast<const R*>(P.in.y_g) + (size_t)b * T * m;
      const R* xi = static_cast<const R*>(P.in.xi_g) + (size_t)b * T * m;
      for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
        zg[e] = z[e];
        yg[e] = y[e];
        xig[e] = xi[e];
      }
    }
  }
  R rho = static_cast<const R*>(P.in.rho_bar)[b];
  const R sw = P.slack_weight ? P.slack_weight[b] : R(0);
  const R al = P.alpha;
  const PackedAcc<NB, R> acc{opS, opP, T};

  const FactorView<NB, R> F{opS, T};
  auto build_operators = [&](R rho_now) {
    if constexpr (DIRECT) {
      assemble_theta_phi<NB>(acc, qp, rho_now * P.rho_f_factor, rho_now, P.sigma, T, n, nx, n0, m);
      __syncthreads();
      if (!riccati_factor_warp<NB>(F, sm + L.fm, n, PackedSrc<NB, R>{F}) && threadIdx.x == 0)
        flag |= TMPC_STATUS_SINGULAR_BLOCK;
      __syncthreads();
    } else {
      assemble_ops<NB>(acc, qp, rho_now * P.rho_f_factor, rho_now, P.sigma, T, n, nx, n0, m, &flag);
    }
  };
  build_operators(rho);

  uint32_t iters = (uint32_t)P.max_iter;
  for (int it = 0; it < P.max_iter; ++it) {
    const R rho_f = rho * P.rho_f_factor;
    admm_targets(ct, gt, qp, yf0, yfd, zg, yg, rho, rho_f, T, nx, n0, m);
    __syncthreads();
    compute_gamma<NB>(gam, w.x, qp, ct, gt, P.sigma, T, n, nx, n0, m);
    TMPC_FOR_ENTRIES(e, o, T, NB, Gm::VSTR) { xold[o] = w.x[o]; }
    __syncthreads();
    if constexpr (DIRECT) {
      riccati_solve_warp<NB, R, false>(F, gam, ysolve, w.x);
      __syncthreads();
    } else {
      pcg_solve<NB, OPS_SMEM>(opS, opP, T, gam, w, red, P.pcg_max_iter, P.pcg_eps);
    }
    apply_constraints<NB>(cx0, cx, gx, w.x, qp, T, n, nx, n0, m);
    __syncthreads();
    admm_relax_duals<NB>(w.x, xold, yf0, yfd, zg, yg, xig, cx0, cx, gx, qp, rho, rho_f, al, sw, P.use_slack != 0, T,
                         nx, n0, m);
    __syncthreads();
    if (P.check_every > 0 && (it % P.check_every) == 0) {
      R rho_new;
      const int st = admm_check<NB>(sc, red, w.x, zg, yg, xig, yf0, yfd, qp, sw, P, it, rho, &rho_new, T, n, nx, n0, m);
      if (st == 1) {
        iters = (uint32_t)(it + 1);
        break;
      }
      if (st == 2) {
        rho = rho_new;
        build_operators(rho);
      }
      __syncthreads();
    }
  }

  // ---- store
  bool nonfinite = false;
  {
    R* xo = static_cast<R*>(P.out.x) + (size_t)b * T * n;
    R* xo2 = P.x_out ? P.x_out + (size_t)b * T * n : nullptr;
    for (int e = threadIdx.x; e < T * n; e += blockDim.x) {
      const int t = e / n, j = e - t * n;
      const R v = w.x[t * Gm::VSTR + j];
      if (!isfinite(v)) nonfinite = true;
      xo[e] = v;
      if (xo2) xo2[e] = v;
    }
    if (n0 > 0) {
      R* a = static_cast<R*>(P.out.y_f0) + (size_t)b * n0;
      for (int e = threadIdx.x; e < n0; e += blockDim.x) a[e] = yf0[e];
    }
    R* a = static_cast<R*>(P.out.y_fdyn) + (size_t)b * N * nx;
    for (int e = threadIdx.x; e < N * nx; e += blockDim.x) a[e] = yfd[e];
    if (m > 0) {
      R* z = static_cast<R*>(P.out.z_g) + (size_t)b * T * m;
      R* y = static_cast<R*>(P.out.y_g) + (size_t)b * T * m;
      R* xi = static_cast<R*>(P.out.xi_g) + (size_t)b * T * m;
      for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
        z[e] = zg[e];
        y[e] = yg[e];
        xi[e] = xig[e];
      }
    }
  }
  if (nonfinite) atomicOr(&flag, TMPC_STATUS_NONFINITE);
  __syncthreads();
  if (threadIdx.x == 0) {
    static_cast<R*>(P.out.rho_bar)[b] = rho;
    if (P.iters_out) P.iters_out[b] = iters;
    if (P.status_out) P.status_out[b] = flag;
  }
}


template <int NB, typename R>
size_t admm_smem_bytes(int T, int nx, int n0, int m, bool ops_smem) {
  return AdmmSmem<NB, R>(T, nx, n0, m, ops_smem).nelem * sizeof(R);
}

template <int NB, typename R>
int launch_admm_direct_nb(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st) {
  const size_t need = (size_t)P.Nb * Geo<NB, R>::op_elems(P.T) * sizeof(R);
  if (P.ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(P.ws) & 15) != 0) return TMPC_ERR_WORKSPACE;
  const size_t smem = AdmmSmem<NB, R>(P.T, P.nx, P.n0, P.m, false, 4).nelem * sizeof(R);
  if ((long)smem > max_dyn_smem()) return TMPC_ERR_SMEM;
  auto k = admm_fused_kernel<NB, R, false, TMPC_LINSYS_DIRECT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  k<<<P.Nb, 32, smem, st>>>(P);
  return (int)cudaPeekAtLastError();
}

template <int NB, typename R>
int launch_admm_nb(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st) {
  const int th = cta_threads(P.T, max_threads_for(NB));
  const int smax = max_dyn_smem();
  const size_t s_res = admm_smem_bytes<NB, R>(P.T, P.nx, P.n0, P.m, true);
  if ((long)s_res <= smax) {
    auto k = admm_fused_kernel<NB, R, true>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s_res);
    if (e != cudaSuccess) return (int)e;
    k<<<P.Nb, th, s_res, st>>>(P);
    return (int)cudaPeekAtLastError();
  }
  const size_t need = (size_t)P.Nb * 2 * Geo<NB, R>::op_elems(P.T) * sizeof(R);
  if (P.ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(P.ws) & 15) != 0) return TMPC_ERR_WORKSPACE;
  const size_t s_str = admm_smem_bytes<NB, R>(P.T, P.nx, P.n0, P.m, false);
  if ((long)s_str > smax) return TMPC_ERR_SMEM;
  auto k = admm_fused_kernel<NB, R, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s_str);
  if (e != cudaSuccess) return (int)e;
  k<<<P.Nb, th, s_str, st>>>(P);
  return (int)cudaPeekAtLastError();
}

}  // namespace tmpc
