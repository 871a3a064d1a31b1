// Fused ADMM solve and Schur assembly for stage blocks wider than 32
// (32 < n <= 96; the reference's own dimension sweep reaches nx = 64,
// nu = 32, benchmarking/linear-system/run_sweeps_oat_turbompc.sh:122).
//
// One CTA per problem, as admm_fused_kernel, with the same ADMM-level steps
// (admm_kernel.cuh: targets, gamma, constraints, relaxation, slack, duals,
// residual checks and the rho rule) and the reference's PCG semantics
// (admm_fused.cu:54-161).  What changes is the linear-system layer:
//   * S and Phiinv live in the caller's workspace in the reference layout
//     [T][n][3n] (too large for a CTA's shared memory at these sizes), built
//     by gen_build below: per stage Theta_t and Phi_t (admm.py:86-101), Theta_t^-1
//     by Gauss-Jordan elimination on [Theta_t | I] in a workspace scratch
//     (Theta_t is symmetric positive definite: no row exchanges; a pivot that
//     is not positive and finite sets TMPC_STATUS_SINGULAR_BLOCK), then the
//     preconditioner's off-diagonal blocks Theta_t^-1 Phi_{t-1} Theta_{t-1}^-1 and
//     Theta_t^-1 Phi_t^T Theta_{t+1}^-1 (admm.py:123-153);
//   * every PCG matvec streams its operator's rows from L2 / HBM, one thread
//     per row (the operators are written inside the kernel, so they are read
//     through the coherent path, not the read-only one).
// The block vectors stay in shared memory as [T][VSTR].
#include "admm_kernel.cuh"

namespace tmpc {
namespace gen {

template <typename R>
struct Ws {
  R* S;   // [T][n][3n]
  R* P;   // [T][n][3n]
  R* gj;  // [n][2n] Gauss-Jordan scratch (also pass 2's n x n temporary)
};

__host__ __device__ inline size_t ws_elems_per_problem(int T, int n) {
  const size_t e = 2 * (size_t)T * n * 3 * n + 2 * (size_t)n * n;
  return (e + 3) & ~size_t(3);  // keep each problem's area 16-byte aligned in fp32
}

// Pass 1 for one problem (all threads of the CTA): for every stage the S
// row blocks [Phi_{t-1} | Theta_t | Phi_t^T] and -Theta_t^-1 in Phiinv's
// middle block.  The Gauss-Jordan elimination runs on [Theta_t | I] in
// `gj` (row stride gs >= 2n); with gj == nullptr it runs in place in the
// stage's own Phiinv row block (row stride 3n), so that Theta_t^-1 ends up in
// the middle block (the outer blocks are written by pass 2).
template <typename R>
__device__ void build_pass1(const QPView<R>& qp, R* S, R* Pm, R* gj_ws, R* fcol, R rho_f, R rho, R sigma, int T,
                            int n, int nx, int n0, int m, int* flag) {
  const int N = T - 1, n3 = 3 * n;
  for (int t = 0; t < T; ++t) {
    R* Srow = S + (size_t)t * n * n3;
    R* Prow = Pm + (size_t)t * n * n3;
    R* gj = gj_ws ? gj_ws : Prow;
    const int gs = gj_ws ? 2 * n : n3;
    for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
      const int i = e / n, j = e - i * n;
      R v = qp.D[((size_t)t * n + i) * n + j] + (i == j ? sigma : R(0));
      R gg = R(0);
      for (int k = 0; k < m; ++k) gg += qp.G[((size_t)t * m + k) * n + i] * qp.G[((size_t)t * m + k) * n + j];
      v += rho * gg;
      R cc = R(0);
      if (t == 0) {
        for (int k = 0; k < n0; ++k) cc += qp.A0[(size_t)k * n + i] * qp.A0[(size_t)k * n + j];
      } else {
        const R* ap = qp.Ap + (size_t)(t - 1) * nx * n;
        for (int k = 0; k < nx; ++k) cc += ap[(size_t)k * n + i] * ap[(size_t)k * n + j];
      }
      if (t < N) {
        const R* am = qp.Am + (size_t)t * nx * n;
        for (int k = 0; k < nx; ++k) cc += am[(size_t)k * n + i] * am[(size_t)k * n + j];
      }
      v += rho_f * cc;
      gj[i * gs + j] = v;
      gj[i * gs + n + j] = (i == j) ? R(1) : R(0);
      Srow[(size_t)i * n3 + n + j] = v;
      // Phi_{t-1}[i][j] in the left block, Phi_t^T[i][j] = Phi_t[j][i] in the right block,
      // Phi_s = E_s + rho_f Ap_s^T Am_s
      R left = R(0), right = R(0);
      if (t > 0) {
        const R* ap = qp.Ap + (size_t)(t - 1) * nx * n;
        const R* am = qp.Am + (size_t)(t - 1) * nx * n;
        R sacc = R(0);
        for (int k = 0; k < nx; ++k) sacc += ap[(size_t)k * n + i] * am[(size_t)k * n + j];
        left = qp.E[((size_t)(t - 1) * n + i) * n + j] + rho_f * sacc;
      }
      if (t < N) {
        const R* ap = qp.Ap + (size_t)t * nx * n;
        const R* am = qp.Am + (size_t)t * nx * n;
        R sacc = R(0);
        for (int k = 0; k < nx; ++k) sacc += ap[(size_t)k * n + j] * am[(size_t)k * n + i];
        right = qp.E[((size_t)t * n + j) * n + i] + rho_f * sacc;
      }
      Srow[(size_t)i * n3 + j] = left;
      Srow[(size_t)i * n3 + 2 * n + j] = right;
    }
    __syncthreads();
    for (int k = 0; k < n; ++k) {
      const R piv = gj[k * gs + k];
      if (threadIdx.x == 0 && (!(piv > R(0)) || !isfinite(piv))) atomicOr(flag, TMPC_STATUS_SINGULAR_BLOCK);
      const R rinv = R(1) / piv;
      for (int i = threadIdx.x; i < n; i += blockDim.x) fcol[i] = gj[i * gs + k];
      __syncthreads();
      for (int j = threadIdx.x; j < 2 * n; j += blockDim.x) gj[k * gs + j] *= rinv;
      __syncthreads();
      for (int e = threadIdx.x; e < n * 2 * n; e += blockDim.x) {
        const int i = e / (2 * n), j = e - i * 2 * n;
        if (i != k) gj[i * gs + j] -= fcol[i] * gj[k * gs + j];
      }
      __syncthreads();
    }
    for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
      const int i = e / n, j = e - i * n;
      Prow[(size_t)i * n3 + n + j] = -gj[i * gs + n + j];  // -Theta_t^-1 (in place when gj is Prow)
    }
    __syncthreads();
  }
}

// Pass 2 for stage t: Phiinv's outer blocks Theta_t^-1 Phi_{t-1} Theta_{t-1}^-1
// and Theta_t^-1 Phi_t^T Theta_{t+1}^-1 (zero at the ends), from S's outer
// blocks and the middle blocks -Theta^-1 of stages t - 1, t, t + 1; tmp is an
// n x n scratch.  Reads only S and middle blocks, writes only outer blocks.
template <typename R>
__device__ void build_pass2_stage(R* S, R* Pm, R* tmp, int t, int T, int n) {
  const int N = T - 1, n3 = 3 * n;
  const R* Pt = Pm + (size_t)t * n * n3;
  const R* St = S + (size_t)t * n * n3;
  R* Pw = Pm + (size_t)t * n * n3;
  for (int side = 0; side < 2; ++side) {
    const bool has = side == 0 ? t > 0 : t < N;
    const int coff = side == 0 ? 0 : 2 * n;
    if (has) {
      for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
        const int i = e / n, j = e - i * n;
        R acc = R(0);
        for (int k = 0; k < n; ++k) acc += Pt[(size_t)i * n3 + n + k] * St[(size_t)k * n3 + coff + j];
        tmp[e] = -acc;  // Theta_t^-1 (S block)
      }
      __syncthreads();
      const R* Pn = Pm + (size_t)(side == 0 ? t - 1 : t + 1) * n * n3;
      for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
        const int i = e / n, j = e - i * n;
        R acc = R(0);
        for (int k = 0; k < n; ++k) acc += tmp[i * n + k] * Pn[(size_t)k * n3 + n + j];
        Pw[(size_t)i * n3 + coff + j] = -acc;
      }
      __syncthreads();
    } else {
      for (int e = threadIdx.x; e < n * n; e += blockDim.x) {
        const int i = e / n, j = e - i * n;
        Pw[(size_t)i * n3 + coff + j] = R(0);
      }
    }
  }
}

// S and Phiinv of one problem for (rho_f, rho) (admm.py:71-154); all threads.
template <typename R>
__device__ void build(const QPView<R>& qp, const Ws<R>& W, R* fcol, R rho_f, R rho, R sigma, int T, int n, int nx,
                      int n0, int m, int* flag) {
  build_pass1<R>(qp, W.S, W.P, W.gj, fcol, rho_f, rho, sigma, T, n, nx, n0, m, flag);
  for (int t = 0; t < T; ++t) build_pass2_stage<R>(W.S, W.P, W.gj, t, T, n);
  __syncthreads();
}

// y = M v for the reference-layout M [T][n][3n]; v, y are [T][VSTR] vectors.
template <int NB, typename R>
__device__ __forceinline__ void matvec(R* y, const R* M, const R* v, int T, int n) {
  using Gm = Geo<NB, R>;
  const int n3 = 3 * n;
  for (int row = threadIdx.x; row < T * n; row += blockDim.x) {
    const int t = row / n, i = row - t * n;
    const R* mr = M + (size_t)row * n3;
    R s = R(0);
    if (t > 0) {
      const R* vp = v + (t - 1) * Gm::VSTR;
#pragma unroll 4
      for (int j = 0; j < n; ++j) s = fma(mr[j], vp[j], s);
    }
    {
      const R* vc = v + t * Gm::VSTR;
#pragma unroll 4
      for (int j = 0; j < n; ++j) s = fma(mr[n + j], vc[j], s);
    }
    if (t < T - 1) {
      const R* vn = v + (t + 1) * Gm::VSTR;
#pragma unroll 4
      for (int j = 0; j < n; ++j) s = fma(mr[2 * n + j], vn[j], s);
    }
    y[t * Gm::VSTR + i] = s;
  }
}

#define TMPC_GEN_FOR(e, o, T, n, VSTR)                                                                 \
  for (int e = threadIdx.x, o = 0; e < (T) * (n) && ((o = (e / (n)) * (VSTR) + e % (n)), true); \
       e += blockDim.x)

// PCG with the semantics of admm_fused.cu:54-161 (stop when |eta| < 1e-12 +
// eps |eta_0|, p.Sp clamped at 1e-30); x is the warm start and the result.
template <int NB, typename R>
__device__ int pcg(const R* S, const R* P, int T, int n, const R* g, R* x, R* r, R* z, R* p, R* d, R* red,
                   int max_iter, R eps) {
  using Gm = Geo<NB, R>;
  matvec<NB>(d, S, x, T, n);
  __syncthreads();
  TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) { r[o] = g[o] - d[o]; }
  __syncthreads();
  matvec<NB>(z, P, r, T, n);
  __syncthreads();
  R part = R(0);
  TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) {
    p[o] = z[o];
    part = fma(r[o], z[o], part);
  }
  R eta = block_sum(part, red);
  const R eta0 = fabs(eta);
  int it = 0;
  for (; it < max_iter; ++it) {
    if (fabs(eta) < R(1e-12) + eps * eta0) break;
    __syncthreads();
    matvec<NB>(d, S, p, T, n);
    __syncthreads();
    part = R(0);
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) { part = fma(p[o], d[o], part); }
    R den = block_sum(part, red + 32);
    if (fabs(den) < R(1e-30)) den = R(1e-30);
    const R alpha = eta / den;
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) {
      x[o] = fma(alpha, p[o], x[o]);
      r[o] = fma(-alpha, d[o], r[o]);
    }
    __syncthreads();
    matvec<NB>(z, P, r, T, n);
    __syncthreads();
    part = R(0);
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) { part = fma(r[o], z[o], part); }
    const R eta_new = block_sum(part, red);
    const R beta = eta_new / eta;
    eta = eta_new;
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) { p[o] = fma(beta, p[o], z[o]); }
  }
  __syncthreads();
  return it;
}

// Shared-memory layout: 7 block vectors (x r z p d gam xold) and the ADMM
// vectors of AdmmSmem (reused with no operators on chip), plus fcol (n).
template <int NB, typename R>
struct Smem {
  AdmmSmem<NB, R> A;
  size_t fcol, nelem;
  __host__ __device__ Smem(int T, int nx, int n0, int m, int n) : A(T, nx, n0, m, false, 7) {
    fcol = A.nelem;
    nelem = (fcol + n + 3) & ~size_t(3);
  }
};

constexpr int kThreads = 512;

template <int NB, typename R>
__global__ void __launch_bounds__(kThreads) admm_kernel(const AdmmParams<R> P) {
  using Gm = Geo<NB, R>;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sm = reinterpret_cast<R*>(smem_raw);
  const int b = blockIdx.x;
  if (b >= P.Nb) return;
  const int T = P.T, N = T - 1, n = P.n, nx = P.nx, n0 = P.n0, m = P.m;
  const Smem<NB, R> L(T, nx, n0, m, n);
  const size_t VS = (size_t)T * Gm::VSTR;
  R* vb = sm + L.A.vec0;
  R *x = vb, *r = vb + VS, *z = vb + 2 * VS, *p = vb + 3 * VS, *d = vb + 4 * VS, *gam = vb + 5 * VS,
    *xold = vb + 6 * VS;
  R* yf0 = sm + L.A.yf0;
  R* yfd = sm + L.A.yfd;
  R* zg = sm + L.A.zg;
  R* yg = sm + L.A.yg;
  R* xig = sm + L.A.xig;
  R* cx0 = sm + L.A.cx0;
  R* cx = sm + L.A.cx;
  R* gx = sm + L.A.gx;
  R* ct = sm + L.A.ct;
  R* gt = sm + L.A.gt;
  R* red = sm + L.A.red;
  R* sc = red + kRedSc;
  R* fcol = sm + L.fcol;
  __shared__ int flag;
  if (threadIdx.x == 0) flag = 0;
  const size_t wpp = ws_elems_per_problem(T, n);
  R* wb = P.ws + (size_t)b * wpp;
  const Ws<R> W{wb, wb + (size_t)T * n * 3 * n, wb + 2 * (size_t)T * n * 3 * n};
  const QPView<R> qp = qp_view<R>(P.qp, b, T, n, nx, n0, m);

  for (size_t e = threadIdx.x; e < 7 * VS; e += blockDim.x) vb[e] = R(0);
  __syncthreads();
  {
    const R* x_in = static_cast<const R*>(P.in.x) + (size_t)b * T * n;
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) { x[o] = x_in[e]; }
    if (n0 > 0) {
      const R* a = static_cast<const R*>(P.in.y_f0) + (size_t)b * n0;
      for (int e = threadIdx.x; e < n0; e += blockDim.x) yf0[e] = a[e];
    }
    const R* a = static_cast<const R*>(P.in.y_fdyn) + (size_t)b * N * nx;
    for (int e = threadIdx.x; e < N * nx; e += blockDim.x) yfd[e] = a[e];
    if (m > 0) {
      const R* zz = static_cast<const R*>(P.in.z_g) + (size_t)b * T * m;
      const R* yy = static_cast<const R*>(P.in.y_g) + (size_t)b * T * m;
      const R* xi = static_cast<const R*>(P.in.xi_g) + (size_t)b * T * m;
      for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
        zg[e] = zz[e];
        yg[e] = yy[e];
        xig[e] = xi[e];
      }
    }
  }
  R rho = static_cast<const R*>(P.in.rho_bar)[b];
  const R sw = P.slack_weight ? P.slack_weight[b] : R(0);
  const R al = P.alpha;
  __syncthreads();
  build<R>(qp, W, fcol, rho * P.rho_f_factor, rho, P.sigma, T, n, nx, n0, m, &flag);

  uint32_t iters = (uint32_t)P.max_iter;
  for (int it = 0; it < P.max_iter; ++it) {
    const R rho_f = rho * P.rho_f_factor;
    admm_targets(ct, gt, qp, yf0, yfd, zg, yg, rho, rho_f, T, nx, n0, m);
    __syncthreads();
    compute_gamma<NB>(gam, x, qp, ct, gt, P.sigma, T, n, nx, n0, m);
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) { xold[o] = x[o]; }
    __syncthreads();
    pcg<NB>(W.S, W.P, T, n, gam, x, r, z, p, d, red, P.pcg_max_iter, P.pcg_eps);
    apply_constraints<NB>(cx0, cx, gx, x, qp, T, n, nx, n0, m);
    __syncthreads();
    admm_relax_duals<NB>(x, xold, yf0, yfd, zg, yg, xig, cx0, cx, gx, qp, rho, rho_f, al, sw, P.use_slack != 0, T, nx,
                         n0, m);
    __syncthreads();
    if (P.check_every > 0 && (it % P.check_every) == 0) {
      R rho_new;
      const int st = admm_check<NB>(sc, red, x, zg, yg, xig, yf0, yfd, qp, sw, P, it, rho, &rho_new, T, n, nx, n0, m);
      if (st == 1) {
        iters = (uint32_t)(it + 1);
        break;
      }
      if (st == 2) {
        rho = rho_new;
        build<R>(qp, W, fcol, rho * P.rho_f_factor, rho, P.sigma, T, n, nx, n0, m, &flag);
      }
      __syncthreads();
    }
  }

  bool nonfinite = false;
  {
    R* xo = static_cast<R*>(P.out.x) + (size_t)b * T * n;
    R* xo2 = P.x_out ? P.x_out + (size_t)b * T * n : nullptr;
    TMPC_GEN_FOR(e, o, T, n, Gm::VSTR) {
      const R v = x[o];
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
      R* zz = static_cast<R*>(P.out.z_g) + (size_t)b * T * m;
      R* yy = static_cast<R*>(P.out.y_g) + (size_t)b * T * m;
      R* xi = static_cast<R*>(P.out.xi_g) + (size_t)b * T * m;
      for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
        zz[e] = zg[e];
        yy[e] = yg[e];
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

// Standalone assembly (tmpc_schur_assemble_* for n > 32) into the caller's
// S / Phiinv, with no workspace: pass 1 per problem (Gauss-Jordan in each
// stage's Phiinv row block), then pass 2 per (problem, stage).
template <typename R>
__global__ void __launch_bounds__(256) assemble_pass1_kernel(const TmpcQP qpp, const R* rho, R sigma, R rff, R* S,
                                                             R* Pm, int32_t* status, int Nb, int T, int n, int nx,
                                                             int n0, int m) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* fcol = reinterpret_cast<R*>(smem_raw);
  __shared__ int flag;
  const int b = blockIdx.x;
  if (b >= Nb) return;
  if (threadIdx.x == 0) flag = 0;
  __syncthreads();
  const size_t per = (size_t)T * n * 3 * n;
  const QPView<R> qp = qp_view<R>(qpp, b, T, n, nx, n0, m);
  const R r = rho[b];
  build_pass1<R>(qp, S + (size_t)b * per, Pm + (size_t)b * per, nullptr, fcol, r * rff, r, sigma, T, n, nx, n0, m,
                 &flag);
  if (threadIdx.x == 0 && status) status[b] = flag;
}

template <typename R>
__global__ void __launch_bounds__(256) assemble_pass2_kernel(R* S, R* Pm, int Nb, int T, int n) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* tmp = reinterpret_cast<R*>(smem_raw);
  const int t = blockIdx.x, b = blockIdx.y;
  if (b >= Nb || t >= T) return;
  const size_t per = (size_t)T * n * 3 * n;
  build_pass2_stage<R>(S + (size_t)b * per, Pm + (size_t)b * per, tmp, t, T, n);
}

template <typename R, class F>
int dispatch(int n, F&& f) {
  if (n <= 48) return f(std::integral_constant<int, 48>{});
  if (n <= 64) return f(std::integral_constant<int, 64>{});
  if (n <= 96) return f(std::integral_constant<int, 96>{});
  return TMPC_ERR_UNSUPPORTED;
}

}  // namespace gen

constexpr int kGenMaxN = 96;

template <typename R>
size_t admm_generic_ws_bytes(const TmpcDims& d) {
  if (d.n <= 32 || d.n > kGenMaxN) return 0;
  return (size_t)d.Nb * gen::ws_elems_per_problem(d.T, d.n) * sizeof(R);
}

template <typename R>
int launch_admm_generic(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st) {
  if (P.n > kGenMaxN) return TMPC_ERR_UNSUPPORTED;
  const size_t need = (size_t)P.Nb * gen::ws_elems_per_problem(P.T, P.n) * sizeof(R);
  if (P.ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(P.ws) & 15) != 0) return TMPC_ERR_WORKSPACE;
  return gen::dispatch<R>(P.n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    const size_t smem = gen::Smem<NB, R>(P.T, P.nx, P.n0, P.m, P.n).nelem * sizeof(R);
    if ((long)smem > max_dyn_smem()) return (int)TMPC_ERR_SMEM;
    auto k = gen::admm_kernel<NB, R>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    k<<<P.Nb, gen::kThreads, smem, st>>>(P);
    return (int)cudaPeekAtLastError();
  });
}

template <typename R>
int assemble_generic(const TmpcDims* d, const TmpcQP* qp, const R* rho, R sigma, R rff, R* S, R* P, int32_t* status,
                     cudaStream_t st) {
  if (d->n > kGenMaxN) return TMPC_ERR_UNSUPPORTED;
  if (d->Nb > 65535) return TMPC_ERR_BAD_DIMS;  // grid.y of pass 2
  gen::assemble_pass1_kernel<R><<<d->Nb, 256, (size_t)(d->n + 4) * sizeof(R), st>>>(
      *qp, rho, sigma, rff, S, P, status, d->Nb, d->T, d->n, d->nx, d->n0, d->m);
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return (int)e;
  const size_t smem = (size_t)d->n * d->n * sizeof(R);
  auto k2 = gen::assemble_pass2_kernel<R>;
  e = cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  k2<<<dim3(d->T, d->Nb), 256, smem, st>>>(S, P, d->Nb, d->T, d->n);
  return (int)cudaPeekAtLastError();
}

template size_t admm_generic_ws_bytes<float>(const TmpcDims&);
template size_t admm_generic_ws_bytes<double>(const TmpcDims&);
template int launch_admm_generic<float>(const AdmmParams<float>&, size_t, cudaStream_t);
template int launch_admm_generic<double>(const AdmmParams<double>&, size_t, cudaStream_t);
template int assemble_generic<float>(const TmpcDims*, const TmpcQP*, const float*, float, float, float*, float*,
                                     int32_t*, cudaStream_t);
template int assemble_generic<double>(const TmpcDims*, const TmpcQP*, const double*, double, double, double*,
                                      double*, int32_t*, cudaStream_t);

}  // namespace tmpc
