// Fused ADMM with the direct (block-Cholesky) linear solve on the
// batch-interleaved layout: the `linsys = DIRECT` path (the drop-in for the
// reference's admm_fused_cudss, turbompc/solvers/admm/csrc/admm_cudss.cu) for
// stage blocks up to the interleaved factor's limit (n <= 16 fp32, n <= 12
// fp64).
//
// Same iteration as admm_fused_kernel (admm_kernel.cuh; order of
// turbompc/solvers/admm/admm.py:795-1049):
//   gamma = sigma x - q + C^T(rho_f c - y_f) + G^T(rho z - y_g)
//   x~ = S^-1 gamma                       (S = L L^T, block Cholesky)
//   C x~, G x~ on x~; y_f += rho_f alpha (C x~ - c);
//   z~ = alpha G x~ + (1 - alpha) z + y_g / rho, z = clamp (or the slack form),
//   y_g += rho (alpha G x~ + (1 - alpha) z_old - z);  x = alpha x~ + (1 - alpha) x
//   every check_every iterations: residuals, convergence, rho adaptation and
//   a new factor.
//
// Layout: every per-problem array lives in the workspace in the interleaved
// form (groups of 32 problems, element-major, problem-minor; riccati_il.cuh),
// so a warp whose lanes are 32 problems touches every element with one
// 128-byte (fp32) transaction.  One block of kIlWarps warps runs one group
// for a chunk of ADMM iterations.  An iteration is two sweeps over the stages:
//   forward  (t = 0 .. T-1):  y_t = L_t^-1 (gamma_t - W_{t-1} y_{t-1})
//   backward (t = T-1 .. 0):  x~_t = L_t^-T (y_t - W_t^T x~_{t+1}), then on the
//            spot the stage's dynamics rows (they need x~_t and x~_{t+1}), its
//            inequality rows, the relaxation of x_t, and gamma for the next
//            iteration (gamma_t needs the new duals of the dynamics rows t - 1
//            and t, so it is completed one step later).
// Each stage's data (factor blocks, QP rows, state) is a set of contiguous
// byte ranges of the interleaved arrays; the whole block copies them into
// shared memory with 16-byte cp.async ahead of use (forward: two stage
// buffers; backward: the factor part and the QP / state part of a stage in
// separate buffers, each refilled as soon as it is consumed), so the QP
// blocks are read once per iteration and no thread waits on global memory
// inside a stage.
//
// Host sequence per call (stream-ordered, no host synchronisation): convert
// the QP and the state to the interleaved layout, assemble Theta / Phi,
// factor in place, form the first gamma, then run the iterations in chunks
// that end at the residual checks (one launch when check_every = 0).  A
// check that changes some problem's rho re-assembles and re-factors (the
// factor overwrote the operator) and recomputes gamma for those problems.
#include "admm_kernel.cuh"
#include "riccati_il.cuh"

namespace tmpc {
namespace il {

constexpr int kIlWarps = 8;
constexpr int kIlThreads = 32 * kIlWarps;

// Element counts per problem of the interleaved workspace arrays.
struct IlSizes {
  size_t ops, q, a0, am, g, c0, c, lu, x, yf0, yfd, zm;
  __host__ __device__ IlSizes(int T, int n, int nx, int n0, int m) {
    const size_t N = T - 1;
    ops = op_elems(T, n);
    q = (size_t)T * n;
    a0 = (size_t)n0 * n;
    am = N * nx * n;
    g = (size_t)T * m * n;
    c0 = n0;
    c = N * nx;
    lu = (size_t)T * m;
    x = (size_t)T * n;
    yf0 = n0;
    yfd = N * nx;
    zm = (size_t)T * m;
  }
};

// Workspace layout: R arrays (each G32 x elems, G32 = 32 x groups) then int arrays.
template <typename R>
struct IlWs {
  size_t ops, q, a0, am, ap, g, c0, c, l, u, x, yf0, yfd, zg, yg, xig, gam, ys, rho, sw;  // R offsets
  size_t act, iters, status, fstat, chg, gate;                                           // int offsets
  size_t rbytes, bytes;
  IlWs(int Nb, int T, int n, int nx, int n0, int m) {
    const IlSizes z(T, n, nx, n0, m);
    const size_t G32 = groups(Nb) * kWarp;
    size_t o = 0;
    auto take = [&](size_t e) {
      const size_t r = o;
      o += e * G32;
      return r;
    };
    ops = take(z.ops); q = take(z.q); a0 = take(z.a0); am = take(z.am); ap = take(z.am); g = take(z.g);
    c0 = take(z.c0); c = take(z.c); l = take(z.lu); u = take(z.lu); x = take(z.x); yf0 = take(z.yf0);
    yfd = take(z.yfd); zg = take(z.zm); yg = take(z.zm); xig = take(z.zm); gam = take(z.x); ys = take(z.x);
    rho = take(1); sw = take(1);
    rbytes = (o * sizeof(R) + 255) & ~size_t(255);
    size_t io = 0;
    act = io; io += G32;
    iters = io; io += G32;
    status = io; io += G32;
    fstat = io; io += G32;
    chg = io; io += G32;
    gate = io; io += 4;
    bytes = rbytes + io * sizeof(int);
  }
};

// Pointers and parameters of the interleaved kernels.
template <typename R>
struct IlArgs {
  R *ops, *q, *a0, *am, *ap, *g, *c0, *c, *l, *u, *x, *yf0, *yfd, *zg, *yg, *xig, *gam, *ys, *rho, *sw;
  int *act, *iters, *status, *fstat, *chg, *gate;
  int Nb, T, n, nx, n0, m, use_slack;
  R sigma, alpha, rff;
};

template <typename R>
IlArgs<R> il_args(void* ws, const AdmmParams<R>& P) {
  const IlWs<R> L(P.Nb, P.T, P.n, P.nx, P.n0, P.m);
  R* r = static_cast<R*>(ws);
  int* i = reinterpret_cast<int*>(static_cast<unsigned char*>(ws) + L.rbytes);
  IlArgs<R> a;
  a.ops = r + L.ops; a.q = r + L.q; a.a0 = r + L.a0; a.am = r + L.am; a.ap = r + L.ap; a.g = r + L.g;
  a.c0 = r + L.c0; a.c = r + L.c; a.l = r + L.l; a.u = r + L.u; a.x = r + L.x; a.yf0 = r + L.yf0;
  a.yfd = r + L.yfd; a.zg = r + L.zg; a.yg = r + L.yg; a.xig = r + L.xig; a.gam = r + L.gam; a.ys = r + L.ys;
  a.rho = r + L.rho; a.sw = r + L.sw;
  a.act = i + L.act; a.iters = i + L.iters; a.status = i + L.status; a.fstat = i + L.fstat; a.chg = i + L.chg;
  a.gate = i + L.gate;
  a.Nb = P.Nb; a.T = P.T; a.n = P.n; a.nx = P.nx; a.n0 = P.n0; a.m = P.m; a.use_slack = P.use_slack;
  a.sigma = P.sigma; a.alpha = P.alpha; a.rff = P.rho_f_factor;
  return a;
}

// Element e of problem b of an interleaved array with E elements per problem.
__host__ __device__ __forceinline__ size_t ix(int b, size_t E, size_t e) {
  return ((size_t)(b / kWarp) * E + e) * kWarp + (b % kWarp);
}

// ---------------------------------------------------------------------------
// Per-problem scalars in: rho, slack weight, active flags, iteration counts.
// ---------------------------------------------------------------------------
template <typename R>
__global__ void il_scalars_in_kernel(IlArgs<R> A, const R* rho_in, const R* sw_in, int max_iter) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  const int G32 = (int)(groups(A.Nb) * kWarp);
  if (b >= G32) return;
  const bool valid = b < A.Nb;
  A.rho[b] = valid ? rho_in[b] : R(1);
  A.sw[b] = (valid && sw_in) ? sw_in[b] : R(0);
  A.act[b] = valid ? 1 : 0;
  A.iters[b] = max_iter;
  A.status[b] = 0;
  A.fstat[b] = 0;
  A.chg[b] = 0;
  if (b == 0) A.gate[0] = 0;
}

// ---------------------------------------------------------------------------
// Theta_t (lower, packed) and Phi_t of one problem at its rho, written into
// the interleaved operator (the factor's input format), one CTA per problem,
// with the assembly arithmetic of assemble.cuh.
// ---------------------------------------------------------------------------
template <typename R>
struct IlOpAcc {
  R* ops;
  int b, T, n;
  size_t E;
  __device__ void set_theta(int t, int i, int j, R v) const {  // i <= j: lower element (j, i)
    if (i < n && j < n) ops[ix(b, E, (size_t)t * tri(n) + LI(j, i))] = v;
  }
  __device__ void set_phi(int t, int i, int j, R v) const {
    if (i < n && j < n) ops[ix(b, E, (size_t)T * tri(n) + ((size_t)t * n + i) * n + j)] = v;
  }
};

template <int NB, typename R>
__global__ void __launch_bounds__(128) il_assemble_kernel(IlArgs<R> A, TmpcQP qp, const int* gate) {
  if (gate && *gate == 0) return;
  const int b = blockIdx.x;
  const QPView<R> v = qp_view<R>(qp, b, A.T, A.n, A.nx, A.n0, A.m);
  const R rho = A.rho[b];
  const IlOpAcc<R> acc{A.ops, b, A.T, A.n, op_elems(A.T, A.n)};
  assemble_theta_phi<NB>(acc, v, rho * A.rff, rho, A.sigma, A.T, A.n, A.nx, A.n0, A.m);
}

// ---------------------------------------------------------------------------
// gamma from the current state (compute_gamma's formula and order), one
// thread per (problem, stage).  Also ORs the last factor's status bits into
// the problem's status.  With chg, only problems whose rho just changed.
// ---------------------------------------------------------------------------
template <typename R>
__global__ void __launch_bounds__(kWarp) il_gamma_kernel(IlArgs<R> A, const int* gate, int use_chg) {
  if (gate && *gate == 0) return;
  const int lane = threadIdx.x, t = blockIdx.y;
  const int b = blockIdx.x * kWarp + lane;
  if (b >= A.Nb) return;
  if (t == 0) {
    A.status[b] |= A.fstat[b];
  }
  if (use_chg && !A.chg[b]) return;
  const int T = A.T, N = T - 1, n = A.n, nx = A.nx, n0 = A.n0, m = A.m;
  const IlSizes z(T, n, nx, n0, m);
  const R rho = A.rho[b], rf = rho * A.rff;
  auto ctd = [&](int k) {  // rho_f c - y_f, dynamics row k = t nx + i
    return rf * A.c[ix(b, z.c, k)] - A.yfd[ix(b, z.yfd, k)];
  };
  for (int j = 0; j < n; ++j) {
    R val = A.sigma * A.x[ix(b, z.x, (size_t)t * n + j)] - A.q[ix(b, z.q, (size_t)t * n + j)];
    R eq = R(0);
    if (t == 0) {
      for (int k = 0; k < n0; ++k)
        eq += A.a0[ix(b, z.a0, (size_t)k * n + j)] * (rf * A.c0[ix(b, z.c0, k)] - A.yf0[ix(b, z.yf0, k)]);
      if (N > 0)
        for (int k = 0; k < nx; ++k) eq += A.am[ix(b, z.am, (size_t)k * n + j)] * ctd(k);
    } else {
      for (int k = 0; k < nx; ++k)
        eq += A.ap[ix(b, z.am, ((size_t)(t - 1) * nx + k) * n + j)] * ctd((t - 1) * nx + k);
      if (t < N)
        for (int k = 0; k < nx; ++k) eq += A.am[ix(b, z.am, ((size_t)t * nx + k) * n + j)] * ctd(t * nx + k);
    }
    val += eq;
    R iq = R(0);
    for (int k = 0; k < m; ++k)
      iq += A.g[ix(b, z.g, ((size_t)t * m + k) * n + j)] *
            (rho * A.zg[ix(b, z.zm, (size_t)t * m + k)] - A.yg[ix(b, z.zm, (size_t)t * m + k)]);
    val += iq;
    A.gam[ix(b, z.x, (size_t)t * n + j)] = val;
  }
}

// Resets the per-problem rho-change flags after the gamma pass that used them.
__global__ void il_clear_chg_kernel(int* chg, int G32, int* gate) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < G32) chg[b] = 0;
  if (b == 0) gate[0] = 0;
}

// ---------------------------------------------------------------------------
// The ADMM iterations [it0, it1) of one group of 32 problems.
// ---------------------------------------------------------------------------
// Stage buffer sizes (elements per problem).
__host__ __device__ inline int il_fwd_elems(int n) { return (int)(tri(n) + (size_t)n * n + n); }
__host__ __device__ inline int il_qp_elems(int n, int nx, int m) { return 2 * nx * n + m * n + 2 * n + 2 * nx + 4 * m; }
__host__ __device__ inline int il_buf_b_elems(int n, int nx, int m) {
  const int a = il_fwd_elems(n), q = il_qp_elems(n, nx, m);
  return a > q ? a : q;
}
// Dynamic shared memory: buffer A, buffer B, then the vectors
// ush[NB], xs0[NB], xs1[NB], ctv[nx], gtv[m], ct0v[n0] (each x 32 lanes).
template <int NB, typename R>
size_t il_admm_smem(int n, int nx, int n0, int m) {
  const size_t e = (size_t)il_fwd_elems(n) + il_buf_b_elems(n, nx, m) + 3 * NB + nx + m + n0;
  return e * kWarp * sizeof(R);
}

template <int NB, typename R>
__global__ void __launch_bounds__(kIlThreads, 1) il_admm_kernel(const IlArgs<R> A, int it0, int it1) {
  constexpr int NW = kIlWarps;
  constexpr int RPT = (NB + NW - 1) / NW;  // rows of a stage per thread
  constexpr int V = 16 / sizeof(R);
  extern __shared__ __align__(16) unsigned char il_smem[];
  const int lane = threadIdx.x & (kWarp - 1), w = threadIdx.x / kWarp;
  const int grp = blockIdx.x;
  const int b = grp * kWarp + lane;
  const int T = A.T, N = T - 1, n = A.n, nx = A.nx, n0 = A.n0, m = A.m;
  const bool act = b < A.Nb && A.act[b] != 0;
  if (!__syncthreads_or(act)) return;  // every problem of the group has converged
  const IlSizes z(T, n, nx, n0, m);
  const size_t trin = tri(n), nn = (size_t)n * n, woff = (size_t)T * trin;
  const R rho = A.rho[b], rf = rho * A.rff, al = A.alpha, sw = A.sw[b];
  const bool slack = A.use_slack != 0;
  // group bases of the interleaved arrays (element e, lane: base[e * 32 + lane])
  auto gb = [&](R* p, size_t E) { return p + (size_t)grp * E * kWarp; };
  R* F = gb(A.ops, z.ops);
  R* Q = gb(A.q, z.q);
  R* AM = gb(A.am, z.am);
  R* AP = gb(A.ap, z.am);
  R* Gm = m > 0 ? gb(A.g, z.g) : nullptr;
  R* CC = gb(A.c, z.c);
  R* LL = m > 0 ? gb(A.l, z.lu) : nullptr;
  R* UU = m > 0 ? gb(A.u, z.lu) : nullptr;
  R* X = gb(A.x, z.x);
  R* YFD = gb(A.yfd, z.yfd);
  R* ZG = m > 0 ? gb(A.zg, z.zm) : nullptr;
  R* YG = m > 0 ? gb(A.yg, z.zm) : nullptr;
  R* XIG = m > 0 ? gb(A.xig, z.zm) : nullptr;
  R* GAM = gb(A.gam, z.x);
  R* YS = gb(A.ys, z.x);
  R* sm = reinterpret_cast<R*>(il_smem);
  const int SA = il_fwd_elems(n), SB = il_buf_b_elems(n, nx, m);
  R* BA = sm;
  R* BB = sm + (size_t)SA * kWarp;
  R* ush = BB + (size_t)SB * kWarp;
  R* xs0 = ush + NB * kWarp;
  R* xs1 = xs0 + NB * kWarp;
  R* ctv = xs1 + NB * kWarp;
  R* gtv = ctv + (size_t)nx * kWarp;
  R* ct0v = gtv + (size_t)m * kWarp;
  auto S = [&](R* p, int e) -> R& { return p[(size_t)e * kWarp + lane]; };  // shared / group element e of this lane
  // copy `elems` interleaved elements from src (group base + e0 * 32) to dst, 16 bytes per cp.async
  auto copy = [&](R* dst, const R* src, int elems) {
    const int chunks = elems * kWarp / V;
    for (int c = threadIdx.x; c < chunks; c += kIlThreads) cp_async16(dst + c * V, src + c * V);
  };
  // buffer B (backward) offsets
  const int oAm = 0, oAp = nx * n, oG = 2 * nx * n, oq = oG + m * n, oc = oq + n, ox = oc + nx, oyf = ox + n,
            ozg = oyf + nx, oyg = ozg + m, ol = oyg + m, ou = ol + m;
  auto fetch_fwd = [&](R* dst, int t) {
    copy(dst, F + (size_t)t * trin * kWarp, (int)trin);
    if (t > 0) copy(dst + trin * kWarp, F + (woff + (size_t)(t - 1) * nn) * kWarp, (int)nn);
    copy(dst + (trin + nn) * kWarp, GAM + (size_t)t * n * kWarp, n);
  };
  auto fetch_bwd_a = [&](int t) {
    copy(BA, F + (size_t)t * trin * kWarp, (int)trin);
    if (t < N) copy(BA + trin * kWarp, F + (woff + (size_t)t * nn) * kWarp, (int)nn);
    copy(BA + (trin + nn) * kWarp, YS + (size_t)t * n * kWarp, n);
  };
  auto fetch_bwd_b = [&](int t) {
    if (t < N) {
      copy(BB + (size_t)oAm * kWarp, AM + (size_t)t * nx * n * kWarp, nx * n);
      copy(BB + (size_t)oAp * kWarp, AP + (size_t)t * nx * n * kWarp, nx * n);
      copy(BB + (size_t)oc * kWarp, CC + (size_t)t * nx * kWarp, nx);
      copy(BB + (size_t)oyf * kWarp, YFD + (size_t)t * nx * kWarp, nx);
    }
    if (m > 0) {
      copy(BB + (size_t)oG * kWarp, Gm + (size_t)t * m * n * kWarp, m * n);
      copy(BB + (size_t)ozg * kWarp, ZG + (size_t)t * m * kWarp, m);
      copy(BB + (size_t)oyg * kWarp, YG + (size_t)t * m * kWarp, m);
      copy(BB + (size_t)ol * kWarp, LL + (size_t)t * m * kWarp, m);
      copy(BB + (size_t)ou * kWarp, UU + (size_t)t * m * kWarp, m);
    }
    copy(BB + (size_t)oq * kWarp, Q + (size_t)t * n * kWarp, n);
    copy(BB + (size_t)ox * kWarp, X + (size_t)t * n * kWarp, n);
  };

  for (int it = it0; it < it1; ++it) {
    // ---------------- forward sweep: y_t = L_t^-1 (gamma_t - W_{t-1} y_{t-1})
    fetch_fwd(BA, 0);
    cp_async_commit();
    fetch_fwd(BB, 1);
    cp_async_commit();
    for (int t = 0; t < T; ++t) {
      R* buf = (t & 1) ? BB : BA;
      cp_async_wait<1>();
      __syncthreads();
      R* Wb = buf + trin * kWarp;
      R* gb_ = buf + (trin + nn) * kWarp;
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        if (i < n) {
          R u = S(gb_, i);
          if (t > 0)
            for (int k = 0; k < n; ++k) u = fma(-S(Wb, i * n + k), S(xs0, k), u);
          S(ush, i) = u;
        }
      }
      __syncthreads();
      R y[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        R acc = R(0);
        if (i < n) {
          for (int c = 0; c <= i; ++c) acc = fma(S(buf, LI(i, c)), S(ush, c), acc);
          if (act) S(YS, t * n + i) = acc;
        }
        y[r] = acc;
      }
      __syncthreads();  // every read of this stage's buffer, ush and xs0 is done
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int i = w + NW * r;
        if (i < n) S(xs0, i) = y[r];
      }
      if (t + 2 < T) fetch_fwd(buf, t + 2);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---------------- backward sweep with the ADMM-level updates
    // x~_{t+1} in xs[(t + 1) & 1], x~_t into xs[t & 1]; gamma_t's pieces of
    // step t wait in registers for the A+ terms of step t - 1.
    R gval[RPT], gam_[RPT], giq[RPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r) {
      gval[r] = gam_[r] = giq[r] = R(0);
      const int i = w + NW * r;
      if (i < n) S((N & 1) ? xs0 : xs1, i) = R(0);  // x~_T = 0 (slot of t = N + 1)
    }
    fetch_bwd_a(N);
    cp_async_commit();
    fetch_bwd_b(N);
    cp_async_commit();
    for (int t = N; t >= 0; --t) {
      R* xt = (t & 1) ? xs1 : xs0;   // x~_t
      R* xn = (t & 1) ? xs0 : xs1;   // x~_{t+1}
      cp_async_wait<1>();
      __syncthreads();
      R* Wb = BA + trin * kWarp;
      R* yb = BA + (trin + nn) * kWarp;
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int k = w + NW * r;
        if (k < n) {
          R u = S(yb, k);
          if (t < N)
            for (int i = 0; i < n; ++i) u = fma(-S(Wb, i * n + k), S(xn, i), u);
          S(ush, k) = u;
        }
      }
      __syncthreads();
      R xv[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int k = w + NW * r;
        R acc = R(0);
        if (k < n) {
          for (int i = k; i < n; ++i) acc = fma(S(BA, LI(i, k)), S(ush, i), acc);
          S(xt, k) = acc;
        }
        xv[r] = acc;
      }
      cp_async_wait<0>();
      __syncthreads();  // x~_t complete, buffer B of stage t landed, buffer A consumed
      if (t > 0) fetch_bwd_a(t - 1);
      cp_async_commit();
      // dynamics rows of stage t: C x~ = Am_t x~_t + Ap_t x~_{t+1}
      if (t < N) {
        for (int r = w; r < nx; r += NW) {
          R s1 = R(0), s2 = R(0);
          for (int j = 0; j < n; ++j) s1 = fma(S(BB, oAm + r * n + j), S(xt, j), s1);
          for (int j = 0; j < n; ++j) s2 = fma(S(BB, oAp + r * n + j), S(xn, j), s2);
          const R cx = s1 + s2;
          const R cr = S(BB, oc + r);
          const R y = S(BB, oyf + r) + rf * al * (cx - cr);
          if (act) S(YFD, t * nx + r) = y;
          S(ctv, r) = rf * cr - y;
        }
      }
      // inequality rows of stage t
      for (int k = w; k < m; k += NW) {
        R gx = R(0);
        for (int j = 0; j < n; ++j) gx = fma(S(BB, oG + k * n + j), S(xt, j), gx);
        const R zold = S(BB, ozg + k), ygo = S(BB, oyg + k);
        const R zt = al * gx + (R(1) - al) * zold + ygo / rho;
        R cl = zt;
        const R lb = S(BB, ol + k), ub = S(BB, ou + k);
        if (cl < lb) cl = lb;
        if (cl > ub) cl = ub;
        R znew;
        if (slack) {
          const R f = sw / (sw + rho);
          znew = (R(1) - f) * zt + f * cl;
          if (act) S(XIG, t * m + k) = (rho / (sw + rho)) * (cl - zt);
        } else {
          znew = cl;
        }
        const R ygn = ygo + rho * (al * gx + (R(1) - al) * zold - znew);
        if (act) {
          S(ZG, t * m + k) = znew;
          S(YG, t * m + k) = ygn;
        }
        S(gtv, k) = rho * znew - ygn;
      }
      // initial-condition rows (stage 0)
      if (t == 0) {
        for (int k = w; k < n0; k += NW) {
          R s = R(0);
          for (int j = 0; j < n; ++j) s = fma(A.a0[ix(b, z.a0, (size_t)k * n + j)], S(xt, j), s);
          const R c0 = A.c0[ix(b, z.c0, k)];
          const R y = A.yf0[ix(b, z.yf0, k)] + rf * al * (s - c0);
          if (act) A.yf0[ix(b, z.yf0, k)] = y;
          S(ct0v, k) = rf * c0 - y;
        }
      }
      // relaxation of x_t
      R xr[RPT];
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int j = w + NW * r;
        xr[r] = R(0);
        if (j < n) {
          xr[r] = al * xv[r] + (R(1) - al) * S(BB, ox + j);
          if (act) S(X, t * n + j) = xr[r];
        }
      }
      __syncthreads();  // ctv, gtv, ct0v complete
      // gamma for the next iteration
#pragma unroll
      for (int r = 0; r < RPT; ++r) {
        const int j = w + NW * r;
        if (j >= n) continue;
        // A+ terms of the dynamics rows of stage t complete gamma_{t+1}
        if (t < N) {
          R ap = R(0);
          for (int k = 0; k < nx; ++k) ap += S(BB, oAp + k * n + j) * S(ctv, k);
          if (act) S(GAM, (t + 1) * n + j) = (gval[r] + (ap + gam_[r])) + giq[r];
        }
        R val = A.sigma * xr[r] - S(BB, oq + j);
        R eq = R(0);
        if (t == 0) {
          for (int k = 0; k < n0; ++k) eq += A.a0[ix(b, z.a0, (size_t)k * n + j)] * S(ct0v, k);
        }
        if (t < N) {
          for (int k = 0; k < nx; ++k) eq += S(BB, oAm + k * n + j) * S(ctv, k);
        }
        R iq = R(0);
        for (int k = 0; k < m; ++k) iq += S(BB, oG + k * n + j) * S(gtv, k);
        if (t == 0) {
          if (act) S(GAM, j) = (val + eq) + iq;
        } else {
          gval[r] = val;
          gam_[r] = eq;
          giq[r] = iq;
        }
      }
      __syncthreads();  // buffer B, ctv, gtv consumed
      if (t > 0) fetch_bwd_b(t - 1);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Residual check at iteration `it` (admm_check's rule), one CTA per active
// problem: the state comes from the interleaved arrays, the QP from the
// caller's problem-major arrays.  Converged: iteration count stored and the
// problem deactivated.  New rho: stored, the problem flagged and the gate
// opened for the re-factor.
// ---------------------------------------------------------------------------
template <int NB, typename R>
__global__ void __launch_bounds__(128) il_check_kernel(IlArgs<R> A, TmpcQP qp, int it, int adapt_every, R eps_abs,
                                                       R eps_rel, R adapt_tol, R rho_min, R rho_max) {
  using Gm = Geo<NB, R>;
  const int b = blockIdx.x;
  if (!A.act[b]) return;
  const int T = A.T, N = T - 1, n = A.n, nx = A.nx, n0 = A.n0, m = A.m;
  const IlSizes z(T, n, nx, n0, m);
  extern __shared__ __align__(16) unsigned char ck_smem[];
  R* x = reinterpret_cast<R*>(ck_smem);
  auto a4 = [](size_t v) { return (v + 3) & ~size_t(3); };
  size_t o = a4((size_t)T * Gm::VSTR);
  R* zg = x + o; o = a4(o + (size_t)T * m);
  R* yg = x + o; o = a4(o + (size_t)T * m);
  R* xig = x + o; o = a4(o + (size_t)T * m);
  R* yf0 = x + o; o = a4(o + n0);
  R* yfd = x + o; o = a4(o + (size_t)N * nx);
  R* red = x + o;
  for (int e = threadIdx.x; e < T * Gm::VSTR; e += blockDim.x) {
    const int t = e / Gm::VSTR, j = e - t * Gm::VSTR;
    x[e] = j < n ? A.x[ix(b, z.x, (size_t)t * n + j)] : R(0);
  }
  for (int e = threadIdx.x; e < T * m; e += blockDim.x) {
    zg[e] = A.zg[ix(b, z.zm, e)];
    yg[e] = A.yg[ix(b, z.zm, e)];
    xig[e] = A.xig[ix(b, z.zm, e)];
  }
  for (int e = threadIdx.x; e < n0; e += blockDim.x) yf0[e] = A.yf0[ix(b, z.yf0, e)];
  for (int e = threadIdx.x; e < N * nx; e += blockDim.x) yfd[e] = A.yfd[ix(b, z.yfd, e)];
  __syncthreads();
  const QPView<R> v = qp_view<R>(qp, b, T, n, nx, n0, m);
  R* sc = red + kRedSc;
  const R sw = A.sw[b];
  compute_residuals<NB>(sc, red, x, zg, yg, xig, yf0, yfd, v, sw, A.use_slack != 0, T, n, nx, n0, m);
  if (threadIdx.x != 0) return;
  const bool conv = (sc[0] < eps_abs + eps_rel * sc[4]) && (sc[1] < eps_abs + eps_rel * sc[5]);
  if (conv) {
    A.iters[b] = it + 1;
    A.act[b] = 0;
    return;
  }
  if (adapt_every > 0 && it >= 2 && (it % adapt_every) == 0) {
    const R rho = A.rho[b];
    R cand = rho * sqrt(sc[2] / (sc[3] + R(1e-30)));
    if (cand < rho_min) cand = rho_min;
    if (cand > rho_max) cand = rho_max;
    R ratio = cand / rho;
    if (ratio < R(1)) ratio = R(1) / ratio;
    if (ratio >= adapt_tol) {
      A.rho[b] = cand;
      A.chg[b] = 1;
      atomicOr(A.gate, 1);
    }
  }
}

template <int NB, typename R>
size_t il_check_smem(int T, int nx, int n0, int m) {
  using Gm = Geo<NB, R>;
  auto a4 = [](size_t v) { return (v + 3) & ~size_t(3); };
  const size_t N = T - 1;
  size_t o = a4((size_t)T * Gm::VSTR);
  o = a4(o + (size_t)T * m);
  o = a4(o + (size_t)T * m);
  o = a4(o + (size_t)T * m);
  o = a4(o + n0);
  o = a4(o + N * nx);
  return (o + kRedSize) * sizeof(R);
}

// Scalars out: rho, iteration count, status (factor bits, non-finite x).
template <typename R>
__global__ void il_scalars_out_kernel(IlArgs<R> A, R* rho_out, uint32_t* iters_out, int32_t* status_out) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= A.Nb) return;
  const IlSizes z(A.T, A.n, A.nx, A.n0, A.m);
  bool nonfinite = false;
  for (size_t e = 0; e < z.x; ++e)
    if (!isfinite(A.x[ix(b, z.x, e)])) nonfinite = true;
  rho_out[b] = A.rho[b];
  if (iters_out) iters_out[b] = (uint32_t)A.iters[b];
  if (status_out) status_out[b] = A.status[b] | (nonfinite ? TMPC_STATUS_NONFINITE : 0);
}

template <int NB, typename R>
bool il_fits(const TmpcDims& d) {
  if (d.n > max_nb<R>() || d.Nb <= 0 || !grid_ok(d.Nb, op_elems(d.T, d.n))) return false;
  if ((long)il_admm_smem<NB, R>(d.n, d.nx, d.n0, d.m) > max_dyn_smem()) return false;
  if ((long)il_check_smem<NB, R>(d.T, d.nx, d.n0, d.m) > max_dyn_smem()) return false;
  return (long)staged_smem_elems<R>(d.n, false) * (long)sizeof(R) <= max_dyn_smem();
}

template <typename R, class F>
int il_dispatch(int n, F&& f) {
  if (n <= 8) return f(std::integral_constant<int, 8>{});
  if (n <= 12) return f(std::integral_constant<int, 12>{});
  if constexpr (max_nb<R>() >= 16) {
    if (n <= 16) return f(std::integral_constant<int, 16>{});
  }
  return TMPC_ERR_UNSUPPORTED;
}

}  // namespace il

// Workspace of the interleaved direct path, 0 when it does not apply.
template <typename R>
size_t admm_il_ws_bytes(const TmpcDims& d) {
  if (d.n > il::max_nb<R>() || d.Nb <= 0) return 0;
  bool ok = false;
  il::il_dispatch<R>(d.n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    ok = il::il_fits<NB, R>(d);
    return 0;
  });
  return ok ? il::IlWs<R>(d.Nb, d.T, d.n, d.nx, d.n0, d.m).bytes : 0;
}

template <typename R>
int launch_admm_direct_il(const AdmmParams<R>& P, size_t ws_bytes, cudaStream_t st) {
  using namespace il;
  TmpcDims d{};
  d.Nb = P.Nb; d.T = P.T; d.n = P.n; d.nx = P.nx; d.n0 = P.n0; d.m = P.m;
  const size_t need = admm_il_ws_bytes<R>(d);
  if (need == 0) return TMPC_ERR_UNSUPPORTED;
  if (P.ws == nullptr || ws_bytes < need || (reinterpret_cast<uintptr_t>(P.ws) & 255) != 0) return TMPC_ERR_WORKSPACE;
  const IlArgs<R> A = il_args<R>(P.ws, P);
  const int T = P.T, N = T - 1, n = P.n, nx = P.nx, n0 = P.n0, m = P.m, Nb = P.Nb;
  const IlSizes z(T, n, nx, n0, m);
  const int G32 = (int)(groups(Nb) * kWarp);
  int rc = TMPC_OK;
  auto chk = [&](int r) {
    if (rc == TMPC_OK && r != TMPC_OK) rc = r;
  };
  auto inl = [&](const void* src, R* dst, size_t E) {
    if (E == 0 || src == nullptr) return;
    chk(interleave<R>(Nb, E, E, static_cast<const R*>(src), dst, IdentityMap{}, st));
  };
  // ---- inputs
  il_scalars_in_kernel<R><<<(G32 + 255) / 256, 256, 0, st>>>(A, static_cast<const R*>(P.in.rho_bar),
                                                             P.slack_weight, P.max_iter);
  chk((int)cudaPeekAtLastError());
  inl(P.qp.q, A.q, z.q);
  inl(P.qp.A0, A.a0, z.a0);
  inl(P.qp.A_minus, A.am, z.am);
  inl(P.qp.A_plus, A.ap, z.am);
  inl(P.qp.G, A.g, z.g);
  inl(P.qp.c0, A.c0, z.c0);
  inl(P.qp.c, A.c, z.c);
  inl(P.qp.l, A.l, z.lu);
  inl(P.qp.u, A.u, z.lu);
  inl(P.in.x, A.x, z.x);
  inl(P.in.y_f0, A.yf0, z.yf0);
  inl(P.in.y_fdyn, A.yfd, z.yfd);
  inl(P.in.z_g, A.zg, z.zm);
  inl(P.in.y_g, A.yg, z.zm);
  inl(P.in.xi_g, A.xig, z.zm);
  if (rc) return rc;
  return il_dispatch<R>(n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    const size_t smem = il_admm_smem<NB, R>(n, nx, n0, m);
    const size_t csmem = il_check_smem<NB, R>(T, nx, n0, m);
    chk((int)cudaFuncSetAttribute(il_admm_kernel<NB, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    chk((int)cudaFuncSetAttribute(il_check_kernel<NB, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem));
    if (rc) return rc;
    const dim3 ggrid((unsigned)groups(Nb), (unsigned)T);
    // operator, factor (in place) and the first gamma; with `gate`, only
    // when a check opened it, gamma only for the flagged problems
    auto build = [&](const int* gate) {
      il_assemble_kernel<NB, R><<<Nb, 128, 0, st>>>(A, P.qp, gate);
      chk((int)cudaPeekAtLastError());
      chk(launch_factor<NB, R>(Nb, T, n, A.ops, A.ops, A.fstat, gate, st));
      il_gamma_kernel<R><<<ggrid, kWarp, 0, st>>>(A, gate, gate ? 1 : 0);
      chk((int)cudaPeekAtLastError());
      if (gate) {
        il_clear_chg_kernel<<<(G32 + 255) / 256, 256, 0, st>>>(A.chg, G32, A.gate);
        chk((int)cudaPeekAtLastError());
      }
    };
    auto iterate = [&](int a, int e) {
      if (e <= a) return;
      il_admm_kernel<NB, R><<<(unsigned)groups(Nb), kIlThreads, smem, st>>>(A, a, e);
      chk((int)cudaPeekAtLastError());
    };
    build(nullptr);
    const int ce = P.check_every;
    if (ce <= 0) {
      iterate(0, P.max_iter);
    } else {
      int it = 0;
      while (it < P.max_iter && rc == TMPC_OK) {
        const int c = ((it + ce - 1) / ce) * ce;  // next checked iteration >= it
        if (c >= P.max_iter) {
          iterate(it, P.max_iter);
          break;
        }
        iterate(it, c + 1);
        il_check_kernel<NB, R><<<Nb, 128, csmem, st>>>(A, P.qp, c, P.adapt_every, P.eps_abs, P.eps_rel, P.adapt_tol,
                                                      P.rho_min, P.rho_max);
        chk((int)cudaPeekAtLastError());
        if (P.adapt_every > 0 && c >= 2 && (c % P.adapt_every) == 0) build(A.gate);
        it = c + 1;
      }
    }
    // ---- outputs
    chk(deinterleave<R>(Nb, z.x, A.x, static_cast<R*>(P.out.x), st));
    if (P.x_out) chk(deinterleave<R>(Nb, z.x, A.x, P.x_out, st));
    if (n0 > 0) chk(deinterleave<R>(Nb, z.yf0, A.yf0, static_cast<R*>(P.out.y_f0), st));
    chk(deinterleave<R>(Nb, z.yfd, A.yfd, static_cast<R*>(P.out.y_fdyn), st));
    if (m > 0) {
      chk(deinterleave<R>(Nb, z.zm, A.zg, static_cast<R*>(P.out.z_g), st));
      chk(deinterleave<R>(Nb, z.zm, A.yg, static_cast<R*>(P.out.y_g), st));
      chk(deinterleave<R>(Nb, z.zm, A.xig, static_cast<R*>(P.out.xi_g), st));
    }
    il_scalars_out_kernel<R><<<(Nb + 255) / 256, 256, 0, st>>>(A, static_cast<R*>(P.out.rho_bar), P.iters_out,
                                                               P.status_out);
    chk((int)cudaPeekAtLastError());
    (void)N;
    return rc;
  });
}

template size_t admm_il_ws_bytes<float>(const TmpcDims&);
template size_t admm_il_ws_bytes<double>(const TmpcDims&);
template int launch_admm_direct_il<float>(const AdmmParams<float>&, size_t, cudaStream_t);
template int launch_admm_direct_il<double>(const AdmmParams<double>&, size_t, cudaStream_t);

}  // namespace tmpc
