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
#include <mutex>
#include <vector>

#include "admm_kernel.cuh"
#include "riccati_il.cuh"

namespace tmpc {
namespace il {

constexpr int kIlWarps = 16;  // one warp per stage row (NB <= 16)
constexpr int kIlThreads = 32 * kIlWarps;
constexpr int kIlCmpWarps = 8;  // compact variant: two stage rows per warp, two blocks per SM

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
  size_t act, iters, status, fstat, chg, apid, gsel, gcol, wrow, gate;                   // int offsets
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
    apid = io; io += groups(Nb);
    gsel = io; io += groups(Nb);
    gcol = io; io += groups(Nb) * (size_t)(m > 0 ? m : 1);
    wrow = io; io += groups(Nb);
    gate = io; io += 4;
    bytes = rbytes + io * sizeof(int);
  }
};

// Pointers and parameters of the interleaved kernels.
template <typename R>
struct IlArgs {
  R *ops, *q, *a0, *am, *ap, *g, *c0, *c, *l, *u, *x, *yf0, *yfd, *zg, *yg, *xig, *gam, *ys, *rho, *sw;
  int *act, *iters, *status, *fstat, *chg, *apid, *gsel, *gcol, *wrow, *gate;
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
  a.apid = i + L.apid;
  a.gsel = i + L.gsel;
  a.gcol = i + L.gcol;
  a.wrow = i + L.wrow;
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
  if ((b & (kWarp - 1)) == 0) {  // per-group structure flags, cleared by the checks on a mismatch
    A.apid[b / kWarp] = 1;
    A.gsel[b / kWarp] = 1;
  }
  if (b == 0) A.gate[0] = 0;
}

// ---------------------------------------------------------------------------
// Structure of A+: the explicit integrators give A+_t = [-I 0] for every
// stage (turbompc/problems/optimal_control_problem.py:1256-1271).  One pass
// over the caller's problem-major array (a block per problem, a thread per
// row) checks every problem's A+ exactly, before any layout conversion; where all 32 problems of a group
// match, the group's A+ is not
// converted to the interleaved layout and the assembly, the first gamma and
// the iteration kernel form its products from the identity (bit-identical:
// the products with the exact -1 and 0 entries are exact).
// ---------------------------------------------------------------------------
constexpr int kFlatThreads = 256;

// Whether a row of n values equals `one` at column c and 0 elsewhere (128-bit
// loads when the row is 16-byte aligned and n a multiple of the vector width).
template <typename R>
__device__ __forceinline__ bool row_is_unit(const R* row, int n, int c, R one) {
  constexpr int V = 16 / sizeof(R);
  int bad = 0;  // no short-circuit: the loads stay independent
  if (n % V == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    for (int j = 0; j < n; j += V) {
      R w[V];
      ld128(w, row + j);
#pragma unroll
      for (int v = 0; v < V; ++v) bad |= w[v] != (j + v == c ? one : R(0));
    }
  } else {
    for (int j = 0; j < n; ++j) bad |= row[j] != (j == c ? one : R(0));
  }
  return bad == 0;
}

template <typename R>
__global__ void __launch_bounds__(kFlatThreads) il_ap_identity_kernel(IlArgs<R> A, const R* __restrict__ ap_pm) {
  // one block per problem, one thread per row (t, k) of its A+ (the rows of a
  // warp are one contiguous run): row k of A+_t must be -e_k.  apid[grp] was
  // set to 1 by il_scalars_in_kernel and is cleared (plain stores of 0) on a
  // mismatch
  const int b = blockIdx.x, n = A.n, nx = A.nx, rows = (A.T - 1) * nx;
  const R* P = ap_pm + (size_t)b * rows * n;
  bool ok = true;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) ok &= row_is_unit(P + (size_t)r * n, n, r % nx, R(-1));
  if (!__syncthreads_and(ok) && threadIdx.x == 0) A.apid[b / kWarp] = 0;
}

// ---------------------------------------------------------------------------
// Structure of G: box constraints on single variables (the quadrotor's thrust
// bounds) make every inequality row a unit vector, G_t[k] = e_{c_k}, with the
// same columns c_k in every stage.  One thread per (group, row) takes the
// columns from the group's first problem's first stage, then one pass over
// the caller's problem-major array (a block per problem, a thread per row)
// checks every row exactly; where
// all 32 problems of a group match, the group's G is not
// converted to the interleaved layout and the assembly, the first gamma and
// the iteration kernel form G x and G^T y from the columns (the same sums:
// the other terms are exact zeros).
// ---------------------------------------------------------------------------
template <typename R>
__global__ void __launch_bounds__(kFlatThreads) il_g_columns_kernel(IlArgs<R> A, const R* __restrict__ g_pm) {
  // thread per (group, row k): the column of the single 1 in row k of the
  // group's first problem, first stage (the last 1 of the row; -1 if none)
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = A.m, n = A.n;
  if (i >= (int)groups(A.Nb) * m) return;
  const int grp = i / m, k = i - grp * m;
  const R* row = g_pm + (size_t)grp * kWarp * A.T * m * n + (size_t)k * n;
  int c = -1;
  for (int j = 0; j < n; ++j)
    if (row[j] == R(1)) c = j;
  A.gcol[i] = c;
  if (c < 0) A.gsel[grp] = 0;
}

template <typename R>
__global__ void __launch_bounds__(kFlatThreads) il_g_select_kernel(IlArgs<R> A, const R* __restrict__ g_pm) {
  // one block per problem, one thread per row (t, k) of its G: row k of every
  // stage must equal e_{gcol[k]}; gsel[grp] is cleared (plain stores of 0)
  // on a mismatch
  const int b = blockIdx.x, n = A.n, m = A.m, rows = A.T * m;
  const int* gc = A.gcol + (size_t)(b / kWarp) * m;
  const R* P = g_pm + (size_t)b * rows * n;
  bool ok = true;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) ok &= row_is_unit(P + (size_t)r * n, n, gc[r % m], R(1));
  if (!__syncthreads_and(ok) && threadIdx.x == 0) A.gsel[b / kWarp] = 0;
}

// ---------------------------------------------------------------------------
// Rows of the factor's off-diagonal blocks W_t = Phi_t L_t^-T that are exact
// zeros.  Phi_t = E_t + rho_f A+_t^T A-_t couples stage t + 1's variables
// (rows) to stage t's (columns); with A+_t = [-I 0] and no control-rate term
// in E_t (the quadrotor's case) its rows nx..n-1 are zero, and so are those
// rows of W_t.  One block per group reads rows nx..n-1 of every W_t of its
// 32 problems (after each factor) and records in wrow[grp] how many leading
// rows the iteration kernel has to read: nx where all the others are exact
// zeros, n otherwise.  Skipping exact-zero products leaves every sum as it
// was, so the iterates do not change.
// ---------------------------------------------------------------------------
constexpr int kWrowThreads = 128;
template <typename R>
__global__ void __launch_bounds__(kWrowThreads) il_w_rows_kernel(IlArgs<R> A, const int* gate) {
  if (gate && *gate == 0) return;
  const int lane = threadIdx.x & (kWarp - 1), w = threadIdx.x / kWarp, grp = blockIdx.x;
  const int b = grp * kWarp + lane;
  const int T = A.T, N = T - 1, n = A.n, nx = A.nx;
  const size_t trin = tri(n), nn = (size_t)n * n;
  const R* F = A.ops + (size_t)grp * op_elems(T, n) * kWarp + lane;
  int bad = nx >= n ? 1 : 0;  // nothing to skip
  if (b < A.Nb && !bad) {
    for (int t = w; t < N; t += kWrowThreads / kWarp) {
      const R* W = F + ((size_t)T * trin + (size_t)t * nn + (size_t)nx * n) * kWarp;
#pragma unroll 8
      for (int e = 0; e < (n - nx) * n; ++e) bad |= W[(size_t)e * kWarp] != R(0);
    }
  }
  const int any = __syncthreads_or(bad);
  if (threadIdx.x == 0) A.wrow[grp] = any ? n : nx;
}

// ---------------------------------------------------------------------------
// Theta_t (lower, packed) and Phi_t at each problem's rho, written into the
// interleaved operator (the factor's input format): a block of four warps per
// (group, stage), lane = problem; warp p forms a quarter of Theta_t's lower
// triangle (a range of its columns, split by entry count: column c takes row c
// of D_t) and a quarter of Phi_t's rows.  The sums of assemble.cuh
// (admm.py:93-101), in the same order, formed as rank-1 updates of register
// accumulators, one row of G / A0 / A- / A+ at a time (each row read once,
// coalesced from the interleaved copies):
//   Theta = ((D + sigma I) + rho_ineq sum_k g_k g_k^T) + rho_f sum_k a_k a_k^T
//   Phi_t = E_t + rho_f sum_k Ap_t[k]^T Am_t[k]
// D and E come from the caller's problem-major arrays (Theta's element (r, c),
// r >= c, takes D[c][r], as the other assembly paths do).
// ---------------------------------------------------------------------------
// A row of n <= NB values of a problem-major array into registers (zero
// beyond n): 128-bit loads when vec (16-byte aligned row, n a multiple of the
// vector width), else scalar loads.
template <int NB, typename R>
__device__ __forceinline__ void il_load_row(R (&dst)[NB], const R* src, int n, bool vec) {
  constexpr int V = 16 / sizeof(R);
  if (vec) {
#pragma unroll
    for (int j = 0; j < NB; j += V) {
      if (j < n) {
        ld128(&dst[j], src + j);
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v) dst[j + v] = R(0);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < NB; ++j) dst[j] = j < n ? src[j] : R(0);
  }
}

// Columns of the lower triangle of a stage block split into kAsmParts parts
// of about equal entry counts: part p covers columns [asm_bound(NB, p),
// asm_bound(NB, p + 1)) (column c holds the NB - c entries (r >= c, c) and
// takes row c of D, so no part reads another's rows of D).
constexpr int kAsmParts = 4;
__host__ __device__ constexpr int asm_cum(int NB, int c) { return c * NB - c * (c - 1) / 2; }  // entries of columns < c
__host__ __device__ constexpr int asm_bound(int NB, int p) {
  if (p <= 0) return 0;
  if (p >= kAsmParts) return NB;
  const int target = p * NB * (NB + 1) / 2 / kAsmParts;
  int best = 0, bd = 1 << 30;
  for (int c = 0; c <= NB; ++c) {
    const int d = asm_cum(NB, c) - target;
    const int ad = d < 0 ? -d : d;
    if (ad < bd) {
      bd = ad;
      best = c;
    }
  }
  return best;
}
// Index of entry (r, c), r >= c, among the entries of the columns [C0, ...).
__host__ __device__ constexpr int asm_idx(int NB, int C0, int r, int c) {
  return asm_cum(NB, c) - asm_cum(NB, C0) + (r - c);
}

// Part P of the stage's Theta columns and Phi rows (one warp; lane = problem).
template <int NB, typename R, int P>
__device__ __forceinline__ void il_assemble_part(const IlArgs<R>& A, const TmpcQP& qp, int grp, int t, int lane) {
  constexpr int C0 = asm_bound(NB, P), C1 = asm_bound(NB, P + 1);
  constexpr int CNT = asm_cum(NB, C1) - asm_cum(NB, C0);
  constexpr int H0 = P * NB / kAsmParts, H1 = (P + 1) * NB / kAsmParts, HR = H1 - H0;  // Phi rows
  const int b = grp * kWarp + lane;
  const int T = A.T, N = T - 1, n = A.n, nx = A.nx, n0 = A.n0, m = A.m;
  const IlSizes z(T, n, nx, n0, m);
  const int trin = (int)tri(n);
  const R rho = A.rho[b], rf = rho * A.rff;
  // A+_t = [-I 0] / unit inequality rows (detected per group): the rank-1
  // terms of those rows are formed from the structure (the same values: every
  // other product is an exact zero) and the rows are not read
  const bool apI = A.apid[grp] != 0, gS = m > 0 && A.gsel[grp] != 0;
  const int* gc = A.gcol + (size_t)grp * (m > 0 ? m : 1);
  auto lv = [&](R* p, size_t E) { return p + (size_t)grp * E * kWarp + lane; };
  R* O = lv(A.ops, z.ops);
  const R* Gl = m > 0 ? lv(A.g, z.g) : nullptr;
  const R* A0l = n0 > 0 ? lv(A.a0, z.a0) : nullptr;
  const R* AMl = lv(A.am, z.am);
  const R* APl = lv(A.ap, z.am);
  const R* D = static_cast<const R*>(qp.D) + ((size_t)b * T + t) * n * n;
  R acc[CNT > 0 ? CNT : 1];
  // rank-1 updates acc += a a^T (columns C0..C1-1) from a row of n values at p (interleaved, stride 32)
  auto rank1 = [&](R (&ac)[CNT > 0 ? CNT : 1], const R* p) {
    R a[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) a[j] = (j >= C0 && j < n) ? p[j * kWarp] : R(0);
#pragma unroll
    for (int c = C0; c < C1; ++c)
#pragma unroll
      for (int r = c; r < NB; ++r) ac[asm_idx(NB, C0, r, c)] = fma(a[c], a[r], ac[asm_idx(NB, C0, r, c)]);
  };
  if (CNT > 0) {
    // ---- Theta_t: (D + sigma I) + rho_ineq G^T G
#pragma unroll
    for (int e = 0; e < CNT; ++e) acc[e] = R(0);
    if (gS) {
      for (int k = 0; k < m; ++k) {
        const int c = gc[k];
#pragma unroll
        for (int r = C0; r < C1; ++r)
          if (r == c) acc[asm_idx(NB, C0, r, r)] = fma(R(1), R(1), acc[asm_idx(NB, C0, r, r)]);
      }
    } else {
      for (int k = 0; k < m; ++k) rank1(acc, Gl + (size_t)(t * m + k) * n * kWarp);
    }
    // Theta's column c takes row c of D_t (D[c][r], r >= c): rows read whole, with
    // 128-bit loads where the rows are 16-byte aligned (a lane's row is one
    // contiguous run in the caller's problem-major array)
    const bool vec = (n * sizeof(R)) % 16 == 0 && (reinterpret_cast<uintptr_t>(D) & 15) == 0;
#pragma unroll
    for (int c = C0; c < C1; ++c) {
      if (c < n) {
        R dr[NB];
        il_load_row<NB>(dr, D + c * n, n, vec);
#pragma unroll
        for (int r = c; r < NB; ++r) {
          if (r < n) {
            R v = dr[r];
            if (r == c) v += A.sigma;
            v += rho * acc[asm_idx(NB, C0, r, c)];
            acc[asm_idx(NB, C0, r, c)] = v;
          }
        }
      }
    }
    // + rho_f A^T A, accumulated apart and added last
    R ac2[CNT > 0 ? CNT : 1];
#pragma unroll
    for (int e = 0; e < CNT; ++e) ac2[e] = R(0);
    if (t == 0) {
      for (int k = 0; k < n0; ++k) rank1(ac2, A0l + (size_t)k * n * kWarp);
      if (N > 0)
        for (int k = 0; k < nx; ++k) rank1(ac2, AMl + (size_t)k * n * kWarp);
    } else {
      if (apI) {
#pragma unroll
        for (int r = C0; r < C1; ++r)
          if (r < nx) ac2[asm_idx(NB, C0, r, r)] = fma(R(-1), R(-1), ac2[asm_idx(NB, C0, r, r)]);
      } else {
        for (int k = 0; k < nx; ++k) rank1(ac2, APl + (size_t)((t - 1) * nx + k) * n * kWarp);
      }
      if (t < N)
        for (int k = 0; k < nx; ++k) rank1(ac2, AMl + (size_t)(t * nx + k) * n * kWarp);
    }
#pragma unroll
    for (int c = C0; c < C1; ++c)
#pragma unroll
      for (int r = c; r < NB; ++r)
        if (r < n) O[(size_t)(t * trin + LI(r, c)) * kWarp] = acc[asm_idx(NB, C0, r, c)] + rf * ac2[asm_idx(NB, C0, r, c)];
  }
  if (t >= N || HR <= 0) return;
  // ---- Phi_t = E_t + rho_f Ap_t^T Am_t, rows [H0, H1)
  const R* E = static_cast<const R*>(qp.E) + ((size_t)b * N + t) * n * n;
  R ph[HR > 0 ? HR * NB : 1];
#pragma unroll
  for (int e = 0; e < HR * NB; ++e) ph[e] = R(0);
  if (apI) {  // A+^T A- has the rows -A-_t[k] (k < nx) and zero rows below
#pragma unroll
    for (int i = 0; i < HR; ++i)
      if (H0 + i < nx) {
        const R* am = AMl + (size_t)(t * nx + H0 + i) * n * kWarp;
#pragma unroll
        for (int j = 0; j < NB; ++j) ph[i * NB + j] = fma(R(-1), j < n ? am[j * kWarp] : R(0), R(0));
      }
  } else {
    for (int k = 0; k < nx; ++k) {
      const R* ap = APl + (size_t)(t * nx + k) * n * kWarp;
      const R* am = AMl + (size_t)(t * nx + k) * n * kWarp;
      R x[HR > 0 ? HR : 1], y[NB];
#pragma unroll
      for (int i = 0; i < HR; ++i) x[i] = H0 + i < n ? ap[(H0 + i) * kWarp] : R(0);
#pragma unroll
      for (int j = 0; j < NB; ++j) y[j] = j < n ? am[j * kWarp] : R(0);
#pragma unroll
      for (int i = 0; i < HR; ++i)
#pragma unroll
        for (int j = 0; j < NB; ++j) ph[i * NB + j] = fma(x[i], y[j], ph[i * NB + j]);
    }
  }
  const bool evec = (n * sizeof(R)) % 16 == 0 && (reinterpret_cast<uintptr_t>(E) & 15) == 0;
#pragma unroll
  for (int i = 0; i < HR; ++i) {
    if (H0 + i < n) {
      R er[NB];
      il_load_row<NB>(er, E + (H0 + i) * n, n, evec);
#pragma unroll
      for (int j = 0; j < NB; ++j)
        if (j < n) O[(size_t)(T * trin + (t * n + H0 + i) * n + j) * kWarp] = er[j] + rf * ph[i * NB + j];
    }
  }
}

template <int NB, typename R>
__global__ void __launch_bounds__(kAsmParts * kWarp) il_assemble_kernel(IlArgs<R> A, TmpcQP qp, const int* gate) {
  if (gate && *gate == 0) return;
  const int lane = threadIdx.x & (kWarp - 1), part = threadIdx.x / kWarp, t = blockIdx.y, grp = blockIdx.x;
  if (grp * kWarp + lane >= A.Nb) return;
  static_assert(kAsmParts == 4, "four parts");
  switch (part) {
    case 0: il_assemble_part<NB, R, 0>(A, qp, grp, t, lane); break;
    case 1: il_assemble_part<NB, R, 1>(A, qp, grp, t, lane); break;
    case 2: il_assemble_part<NB, R, 2>(A, qp, grp, t, lane); break;
    default: il_assemble_part<NB, R, 3>(A, qp, grp, t, lane); break;
  }
}

// ---------------------------------------------------------------------------
// gamma from the current state (compute_gamma's formula and order), one
// thread per (problem, stage).  Also ORs the last factor's status bits into
// the problem's status.  With chg, only problems whose rho just changed.
// ---------------------------------------------------------------------------
template <int NB, typename R>
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
  const int grp = blockIdx.x;
  const bool apI = A.apid[grp] != 0, gS = m > 0 && A.gsel[grp] != 0;  // structure: rows not read
  const int* gc = A.gcol + (size_t)grp * (m > 0 ? m : 1);
  // Row by row: each constraint row's values are read once and its target
  // (rho_f c - y_f, or rho z - y_g) multiplies the whole row into the NB
  // per-column sums, which see their terms in compute_gamma's order.
  R eq[NB], iq[NB];
#pragma unroll
  for (int j = 0; j < NB; ++j) eq[j] = iq[j] = R(0);
  auto add_row = [&](R (&s)[NB], const R* row, size_t E, R tgt) {  // row: element offset of the row's first value
#pragma unroll
    for (int j = 0; j < NB; ++j)
      if (j < n) s[j] += row[ix(b, E, j)] * tgt;
  };
  auto ctd = [&](int k) { return rf * A.c[ix(b, z.c, k)] - A.yfd[ix(b, z.yfd, k)]; };
  if (t == 0) {
    for (int k = 0; k < n0; ++k)
      add_row(eq, A.a0 + (size_t)k * n * kWarp, z.a0, rf * A.c0[ix(b, z.c0, k)] - A.yf0[ix(b, z.yf0, k)]);
    if (N > 0)
      for (int k = 0; k < nx; ++k) add_row(eq, A.am + (size_t)k * n * kWarp, z.am, ctd(k));
  } else {
    if (apI) {  // row k of A+ is -e_k: only column k takes its target
#pragma unroll
      for (int j = 0; j < NB; ++j)
        if (j < nx) eq[j] += R(-1) * ctd((t - 1) * nx + j);
    } else {
      for (int k = 0; k < nx; ++k)
        add_row(eq, A.ap + (size_t)((t - 1) * nx + k) * n * kWarp, z.am, ctd((t - 1) * nx + k));
    }
    if (t < N)
      for (int k = 0; k < nx; ++k) add_row(eq, A.am + (size_t)(t * nx + k) * n * kWarp, z.am, ctd(t * nx + k));
  }
  for (int k = 0; k < m; ++k) {
    const R tgt = rho * A.zg[ix(b, z.zm, (size_t)t * m + k)] - A.yg[ix(b, z.zm, (size_t)t * m + k)];
    if (gS) {  // row k of G is e_{gc[k]}
      const int c = gc[k];
#pragma unroll
      for (int j = 0; j < NB; ++j)
        if (j == c) iq[j] += R(1) * tgt;
    } else {
      add_row(iq, A.g + (size_t)(t * m + k) * n * kWarp, z.g, tgt);
    }
  }
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    if (j < n) {
      R val = A.sigma * A.x[ix(b, z.x, (size_t)t * n + j)] - A.q[ix(b, z.q, (size_t)t * n + j)];
      val += eq[j];
      val += iq[j];
      A.gam[ix(b, z.x, (size_t)t * n + j)] = val;
    }
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
// Stage buffer sizes (elements per problem).  The full layout keeps room for
// every block; the compact one (CMP: A+_t = [-I 0], unit inequality rows and
// W_t rows nx..n-1 exact zeros, all detected per group) drops A+, G and the
// zero rows of W.
__host__ __device__ inline int il_fwd_elems(int n, int wrows) { return (int)(tri(n) + (size_t)wrows * n + n); }
__host__ __device__ inline int il_qp_elems(int n, int nx, int m) { return 2 * nx * n + m * n + 2 * n + 2 * nx + 4 * m; }
__host__ __device__ inline int il_qp_elems_cmp(int n, int nx, int m) { return nx * n + 2 * n + 2 * nx + 4 * m; }
__host__ __device__ inline int il_buf_a_elems(int n, int nx, bool cmp) { return il_fwd_elems(n, cmp ? nx : n); }
__host__ __device__ inline int il_buf_b_elems(int n, int nx, int m, bool cmp) {
  const int a = il_buf_a_elems(n, nx, cmp), q = cmp ? il_qp_elems_cmp(n, nx, m) : il_qp_elems(n, nx, m);
  return a > q ? a : q;
}
// Dynamic shared memory: buffer A, buffer B, then the vectors
// ush[NB], xs0[NB], xs1[NB], ctv[nx], gtv[m], ct0v[n0] (each x 32 lanes).
template <int NB, typename R>
size_t il_admm_smem(int n, int nx, int n0, int m, bool cmp) {
  const size_t e = (size_t)il_buf_a_elems(n, nx, cmp) + il_buf_b_elems(n, nx, m, cmp) + 3 * NB + nx + m + n0;
  return e * kWarp * sizeof(R);
}
// The compact layout applies to a group whose structure flags all hold.
__device__ __forceinline__ bool il_group_compact(const int* apid, const int* gsel, const int* wrow, int grp, int nx,
                                                 int m) {
  return apid[grp] != 0 && (m == 0 || gsel[grp] != 0) && wrow[grp] == nx;
}

// sum_{k < cnt} a[k sa] v[k 32] with four partial sums, unrolled to NB terms
// (a and v point at this lane's element 0).
template <int NB, typename R>
__device__ __forceinline__ R il_dot(const R* a, int sa, const R* v, int cnt) {
  R s[4] = {R(0), R(0), R(0), R(0)};
#pragma unroll
  for (int k = 0; k < NB; ++k)
    if (k < cnt) s[k & 3] = fma(a[k * sa], v[k * kWarp], s[k & 3]);
  return (s[0] + s[1]) + (s[2] + s[3]);
}

// EX: n == NB, so every stage-block loop has compile-time bounds and strides.
// NW warps per block; warp w owns the stage rows / columns w, w + NW, ...
// CMP: the compact variant (runs only the groups whose structure flags all
// hold, with the compact buffers: 8 warps and two blocks per SM); the full
// variant skips those groups when skip_cmp is set (the compact launch ran
// them).  Both do the same arithmetic in the same order.
template <int NB, typename R, bool EX, int NW, bool CMP>
__global__ void __launch_bounds__(32 * NW, CMP ? 2 : 1) il_admm_kernel(const IlArgs<R> A, int it0, int it1,
                                                                      int skip_cmp) {
  constexpr int RPW = (NB + NW - 1) / NW;  // stage rows per warp
  constexpr int NT = 32 * NW;
  constexpr int V = 16 / sizeof(R);
  constexpr int L32 = kWarp;
  extern __shared__ __align__(16) unsigned char il_smem[];
  const int lane = threadIdx.x & (kWarp - 1), w = threadIdx.x / kWarp;
  const int grp = blockIdx.x;
  const int b = grp * kWarp + lane;
  const int T = A.T, N = T - 1, n = EX ? NB : A.n, nx = A.nx, n0 = A.n0, m = A.m;
  {
    const bool cg = il_group_compact(A.apid, A.gsel, A.wrow, grp, nx, m);
    if (CMP ? !cg : (skip_cmp && cg)) return;  // the other variant runs this group
  }
  const bool act = b < A.Nb && A.act[b] != 0;
  if (!__syncthreads_or(act)) return;  // every problem of the group has converged
  const IlSizes z(T, n, nx, n0, m);
  const int trin = (int)tri(n), nn = n * n, woff = T * trin;
  const R rho = A.rho[b], rf = rho * A.rff, al = A.alpha, sw = A.sw[b], sigma = A.sigma;
  const bool slack = A.use_slack != 0;
  const bool apI = CMP || A.apid[grp] != 0;        // A+_t = [-I 0] for the whole group
  const bool gS = CMP || A.gsel[grp] != 0;         // G_t[k] = e_{gc[k]} for the whole group
  const int wr = CMP ? nx : A.wrow[grp];           // rows of W_t that are not exact zeros: nx or n
  const int wcap = CMP ? nx : n;                   // W rows the stage buffer holds
  const int* gc = A.gcol + (size_t)grp * (m > 0 ? m : 1);
  // group bases of the interleaved arrays (element e of this group: base[e * 32 + lane])
  auto gb = [&](R* p, size_t E) { return p + (size_t)grp * E * kWarp; };
  const R* F = gb(A.ops, z.ops);
  const R* Q = gb(A.q, z.q);
  const R* AM = gb(A.am, z.am);
  const R* AP = gb(A.ap, z.am);
  const R* Gm = m > 0 ? gb(A.g, z.g) : nullptr;
  const R* CC = gb(A.c, z.c);
  const R* LL = m > 0 ? gb(A.l, z.lu) : nullptr;
  const R* UU = m > 0 ? gb(A.u, z.lu) : nullptr;
  R* X = gb(A.x, z.x) + lane;
  R* YFD = gb(A.yfd, z.yfd);
  R* ZG = m > 0 ? gb(A.zg, z.zm) : nullptr;
  R* YG = m > 0 ? gb(A.yg, z.zm) : nullptr;
  R* XIG = m > 0 ? gb(A.xig, z.zm) + lane : nullptr;
  R* GAM = gb(A.gam, z.x);
  R* YS = gb(A.ys, z.x);
  R* const A0l = n0 > 0 ? gb(A.a0, z.a0) + lane : nullptr;
  R* const C0l = n0 > 0 ? gb(A.c0, z.c0) + lane : nullptr;
  R* const YF0l = n0 > 0 ? gb(A.yf0, z.yf0) + lane : nullptr;
  R* sm = reinterpret_cast<R*>(il_smem);
  const int SA = il_buf_a_elems(n, nx, CMP), SB = il_buf_b_elems(n, nx, m, CMP);
  R* BA = sm;
  R* BB = sm + SA * L32;
  R* ush = BB + SB * L32;
  R* xs0 = ush + NB * L32;
  R* xs1 = xs0 + NB * L32;
  R* ctv = xs1 + NB * L32;
  R* gtv = ctv + nx * L32;
  R* ct0v = gtv + m * L32;
  // copy `elems` interleaved elements (contiguous from src) to dst, 16 bytes per cp.async
  auto copy = [&](R* dst, const R* src, int elems) {
    const int chunks = elems * (L32 / V);
    for (int c = threadIdx.x; c < chunks; c += NT) cp_async16(dst + c * V, src + c * V);
  };
  // stage buffer A / forward buffers: L_t^-1 (packed), W rows, then the vector
  const int ovec = trin + wcap * n;
  // buffer B (backward) offsets; the compact layout has no A+ and no G
  const int oAm = 0, oAp = CMP ? 0 : nx * n, oG = CMP ? nx * n : 2 * nx * n, oq = oG + (CMP ? 0 : m * n),
            oc = oq + n, ox = oc + nx, oyf = ox + n, ozg = oyf + nx, oyg = ozg + m, ol = oyg + m, ou = ol + m;
  auto fetch_fwd = [&](R* dst, int t) {
    copy(dst, F + (size_t)t * trin * L32, trin);
    if (t > 0) copy(dst + trin * L32, F + ((size_t)woff + (size_t)(t - 1) * nn) * L32, wr * n);
    copy(dst + ovec * L32, GAM + (size_t)t * n * L32, n);
  };
  auto fetch_bwd_a = [&](int t) {
    copy(BA, F + (size_t)t * trin * L32, trin);
    if (t < N) copy(BA + trin * L32, F + ((size_t)woff + (size_t)t * nn) * L32, wr * n);
    copy(BA + ovec * L32, YS + (size_t)t * n * L32, n);
  };
  auto fetch_bwd_b = [&](int t) {
    if (t < N) {
      copy(BB + oAm * L32, AM + (size_t)t * nx * n * L32, nx * n);
      if (!apI) copy(BB + oAp * L32, AP + (size_t)t * nx * n * L32, nx * n);
      copy(BB + oc * L32, CC + (size_t)t * nx * L32, nx);
      copy(BB + oyf * L32, YFD + (size_t)t * nx * L32, nx);
    }
    if (m > 0) {
      if (!gS) copy(BB + oG * L32, Gm + (size_t)t * m * n * L32, m * n);
      copy(BB + ozg * L32, ZG + (size_t)t * m * L32, m);
      copy(BB + oyg * L32, YG + (size_t)t * m * L32, m);
      copy(BB + ol * L32, LL + (size_t)t * m * L32, m);
      copy(BB + ou * L32, UU + (size_t)t * m * L32, m);
    }
    copy(BB + oq * L32, Q + (size_t)t * n * L32, n);
    copy(BB + ox * L32, gb(A.x, z.x) + (size_t)t * n * L32, n);
  };
  // this lane's views of the buffers and vectors
  R* const BAl = BA + lane;
  R* const BBl = BB + lane;
  R* const ushl = ush + lane;
  R* const xs0l = xs0 + lane;
  R* const xs1l = xs1 + lane;
  R* const ctvl = ctv + lane;
  R* const gtvl = gtv + lane;
  R* const ct0vl = ct0v + lane;
  R* const YSl = YS + lane;
  R* const GAMl = GAM + lane;
  R* const YFDl = YFD + lane;
  R* const ZGl = m > 0 ? ZG + lane : nullptr;
  R* const YGl = m > 0 ? YG + lane : nullptr;

  for (int it = it0; it < it1; ++it) {
    // ---------------- forward sweep: y_t = L_t^-1 (gamma_t - W_{t-1} y_{t-1})
    fetch_fwd(BA, 0);
    cp_async_commit();
    fetch_fwd(BB, 1);
    cp_async_commit();
    for (int t = 0; t < T; ++t) {
      R* bufl = ((t & 1) ? BB : BA) + lane;
      cp_async_wait<1>();
      __syncthreads();
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        if (i < n) {
          R u = bufl[(ovec + i) * L32];
          if (t > 0 && i < wr) u -= il_dot<NB>(bufl + (trin + i * n) * L32, L32, xs0l, n);
          ushl[i * L32] = u;
        }
      }
      __syncthreads();
      R y[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        y[r] = R(0);
        if (i < n) {
          y[r] = il_dot<NB>(bufl + (i * (i + 1) / 2) * L32, L32, ushl, i + 1);
          if (act) YSl[(t * n + i) * L32] = y[r];
        }
      }
      __syncthreads();  // every read of this stage's buffer, ush and xs0 is done
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        if (i < n) xs0l[i * L32] = y[r];
      }
      if (t + 2 < T) fetch_fwd(bufl - lane, t + 2);
      cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();

    // ---------------- backward sweep with the ADMM-level updates
    // x~_{t+1} in xs[(t + 1) & 1], x~_t into xs[t & 1]; the pieces of gamma_t
    // formed at step t wait in registers for the A+ terms of step t - 1.
    R gval[RPW], geq[RPW], giq[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) gval[r] = geq[r] = giq[r] = R(0);
    fetch_bwd_a(N);
    cp_async_commit();
    fetch_bwd_b(N);
    cp_async_commit();
    for (int t = N; t >= 0; --t) {
      R* xtl = (t & 1) ? xs1l : xs0l;  // x~_t
      R* xnl = (t & 1) ? xs0l : xs1l;  // x~_{t+1}
      cp_async_wait<1>();
      __syncthreads();
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        if (i < n) {
          R u = BAl[(ovec + i) * L32];
          if (t < N) u -= il_dot<NB>(BAl + (trin + i) * L32, n * L32, xnl, wr);  // column i of W_t (rows < wr)
          ushl[i * L32] = u;
        }
      }
      __syncthreads();
      R xv[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        xv[r] = R(0);
        if (i < n) {  // row i of L_t^-T: sum_{r >= i} Linv[r][i] u_r
          R s[4] = {R(0), R(0), R(0), R(0)};
#pragma unroll
          for (int k = 0; k < NB; ++k)
            if (k >= i && k < n) s[k & 3] = fma(BAl[(k * (k + 1) / 2 + i) * L32], ushl[k * L32], s[k & 3]);
          xv[r] = (s[0] + s[1]) + (s[2] + s[3]);
          xtl[i * L32] = xv[r];
        }
      }
      cp_async_wait<0>();
      __syncthreads();  // x~_t complete, buffer B of stage t landed, buffer A consumed
      if (t > 0) fetch_bwd_a(t - 1);
      cp_async_commit();
      // constraint rows of stage t: dynamics (A- x~_t + A+ x~_{t+1}), inequality, initial
      for (int q = w; q < nx + m; q += NW) {
        if (q < nx) {
          if (t < N) {
            const R cx = il_dot<NB>(BBl + (oAm + q * n) * L32, L32, xtl, n) +
                         (apI ? -xnl[q * L32] : il_dot<NB>(BBl + (oAp + q * n) * L32, L32, xnl, n));
            const R cr = BBl[(oc + q) * L32];
            const R y = BBl[(oyf + q) * L32] + rf * al * (cx - cr);
            if (act) YFDl[(t * nx + q) * L32] = y;
            ctvl[q * L32] = rf * cr - y;
          }
        } else {
          const int k = q - nx;
          const R gx = gS ? xtl[gc[k] * L32] : il_dot<NB>(BBl + (oG + k * n) * L32, L32, xtl, n);
          const R zold = BBl[(ozg + k) * L32], ygo = BBl[(oyg + k) * L32];
          const R zt = al * gx + (R(1) - al) * zold + ygo / rho;
          R cl = zt;
          const R lb = BBl[(ol + k) * L32], ub = BBl[(ou + k) * L32];
          if (cl < lb) cl = lb;
          if (cl > ub) cl = ub;
          R znew;
          if (slack) {
            const R f = sw / (sw + rho);
            znew = (R(1) - f) * zt + f * cl;
            if (act) XIG[(t * m + k) * L32] = (rho / (sw + rho)) * (cl - zt);
          } else {
            znew = cl;
          }
          const R ygn = ygo + rho * (al * gx + (R(1) - al) * zold - znew);
          if (act) {
            ZGl[(t * m + k) * L32] = znew;
            YGl[(t * m + k) * L32] = ygn;
          }
          gtvl[k * L32] = rho * znew - ygn;
        }
      }
      if (t == 0) {
        for (int k = w; k < n0; k += NW) {
          const R s = il_dot<NB>(A0l + k * n * L32, L32, xtl, n);
          const R c0 = C0l[k * L32];
          const R y = YF0l[k * L32] + rf * al * (s - c0);
          if (act) YF0l[k * L32] = y;
          ct0vl[k * L32] = rf * c0 - y;
        }
      }
      R xr[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        xr[r] = R(0);
        if (i < n) {  // relaxation of x_t
          xr[r] = al * xv[r] + (R(1) - al) * BBl[(ox + i) * L32];
          if (act) X[(t * n + i) * L32] = xr[r];
        }
      }
      __syncthreads();  // ctv, gtv, ct0v complete
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        const int i = w + r * NW;
        if (i < n) {  // gamma for the next iteration (column i)
          if (t < N) {  // the A+ terms of the dynamics rows of stage t complete gamma_{t+1}
            const R ap =
                apI ? (i < nx ? -ctvl[i * L32] : R(0)) : il_dot<NB>(BBl + (oAp + i) * L32, n * L32, ctvl, nx);
            if (act) GAMl[((t + 1) * n + i) * L32] = (gval[r] + (ap + geq[r])) + giq[r];
          }
          const R val = sigma * xr[r] - BBl[(oq + i) * L32];
          R eq = R(0);
          if (t == 0) {
            for (int k = 0; k < n0; ++k) eq += A0l[(k * n + i) * L32] * ct0vl[k * L32];
          }
          if (t < N) {
            if (t == 0) {
              for (int k = 0; k < nx; ++k) eq += BBl[(oAm + k * n + i) * L32] * ctvl[k * L32];
            } else {
              eq = il_dot<NB>(BBl + (oAm + i) * L32, n * L32, ctvl, nx);
            }
          }
          R iq = R(0);
          if (gS) {
            for (int k = 0; k < m; ++k)
              if (gc[k] == i) iq += gtvl[k * L32];
          } else {
            for (int k = 0; k < m; ++k) iq += BBl[(oG + k * n + i) * L32] * gtvl[k * L32];
          }
          if (t == 0) {
            if (act) GAMl[i * L32] = (val + eq) + iq;
          } else {
            gval[r] = val;
            geq[r] = eq;
            giq[r] = iq;
          }
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
  if ((long)il_admm_smem<NB, R>(d.n, d.nx, d.n0, d.m, false) > max_dyn_smem()) return false;
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

// Diagnostics: CUDA events around the ADMM iteration launches of each call
// (tmpc_admm_iteration_timing).
namespace {
std::mutex g_tm_mu;
bool g_tm_on = false;
std::vector<std::pair<cudaEvent_t, cudaEvent_t>> g_tm;
constexpr size_t kTmMax = 1024;
cudaEvent_t tm_begin(cudaStream_t st) {
  std::lock_guard<std::mutex> lk(g_tm_mu);
  if (!g_tm_on || g_tm.size() >= kTmMax) return nullptr;
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  cudaEventRecord(e, st);
  return e;
}
void tm_end(cudaEvent_t e0, cudaStream_t st) {
  if (!e0) return;
  cudaEvent_t e1 = nullptr;
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    return;
  }
  cudaEventRecord(e1, st);
  std::lock_guard<std::mutex> lk(g_tm_mu);
  g_tm.emplace_back(e0, e1);
}
}  // namespace

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
  // structure of A+ and G on the caller's arrays: groups where it holds
  // convert neither (their rows are formed from the structure)
  if (N > 0) {
    il_ap_identity_kernel<R><<<(unsigned)Nb, kFlatThreads, 0, st>>>(
        A, static_cast<const R*>(P.qp.A_plus));
    chk((int)cudaPeekAtLastError());
  } else {
    cudaMemsetAsync(A.apid, 0, groups(Nb) * sizeof(int), st);
  }
  if (m > 0) {
    il_g_columns_kernel<R><<<(unsigned)((groups(Nb) * m + kFlatThreads - 1) / kFlatThreads), kFlatThreads, 0, st>>>(
        A, static_cast<const R*>(P.qp.G));
    il_g_select_kernel<R><<<(unsigned)Nb, kFlatThreads, 0, st>>>(A, static_cast<const R*>(P.qp.G));
    chk((int)cudaPeekAtLastError());
  } else {
    cudaMemsetAsync(A.gsel, 0, groups(Nb) * sizeof(int), st);
  }
  if (rc) return rc;
  auto inl_skip = [&](const void* src, R* dst, size_t E, const int* skip) {
    if (E == 0 || src == nullptr) return;
    chk(interleave<R>(Nb, E, E, static_cast<const R*>(src), dst, IdentityMap{}, st, skip));
  };
  inl(P.qp.q, A.q, z.q);
  inl(P.qp.A0, A.a0, z.a0);
  inl(P.qp.A_minus, A.am, z.am);
  inl_skip(P.qp.A_plus, A.ap, z.am, A.apid);
  inl_skip(P.qp.G, A.g, z.g, A.gsel);
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
    const size_t smem = il_admm_smem<NB, R>(n, nx, n0, m, false);
    const size_t csmem = il_check_smem<NB, R>(T, nx, n0, m);
    auto kadmm = n == NB ? il_admm_kernel<NB, R, true, kIlWarps, false> : il_admm_kernel<NB, R, false, kIlWarps, false>;
    chk((int)cudaFuncSetAttribute(kadmm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // fp32: the groups with the compact structure run in the compact variant
    // (two blocks per SM) when two of its blocks fit one SM's shared memory
    const size_t csm = il_admm_smem<NB, R>(n, nx, n0, m, true);
    void (*kcmp)(const IlArgs<R>, int, int, int) = nullptr;
    if constexpr (sizeof(R) == 4)
      kcmp = n == NB ? il_admm_kernel<NB, R, true, kIlCmpWarps, true> : il_admm_kernel<NB, R, false, kIlCmpWarps, true>;
    const bool use_cmp = kcmp != nullptr && nx < n && (long)(2 * (csm + 1024)) <= max_sm_smem();
    if (use_cmp) chk((int)cudaFuncSetAttribute(kcmp, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csm));
    chk((int)cudaFuncSetAttribute(il_check_kernel<NB, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)csmem));
    if (rc) return rc;
    const dim3 ggrid((unsigned)groups(Nb), (unsigned)T);
    // operator, factor (in place) and the first gamma; with `gate`, only
    // when a check opened it, gamma only for the flagged problems
    auto build = [&](const int* gate) {
      il_assemble_kernel<NB, R><<<ggrid, kAsmParts * kWarp, 0, st>>>(A, P.qp, gate);
      chk((int)cudaPeekAtLastError());
      chk(launch_factor<NB, R>(Nb, T, n, A.ops, A.ops, A.fstat, gate, st));
      il_w_rows_kernel<R><<<(unsigned)groups(Nb), kWrowThreads, 0, st>>>(A, gate);
      chk((int)cudaPeekAtLastError());
      il_gamma_kernel<NB, R><<<ggrid, kWarp, 0, st>>>(A, gate, gate ? 1 : 0);
      chk((int)cudaPeekAtLastError());
      if (gate) {
        il_clear_chg_kernel<<<(G32 + 255) / 256, 256, 0, st>>>(A.chg, G32, A.gate);
        chk((int)cudaPeekAtLastError());
      }
    };
    auto iterate = [&](int a, int e) {
      if (e <= a) return;
      if (use_cmp) {
        kcmp<<<(unsigned)groups(Nb), 32 * kIlCmpWarps, csm, st>>>(A, a, e, 0);
        chk((int)cudaPeekAtLastError());
      }
      kadmm<<<(unsigned)groups(Nb), kIlThreads, smem, st>>>(A, a, e, use_cmp ? 1 : 0);
      chk((int)cudaPeekAtLastError());
    };
    build(nullptr);
    cudaEvent_t tm0 = tm_begin(st);
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
    tm_end(tm0, st);
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

extern "C" {

int32_t tmpc_admm_iteration_timing(int32_t enable) {
  std::lock_guard<std::mutex> lk(tmpc::g_tm_mu);
  const int32_t prev = tmpc::g_tm_on ? 1 : 0;
  tmpc::g_tm_on = enable != 0;
  return prev;
}

int32_t tmpc_admm_iteration_timing_read(float* ms_out, int32_t max_out) {
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev;
  {
    std::lock_guard<std::mutex> lk(tmpc::g_tm_mu);
    ev.swap(tmpc::g_tm);
  }
  int32_t k = 0;
  for (auto& p : ev) {
    float ms = -1.f;
    if (cudaEventSynchronize(p.second) == cudaSuccess && cudaEventElapsedTime(&ms, p.first, p.second) == cudaSuccess &&
        ms_out && k < max_out)
      ms_out[k++] = ms;
    cudaEventDestroy(p.first);
    cudaEventDestroy(p.second);
  }
  return k;
}

}  // extern "C"
