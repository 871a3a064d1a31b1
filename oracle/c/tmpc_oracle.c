/*
 * C restatement of TurboMPC's ADMM + PCG inner solve (one call handles a
 * contiguous sub-batch; the caller runs sub-batches on several host threads).
 * TEST INFRASTRUCTURE / CPU BASELINE ONLY: used by bench.py's CPU-baseline
 * leg and `--impl reference`, and checked against the NumPy oracle in tests/.
 * Never linked by the turbompc_b200 package.
 *
 * Per problem (reference layout, see include/tmpc_b200.h):
 *   compute_S_Phiinv   turbompc/solvers/admm/admm.py:71-154 (Gauss-Jordan inverse,
 *                      as admm/csrc/admm_math.cuh:248-310)
 *   ADMM loop          admm/csrc/admm_fused.cu:701-925 at fixed iteration counts
 *                      (residual checks / rho adaptation disabled)
 *   PCG                admm/csrc/admm_fused.cu:54-161
 *   direct solve       (pcg_iters < 0) block-tridiagonal Cholesky of S, factored
 *                      once per problem and applied every ADMM iteration: the
 *                      semantics of the cuDSS backend (admm/csrc/admm_cudss.cu),
 *                      an exact solve of S x = gamma
 * Compiled twice (float / double) from the macro body below.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define DEFINE_ORACLE(R, SUF)                                                                                  \
  static void bt_apply_##SUF(const R* M, const R* v, R* y, int T, int n) {                                    \
    for (int t = 0; t < T; ++t)                                                                               \
      for (int i = 0; i < n; ++i) {                                                                           \
        const R* row = M + ((size_t)t * n + i) * 3 * n;                                                       \
        R s = 0;                                                                                              \
        if (t > 0)                                                                                            \
          for (int j = 0; j < n; ++j) s += row[j] * v[(t - 1) * n + j];                                       \
        for (int j = 0; j < n; ++j) s += row[n + j] * v[t * n + j];                                           \
        if (t < T - 1)                                                                                        \
          for (int j = 0; j < n; ++j) s += row[2 * n + j] * v[(t + 1) * n + j];                               \
        y[t * n + i] = s;                                                                                     \
      }                                                                                                       \
  }                                                                                                           \
  static R dot_##SUF(const R* a, const R* b, int k) {                                                         \
    R s = 0;                                                                                                  \
    for (int i = 0; i < k; ++i) s += a[i] * b[i];                                                             \
    return s;                                                                                                 \
  }                                                                                                           \
  static void inv_##SUF(const R* A, R* Ai, R* w, int n) {                                                     \
    int n2 = 2 * n;                                                                                           \
    for (int i = 0; i < n; ++i)                                                                               \
      for (int j = 0; j < n2; ++j) w[i * n2 + j] = j < n ? A[i * n + j] : (j - n == i ? 1 : 0);               \
    for (int c = 0; c < n; ++c) {                                                                             \
      int p = c;                                                                                              \
      for (int r = c + 1; r < n; ++r)                                                                         \
        if (fabs((double)w[r * n2 + c]) > fabs((double)w[p * n2 + c])) p = r;                                 \
      if (p != c)                                                                                             \
        for (int j = 0; j < n2; ++j) {                                                                        \
          R tmp = w[c * n2 + j];                                                                              \
          w[c * n2 + j] = w[p * n2 + j];                                                                      \
          w[p * n2 + j] = tmp;                                                                                \
        }                                                                                                     \
      R ip = (R)1 / w[c * n2 + c];                                                                            \
      for (int j = 0; j < n2; ++j) w[c * n2 + j] *= ip;                                                       \
      for (int r = 0; r < n; ++r) {                                                                           \
        if (r == c) continue;                                                                                 \
        R f = w[r * n2 + c];                                                                                  \
        for (int j = 0; j < n2; ++j) w[r * n2 + j] -= f * w[c * n2 + j];                                      \
      }                                                                                                       \
    }                                                                                                         \
    for (int i = 0; i < n; ++i)                                                                               \
      for (int j = 0; j < n; ++j) Ai[i * n + j] = w[i * n2 + n + j];                                          \
  }                                                                                                           \
  /* S, Phiinv (T, n, 3n) for one problem; scratch: th (T n n), ti (T n n), ph (N n n), w (2 n n) */           \
  static void schur_##SUF(const R* D, const R* E, const R* A0, const R* Am, const R* Ap, const R* G, int T,    \
                          int n, int nx, int n0, int m, R rf, R ri, R sigma, R* S, R* P, R* th, R* ti, R* ph,  \
                          R* w, int direct) {                                                                 \
    int N = T - 1;                                                                                            \
    for (int t = 0; t < T; ++t)                                                                               \
      for (int i = 0; i < n; ++i)                                                                             \
        for (int j = 0; j < n; ++j) {                                                                         \
          R v = D[((size_t)t * n + i) * n + j] + (i == j ? sigma : 0);                                        \
          R g = 0, a = 0;                                                                                     \
          for (int k = 0; k < m; ++k) g += G[((size_t)t * m + k) * n + i] * G[((size_t)t * m + k) * n + j];    \
          if (t == 0) {                                                                                       \
            for (int k = 0; k < n0; ++k) a += A0[k * n + i] * A0[k * n + j];                                  \
            for (int k = 0; k < nx; ++k) a += Am[k * n + i] * Am[k * n + j];                                  \
          } else {                                                                                            \
            const R* ap = Ap + (size_t)(t - 1) * nx * n;                                                      \
            for (int k = 0; k < nx; ++k) a += ap[k * n + i] * ap[k * n + j];                                  \
            if (t < N) {                                                                                      \
              const R* am = Am + (size_t)t * nx * n;                                                          \
              for (int k = 0; k < nx; ++k) a += am[k * n + i] * am[k * n + j];                                \
            }                                                                                                 \
          }                                                                                                   \
          th[((size_t)t * n + i) * n + j] = v + ri * g + rf * a;                                              \
        }                                                                                                     \
    for (int t = 0; t < N; ++t)                                                                               \
      for (int i = 0; i < n; ++i)                                                                             \
        for (int j = 0; j < n; ++j) {                                                                         \
          R a = 0;                                                                                            \
          for (int k = 0; k < nx; ++k)                                                                        \
            a += Ap[((size_t)t * nx + k) * n + i] * Am[((size_t)t * nx + k) * n + j];                         \
          ph[((size_t)t * n + i) * n + j] = E[((size_t)t * n + i) * n + j] + rf * a;                          \
        }                                                                                                     \
    if (direct) return;                                                                                       \
    for (int t = 0; t < T; ++t) inv_##SUF(th + (size_t)t * n * n, ti + (size_t)t * n * n, w, n);              \
    memset(S, 0, sizeof(R) * (size_t)T * n * 3 * n);                                                          \
    memset(P, 0, sizeof(R) * (size_t)T * n * 3 * n);                                                          \
    for (int t = 0; t < T; ++t)                                                                               \
      for (int i = 0; i < n; ++i) {                                                                           \
        R* sr = S + ((size_t)t * n + i) * 3 * n;                                                              \
        R* pr = P + ((size_t)t * n + i) * 3 * n;                                                              \
        for (int j = 0; j < n; ++j) {                                                                         \
          sr[n + j] = th[((size_t)t * n + i) * n + j];                                                        \
          pr[n + j] = -ti[((size_t)t * n + i) * n + j];                                                       \
          if (t > 0) sr[j] = ph[((size_t)(t - 1) * n + i) * n + j];                                           \
          if (t < N) sr[2 * n + j] = ph[((size_t)t * n + j) * n + i];                                         \
        }                                                                                                     \
      }                                                                                                       \
    /* prev block: ti_t phi_{t-1} ti_{t-1}; next block: ti_t phi_t^T ti_{t+1} */                              \
    for (int t = 0; t < T; ++t) {                                                                             \
      const R* a = ti + (size_t)t * n * n;                                                                    \
      for (int side = 0; side < 2; ++side) {                                                                  \
        if ((side == 0 && t == 0) || (side == 1 && t == N)) continue;                                         \
        const R* c2 = ti + (size_t)(side == 0 ? t - 1 : t + 1) * n * n;                                       \
        for (int i = 0; i < n; ++i)                                                                           \
          for (int j = 0; j < n; ++j) {                                                                       \
            R s = 0;                                                                                          \
            for (int p = 0; p < n; ++p) {                                                                     \
              R u = 0;                                                                                        \
              for (int q = 0; q < n; ++q) {                                                                   \
                R pv = side == 0 ? ph[((size_t)(t - 1) * n + p) * n + q] : ph[((size_t)t * n + q) * n + p];  \
                u += pv * c2[q * n + j];                                                                      \
              }                                                                                               \
              s += a[i * n + p] * u;                                                                          \
            }                                                                                                 \
            P[((size_t)t * n + i) * 3 * n + (side == 0 ? 0 : 2 * n) + j] = s;                                 \
          }                                                                                                   \
      }                                                                                                       \
    }                                                                                                         \
  }                                                                                                           \
  /* Block Cholesky S = L L^T in place: th_t <- L_t (lower), ph_t <- W_t = Phi_t L_t^-T, with            \
     L_0 L_0^T = Theta_0, L_t L_t^T = Theta_t - W_{t-1} W_{t-1}^T.  Returns 0, or -1 on a non-positive pivot. */ \
  static int chol_##SUF(R* th, R* ph, int T, int n) {                                                         \
    for (int t = 0; t < T; ++t) {                                                                             \
      R* L = th + (size_t)t * n * n;                                                                          \
      if (t > 0) {                                                                                            \
        const R* W = ph + (size_t)(t - 1) * n * n;                                                            \
        for (int i = 0; i < n; ++i)                                                                           \
          for (int j = 0; j <= i; ++j) {                                                                      \
            R s = 0;                                                                                          \
            for (int k = 0; k < n; ++k) s += W[i * n + k] * W[j * n + k];                                     \
            L[i * n + j] -= s;                                                                                \
          }                                                                                                   \
      }                                                                                                       \
      for (int j = 0; j < n; ++j) {                                                                           \
        R d = L[j * n + j];                                                                                   \
        for (int k = 0; k < j; ++k) d -= L[j * n + k] * L[j * n + k];                                         \
        if (!(d > 0)) return -1;                                                                              \
        d = (R)sqrt((double)d);                                                                               \
        L[j * n + j] = d;                                                                                     \
        for (int i = j + 1; i < n; ++i) {                                                                     \
          R s = L[i * n + j];                                                                                 \
          for (int k = 0; k < j; ++k) s -= L[i * n + k] * L[j * n + k];                                       \
          L[i * n + j] = s / d;                                                                               \
        }                                                                                                     \
      }                                                                                                       \
      if (t < T - 1) { /* W_t rows: solve L_t w^T = phi_i^T (forward substitution) */                         \
        R* W = ph + (size_t)t * n * n;                                                                        \
        for (int i = 0; i < n; ++i)                                                                           \
          for (int k = 0; k < n; ++k) {                                                                       \
            R s = W[i * n + k];                                                                               \
            for (int c = 0; c < k; ++c) s -= L[k * n + c] * W[i * n + c];                                     \
            W[i * n + k] = s / L[k * n + k];                                                                  \
          }                                                                                                   \
      }                                                                                                       \
    }                                                                                                         \
    return 0;                                                                                                 \
  }                                                                                                           \
  /* x = S^-1 g with the block Cholesky factor; y scratch (T n) */                                            \
  static void chol_solve_##SUF(const R* Lb, const R* Wb, const R* g, R* x, R* y, int T, int n) {              \
    for (int t = 0; t < T; ++t) {                                                                             \
      const R* L = Lb + (size_t)t * n * n;                                                                    \
      for (int i = 0; i < n; ++i) {                                                                           \
        R s = g[t * n + i];                                                                                   \
        if (t > 0) {                                                                                          \
          const R* W = Wb + (size_t)(t - 1) * n * n;                                                          \
          for (int k = 0; k < n; ++k) s -= W[i * n + k] * y[(t - 1) * n + k];                                 \
        }                                                                                                     \
        for (int c = 0; c < i; ++c) s -= L[i * n + c] * y[t * n + c];                                         \
        y[t * n + i] = s / L[i * n + i];                                                                      \
      }                                                                                                       \
    }                                                                                                         \
    for (int t = T - 1; t >= 0; --t) {                                                                        \
      const R* L = Lb + (size_t)t * n * n;                                                                    \
      for (int i = n - 1; i >= 0; --i) {                                                                      \
        R s = y[t * n + i];                                                                                   \
        if (t < T - 1) {                                                                                      \
          const R* W = Wb + (size_t)t * n * n;                                                                \
          for (int k = 0; k < n; ++k) s -= W[k * n + i] * x[(t + 1) * n + k];                                 \
        }                                                                                                     \
        for (int r = i + 1; r < n; ++r) s -= L[r * n + i] * x[t * n + r];                                     \
        x[t * n + i] = s / L[i * n + i];                                                                      \
      }                                                                                                       \
    }                                                                                                         \
  }                                                                                                           \
  static void pcg_##SUF(const R* S, const R* P, const R* g, R* x, int T, int n, int iters, R eps, R* r, R* z,  \
                        R* p, R* sp) {                                                                        \
    int k = T * n;                                                                                            \
    bt_apply_##SUF(S, x, sp, T, n);                                                                           \
    for (int i = 0; i < k; ++i) r[i] = g[i] - sp[i];                                                          \
    bt_apply_##SUF(P, r, z, T, n);                                                                            \
    memcpy(p, z, sizeof(R) * k);                                                                              \
    R eta = dot_##SUF(r, z, k), eta0 = (R)fabs((double)eta);                                                  \
    for (int it = 0; it < iters; ++it) {                                                                      \
      if (fabs((double)eta) < 1e-12 + (double)eps * (double)eta0) break;                                      \
      bt_apply_##SUF(S, p, sp, T, n);                                                                         \
      R den = dot_##SUF(p, sp, k);                                                                            \
      if (fabs((double)den) < 1e-30) den = (R)1e-30;                                                          \
      R a = eta / den;                                                                                        \
      for (int i = 0; i < k; ++i) {                                                                           \
        x[i] += a * p[i];                                                                                     \
        r[i] -= a * sp[i];                                                                                    \
      }                                                                                                       \
      bt_apply_##SUF(P, r, z, T, n);                                                                          \
      R en = dot_##SUF(r, z, k);                                                                              \
      R b = en / eta;                                                                                         \
      eta = en;                                                                                               \
      for (int i = 0; i < k; ++i) p[i] = z[i] + b * p[i];                                                     \
    }                                                                                                         \
  }                                                                                                           \
  /* Batched fixed-count ADMM; state arrays updated in place. Returns 0. */                                   \
  int tmpc_oracle_admm_##SUF(int Nb, int T, int n, int nx, int n0, int m, const R* D, const R* E, const R* q,  \
                             const R* A0, const R* Am, const R* Ap, const R* c0, const R* c, const R* G,       \
                             const R* l, const R* u, R* x, R* yg, R* yf0, R* yfd, R* zg, R* rho_in,            \
                             int admm_iters, int pcg_iters, double sigma, double rho_f_factor, double alpha,   \
                             int threads) {                                                                   \
    int N = T - 1;                                                                                            \
    (void)threads;                                                                                            \
    for (int b = 0; b < Nb; ++b) {                                                                            \
      size_t k = (size_t)T * n, ops = k * 3 * n;                                                              \
      R* buf = (R*)malloc(sizeof(R) * (2 * ops + 3 * (size_t)T * n * n + 2 * n * n + 8 * k + 2 * (size_t)N * nx \
                                       + 2 * n0 + 3 * (size_t)T * m + 16));                                   \
      R *S = buf, *P = S + ops, *th = P + ops, *ti = th + (size_t)T * n * n, *ph = ti + (size_t)T * n * n;     \
      R *w = ph + (size_t)T * n * n, *gam = w + 2 * n * n, *xo = gam + k, *r = xo + k, *zz = r + k;           \
      R *pp = zz + k, *sp = pp + k, *cx = sp + k, *cx0 = cx + (size_t)N * nx, *gx = cx0 + n0;                 \
      const R *Db = D + (size_t)b * T * n * n, *Eb = E + (size_t)b * N * n * n, *qb = q + (size_t)b * k;       \
      const R *A0b = A0 + (size_t)b * n0 * n, *Amb = Am + (size_t)b * N * nx * n, *Apb = Ap + (size_t)b * N * nx * n; \
      const R *c0b = c0 + (size_t)b * n0, *cb = c + (size_t)b * N * nx, *Gb = G + (size_t)b * T * m * n;      \
      const R *lb = l + (size_t)b * T * m, *ub = u + (size_t)b * T * m;                                        \
      R *xb = x + (size_t)b * k, *ygb = yg + (size_t)b * T * m, *yf0b = yf0 + (size_t)b * n0;                  \
      R *yfdb = yfd + (size_t)b * N * nx, *zgb = zg + (size_t)b * T * m;                                       \
      R rho = rho_in[b], rf = rho * (R)rho_f_factor, al = (R)alpha;                                           \
      const int direct = pcg_iters < 0;                                                                       \
      schur_##SUF(Db, Eb, A0b, Amb, Apb, Gb, T, n, nx, n0, m, rf, rho, (R)sigma, S, P, th, ti, ph, w, direct);\
      if (direct) chol_##SUF(th, ph, T, n);                                                                   \
      for (int it = 0; it < admm_iters; ++it) {                                                               \
        for (int t = 0; t < T; ++t)                                                                           \
          for (int j = 0; j < n; ++j) {                                                                       \
            R v = (R)sigma * xb[t * n + j] - qb[t * n + j];                                                   \
            if (t == 0) {                                                                                     \
              for (int kk = 0; kk < n0; ++kk) v += A0b[kk * n + j] * (rf * c0b[kk] - yf0b[kk]);               \
              for (int kk = 0; kk < nx; ++kk) v += Amb[kk * n + j] * (rf * cb[kk] - yfdb[kk]);                \
            } else {                                                                                          \
              for (int kk = 0; kk < nx; ++kk)                                                                 \
                v += Apb[((size_t)(t - 1) * nx + kk) * n + j] *                                               \
                     (rf * cb[(t - 1) * nx + kk] - yfdb[(t - 1) * nx + kk]);                                  \
              if (t < N)                                                                                      \
                for (int kk = 0; kk < nx; ++kk)                                                               \
                  v += Amb[((size_t)t * nx + kk) * n + j] * (rf * cb[t * nx + kk] - yfdb[t * nx + kk]);       \
            }                                                                                                 \
            for (int kk = 0; kk < m; ++kk)                                                                    \
              v += Gb[((size_t)t * m + kk) * n + j] * (rho * zgb[t * m + kk] - ygb[t * m + kk]);              \
            gam[t * n + j] = v;                                                                               \
          }                                                                                                   \
        memcpy(xo, xb, sizeof(R) * k);                                                                        \
        if (direct)                                                                                           \
          chol_solve_##SUF(th, ph, gam, xb, r, T, n);                                                         \
        else                                                                                                  \
          pcg_##SUF(S, P, gam, xb, T, n, pcg_iters, 0, r, zz, pp, sp);                                        \
        for (int i = 0; i < n0; ++i) cx0[i] = dot_##SUF(A0b + i * n, xb, n);                                  \
        for (int t = 0; t < N; ++t)                                                                           \
          for (int i = 0; i < nx; ++i)                                                                        \
            cx[t * nx + i] = dot_##SUF(Amb + ((size_t)t * nx + i) * n, xb + t * n, n) +                       \
                             dot_##SUF(Apb + ((size_t)t * nx + i) * n, xb + (t + 1) * n, n);                  \
        for (int t = 0; t < T; ++t)                                                                           \
          for (int i = 0; i < m; ++i) gx[t * m + i] = dot_##SUF(Gb + ((size_t)t * m + i) * n, xb + t * n, n); \
        for (size_t i = 0; i < k; ++i) xb[i] = al * xb[i] + (1 - al) * xo[i];                                 \
        for (int i = 0; i < n0; ++i) yf0b[i] += rf * al * (cx0[i] - c0b[i]);                                  \
        for (int i = 0; i < N * nx; ++i) yfdb[i] += rf * al * (cx[i] - cb[i]);                                \
        for (int i = 0; i < T * m; ++i) {                                                                     \
          R zo = zgb[i], zt = al * gx[i] + (1 - al) * zo + ygb[i] / rho;                                      \
          R cl = zt < lb[i] ? lb[i] : (zt > ub[i] ? ub[i] : zt);                                              \
          zgb[i] = cl;                                                                                        \
          ygb[i] += rho * (al * gx[i] + (1 - al) * zo - cl);                                                  \
        }                                                                                                     \
      }                                                                                                       \
      free(buf);                                                                                              \
    }                                                                                                         \
    return 0;                                                                                                 \
  }


DEFINE_ORACLE(float, f32)
DEFINE_ORACLE(double, f64)


