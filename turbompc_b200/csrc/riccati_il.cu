// Block-tridiagonal Cholesky (block Riccati recursion) factor and solve on the
// batch-interleaved layout: one problem per thread, 32 problems per warp.
//
// Batch-interleaved layout (TMPC_LAYOUT_INTERLEAVED): problems are grouped by
// 32; inside a group an array of E elements per problem is stored
// element-major and problem-minor,
//     element e of problem b  at  ((b / 32) * E + e) * 32 + b % 32,
// so when the 32 lanes of a warp (32 consecutive problems) touch the same
// element, the warp issues one fully coalesced 128-byte (fp32) or 256-byte
// (fp64) transaction.  Arrays hold ceil(Nb / 32) * 32 problem slots.
//
// Operator format (input of the factor), per problem, E = T n(n+1)/2 + N n^2:
//   Theta_t  lower triangle, row-major packed: (i, j <= i) at t tri(n) + i(i+1)/2 + j
//   Phi_t    = S(t+1, t), full row-major:    (i, k) at T tri(n) + (t n + i) n + k
// Factor format: the same shape, L_t^-1 (lower, packed) in the Theta slots and
// W_t = Phi_t L_t^-T in the Phi slots, for the block-bidiagonal L of S = L L^T
// from the recursion
//   L_0 L_0^T = Theta_0,  W_{t-1} = Phi_{t-1} L_{t-1}^-T,  L_t L_t^T = Theta_t - W_{t-1} W_{t-1}^T.
// Keeping the inverse of each diagonal factor (inverted in registers right
// after its Cholesky) turns every triangular solve into a matrix-vector
// product whose rows are independent: with one problem per thread, the
// substitution chains would otherwise leave each thread waiting on one
// memory latency per row.
// This is the direct solve that replaces the reference's cuDSS path
// (turbompc/solvers/linear_systems_solvers/csrc/cudss_blktridi.cu:60-184).
//
// Factor: each thread keeps its stage's working matrix (packed lower,
// NB(NB+1)/2 values) in registers and runs the Cholesky fully unrolled there;
// W_{t-1} is re-read from the factor it has just written (an L2 hit).
// Solve: four warps per group of 32 problems, each owning a quarter of the
// rows (see solve_kernel).  Block sizes are
// compiled for NB in {4, 8, 12, 16} (fp64: up to 12); n < NB is padded with an
// identity diagonal in registers only (memory holds exact n x n blocks).
#include "tmpc_common.cuh"

namespace tmpc {
namespace il {

constexpr int kWarp = 32;

__host__ __device__ constexpr size_t tri(size_t n) { return n * (n + 1) / 2; }
__host__ __device__ constexpr int LI(int i, int j) { return i * (i + 1) / 2 + j; }

__host__ __device__ inline size_t op_elems(int T, int n) {
  return (size_t)T * tri(n) + (size_t)(T - 1) * n * n;
}
__host__ __device__ inline size_t groups(int Nb) { return ((size_t)Nb + kWarp - 1) / kWarp; }

template <typename R>
__device__ __forceinline__ R ldro(const R* p) {
  return __ldg(p);
}

// Cholesky of the packed working matrix in registers (right-looking), then
// L^-1 in place, column by column from the last: with X = L^-1,
// X[j][j] = 1 / L[j][j] and X[i][j] = -X[j][j] sum_{k=j+1..i} X[i][k] L[k][j]
// (rows i taken from the bottom up, so the L[k][j], k <= i, they read are not
// yet overwritten).  ok turns false on a non-positive or non-finite pivot.
template <int NB, typename R>
__device__ __forceinline__ void chol_inv(R (&m)[NB * (NB + 1) / 2], bool& ok) {
#pragma unroll
  for (int k = 0; k < NB; ++k) {
    const R d = m[LI(k, k)];
    if (!(d > R(0)) || !isfinite(d)) ok = false;
    const R s = sqrt(d);
    const R inv = R(1) / s;
    m[LI(k, k)] = s;
#pragma unroll
    for (int i = k + 1; i < NB; ++i) m[LI(i, k)] *= inv;
#pragma unroll
    for (int j = k + 1; j < NB; ++j) {
#pragma unroll
      for (int i = j; i < NB; ++i) m[LI(i, j)] = fma(-m[LI(i, k)], m[LI(j, k)], m[LI(i, j)]);
    }
  }
#pragma unroll
  for (int j = NB - 1; j >= 0; --j) {
    const R xjj = R(1) / m[LI(j, j)];
    m[LI(j, j)] = xjj;
#pragma unroll
    for (int i = NB - 1; i > j; --i) {
      R acc = R(0);
#pragma unroll
      for (int k = j + 1; k <= i; ++k) acc = fma(m[LI(i, k)], m[LI(k, j)], acc);
      m[LI(i, j)] = -xjj * acc;
    }
  }
}

// ---------------------------------------------------------------------------
// Factor: one problem per thread.
// ---------------------------------------------------------------------------
template <int NB, typename R>
__device__ __forceinline__ void factor_one(const R* __restrict__ op, R* __restrict__ f, int T, int n, bool valid,
                                           bool& ok) {
  constexpr int TR = NB * (NB + 1) / 2;
  const size_t trin = tri(n);
  const size_t woff = (size_t)T * trin;
  const size_t nn = (size_t)n * n;
  R m[TR];
  for (int t = 0; t < T; ++t) {
    // M = Theta_t (identity in the padded rows / columns)
    const R* th = op + (size_t)t * trin * kWarp;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
#pragma unroll
      for (int j = 0; j <= i; ++j) {
        R v = (i == j) ? R(1) : R(0);
        if (i < n && valid) v = ldro(th + (size_t)LI(i, j) * kWarp);
        m[LI(i, j)] = v;
      }
    }
    // M -= W_{t-1} W_{t-1}^T, one column k of W_{t-1} at a time (rank-1 updates)
    if (t > 0) {
      const R* W = f + (woff + (size_t)(t - 1) * nn) * kWarp;
#pragma unroll
      for (int k = 0; k < NB; ++k) {
        if (k < n) {
          R w[NB];
#pragma unroll
          for (int i = 0; i < NB; ++i) w[i] = (i < n) ? W[((size_t)i * n + k) * kWarp] : R(0);
#pragma unroll
          for (int i = 0; i < NB; ++i) {
#pragma unroll
            for (int j = 0; j <= i; ++j) m[LI(i, j)] = fma(-w[i], w[j], m[LI(i, j)]);
          }
        }
      }
    }
    chol_inv<NB, R>(m, ok);
    // store L_t^-1
    R* lt = f + (size_t)t * trin * kWarp;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      if (i < n) {
#pragma unroll
        for (int j = 0; j <= i; ++j) lt[(size_t)LI(i, j) * kWarp] = m[LI(i, j)];
      }
    }
    // W_t = Phi_t L_t^-T: row i is L_t^-1 Phi_t[i, :]^T
    if (t < T - 1) {
      const R* ph = op + (woff + (size_t)t * nn) * kWarp;
      R* W = f + (woff + (size_t)t * nn) * kWarp;
      R xn[NB];
#pragma unroll
      for (int k = 0; k < NB; ++k) xn[k] = (k < n && valid) ? ldro(ph + (size_t)k * kWarp) : R(0);
      for (int i = 0; i < n; ++i) {
        R x[NB];
#pragma unroll
        for (int k = 0; k < NB; ++k) x[k] = xn[k];
        if (i + 1 < n) {  // next row's loads in flight during this row's product
#pragma unroll
          for (int k = 0; k < NB; ++k)
            xn[k] = (k < n && valid) ? ldro(ph + ((size_t)(i + 1) * n + k) * kWarp) : R(0);
        }
#pragma unroll
        for (int k = 0; k < NB; ++k) {
          if (k < n) {
            R acc = R(0);
#pragma unroll
            for (int c = 0; c <= k; ++c) acc = fma(m[LI(k, c)], x[c], acc);
            W[((size_t)i * n + k) * kWarp] = acc;
          }
        }
      }
    }
  }
}

// (Capping the factor at 168 registers for three blocks per SM measured slower
// at every size: 10-47 % at n = 9 and 16, fp32 and fp64.)
// One warp per block: at 200-255 registers per thread an SM holds 8 of these
// warps, and small blocks spread a modest batch over every SM (128-thread
// blocks left 20 of 148 SMs idle at 16,384 problems; the time did not change:
// each warp's chain of dependent stages sets it).
constexpr int kFactorThreads = 32;
template <int NB, typename R>
__global__ void __launch_bounds__(kFactorThreads) factor_kernel(const R* __restrict__ ops, R* __restrict__ factor,
                                                     int32_t* status, int Nb,
                                                     int T, int n) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if ((b & ~(kWarp - 1)) >= Nb) return;  // the whole warp is past the batch
  const bool valid = b < Nb;             // lanes past the batch factor the identity into the padding slots
  const size_t E = op_elems(T, n);
  const size_t base = (size_t)(b / kWarp) * E * kWarp + (b % kWarp);
  bool ok = true;
  factor_one<NB, R>(ops + base, factor + base, T, n, valid, ok);
  if (valid && status) status[b] = ok ? 0 : TMPC_STATUS_SINGULAR_BLOCK;
}

// ---------------------------------------------------------------------------
// Factor with the stage data staged in shared memory.  One warp (one group of
// 32 problems) per block.  A stage's Theta_t and Phi_t blocks are contiguous
// byte ranges of the group's interleaved operator, so the warp copies them
// with 16-byte cp.async while other work runs, and W_t = Phi_t L_t^-T is
// written over Phi_t in shared memory (row i of W needs only row i of Phi),
// where the next stage's rank update reads it.  Theta_{t+1} is requested as
// soon as Theta_t has been read into registers.  Phi is requested
//   DBL:  Phi_{t+1}, into the second of two Phi / W buffers, as soon as the
//         rank update of stage t has read W_{t-1} from it (a whole stage ahead);
//   else: Phi_t, into the one buffer, as soon as the rank update of stage t
//         has read W_{t-1} (it lands during the stage's Cholesky).
// Shared memory per block: (tri(n) + 2 n^2) or (tri(n) + n^2) x 32 values.
// Every group of copies is committed in order (an empty group where a stage
// has nothing to fetch) so that the wait counts are fixed: before Theta_t is
// read at most one group may still be in flight (DBL: Phi_t), before Phi_t is
// read two (DBL: Theta_{t+1}, Phi_{t+1}) or none.  Same arithmetic, in the
// same order, as factor_one.
// ---------------------------------------------------------------------------
constexpr size_t kSmemPerSm = 228 * 1024;  // shared memory of one SM (B200)

template <typename R>
__host__ __device__ constexpr size_t staged_smem_elems(int n, bool dbl) {
  return (tri(n) + (dbl ? 2 : 1) * (size_t)n * n) * kWarp;
}

template <int NB, typename R, bool DBL>
__global__ void __launch_bounds__(kWarp) factor_staged_kernel(const R* __restrict__ ops, R* __restrict__ factor,
                                                              int32_t* status, int Nb, int T, int n) {
  constexpr int TR = NB * (NB + 1) / 2;
  extern __shared__ __align__(16) unsigned char il_smem[];
  const int lane = threadIdx.x;
  const size_t grp = blockIdx.x;
  const bool valid = grp * kWarp + lane < (size_t)Nb;
  const size_t trin = tri(n), nn = (size_t)n * n, woff = (size_t)T * trin;
  const size_t E = op_elems(T, n);
  const R* og = ops + grp * E * kWarp;
  R* fg = factor + grp * E * kWarp;
  R* sth = reinterpret_cast<R*>(il_smem);
  R* const sb0 = sth + trin * kWarp;
  R* const sb1 = DBL ? sb0 + nn * kWarp : sb0;
  // elems interleaved values (elems x 32 R) from global src to shared dst, 16 bytes per copy
  auto fetch = [&](R* dst, const R* src, size_t elems) {
    constexpr int V = 16 / sizeof(R);
    const size_t chunks = elems * kWarp / V;
    for (size_t c = lane; c < chunks; c += kWarp) cp_async16(dst + c * V, src + c * V);
  };
  fetch(sth, og, trin);
  cp_async_commit();
  if (DBL) fetch(sb0, og + woff * kWarp, nn);
  cp_async_commit();
  bool ok = true;
  R m[TR];
  for (int t = 0; t < T; ++t) {
    R* cur = (t & 1) ? sb1 : sb0;  // Phi_t, then W_t
    R* prv = (t & 1) ? sb0 : sb1;  // W_{t-1}, then Phi_{t+1}
    cp_async_wait<1>();
    __syncwarp();
#pragma unroll
    for (int i = 0; i < NB; ++i) {
#pragma unroll
      for (int j = 0; j <= i; ++j) {
        R v = (i == j) ? R(1) : R(0);
        if (i < n && valid) v = sth[(size_t)LI(i, j) * kWarp + lane];
        m[LI(i, j)] = v;
      }
    }
    __syncwarp();  // every lane has read Theta_t
    if (t + 1 < T) fetch(sth, og + (size_t)(t + 1) * trin * kWarp, trin);
    cp_async_commit();
    if (t > 0) {
#pragma unroll
      for (int k = 0; k < NB; ++k) {
        if (k < n) {
          R w[NB];
#pragma unroll
          for (int i = 0; i < NB; ++i) w[i] = (i < n) ? prv[((size_t)i * n + k) * kWarp + lane] : R(0);
#pragma unroll
          for (int i = 0; i < NB; ++i) {
#pragma unroll
            for (int j = 0; j <= i; ++j) m[LI(i, j)] = fma(-w[i], w[j], m[LI(i, j)]);
          }
        }
      }
    }
    __syncwarp();  // every lane has read W_{t-1}
    if (DBL) {
      if (t + 1 < T - 1) fetch(prv, og + (woff + (size_t)(t + 1) * nn) * kWarp, nn);
    } else {
      if (t < T - 1) fetch(cur, og + (woff + (size_t)t * nn) * kWarp, nn);
    }
    cp_async_commit();
    chol_inv<NB, R>(m, ok);
    R* lt = fg + (size_t)t * trin * kWarp + lane;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      if (i < n) {
#pragma unroll
        for (int j = 0; j <= i; ++j) lt[(size_t)LI(i, j) * kWarp] = m[LI(i, j)];
      }
    }
    if (t < T - 1) {
      if (DBL) cp_async_wait<2>(); else cp_async_wait<0>();
      __syncwarp();
      R* W = fg + (woff + (size_t)t * nn) * kWarp + lane;
      for (int i = 0; i < n; ++i) {
        R x[NB];
#pragma unroll
        for (int k = 0; k < NB; ++k) x[k] = (k < n && valid) ? cur[((size_t)i * n + k) * kWarp + lane] : R(0);
#pragma unroll
        for (int k = 0; k < NB; ++k) {
          if (k < n) {
            R acc = R(0);
#pragma unroll
            for (int c = 0; c <= k; ++c) acc = fma(m[LI(k, c)], x[c], acc);
            W[((size_t)i * n + k) * kWarp] = acc;
            cur[((size_t)i * n + k) * kWarp + lane] = acc;
          }
        }
      }
    }
  }
  cp_async_wait<0>();
  if (valid && status) status[grp * kWarp + lane] = ok ? 0 : TMPC_STATUS_SINGULAR_BLOCK;
}

// ---------------------------------------------------------------------------
// Solve S x = b with the factor.  One block of four warps per group of 32
// problems: lane l of every warp works on problem l of the group, and warp w
// owns rows [w NB/4, (w+1) NB/4) of every stage's products, so each problem's
// rows are spread over four threads (four times the memory-level parallelism
// of one thread per problem).  The stage vectors a product needs in full go
// through shared memory, [row][lane], between barriers.  The forward sweep
// writes y into x_out (the same slots, by the thread that owns the row),
// which the backward sweep reads back.
// ---------------------------------------------------------------------------
constexpr int kSolveWarps = 4;

// (Register caps for 3 or 4 resident blocks per SM measured slower at 16,384
// problems, 1.2-2.5x, and within 1 % at 65,536.)
template <int NB, typename R>
__global__ void __launch_bounds__(32 * kSolveWarps) solve_kernel(const R* __restrict__ factor,
                                                                 const R* __restrict__ rhs, R* __restrict__ x_out,
                                                                 int Nb, int T, int n) {
  constexpr int RPW = NB / kSolveWarps;  // rows per warp
  __shared__ R ush[NB][kWarp];           // the vector being multiplied
  __shared__ R vsh[NB][kWarp];           // y_{t-1} (forward) / x_{t+1} (backward)
  const int lane = threadIdx.x & (kWarp - 1), w = threadIdx.x / kWarp;
  const size_t grp = blockIdx.x;
  const bool valid = grp * kWarp + lane < (size_t)Nb;
  const size_t trin = tri(n), nn = (size_t)n * n;
  const size_t woff = (size_t)T * trin;
  const R* F = factor + grp * op_elems(T, n) * kWarp + lane;
  const R* bv = rhs + grp * (size_t)T * n * kWarp + lane;
  R* xv = x_out + grp * (size_t)T * n * kWarp + lane;
  const int r0 = w * RPW;
#pragma unroll
  for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = R(0);
  __syncthreads();
  // Every factor row a thread needs in a stage is loaded into registers at
  // the top of the stage, before the barriers, so a stage costs one memory
  // latency (the compiler does not move loads across __syncthreads).
  // forward: y_t = L_t^-1 (b_t - W_{t-1} y_{t-1})
  for (int t = 0; t < T; ++t) {
    const R* W = F + (woff + (size_t)(t > 0 ? t - 1 : 0) * nn) * kWarp;
    const R* X = F + (size_t)t * trin * kWarp;  // L_t^-1
    R wr[RPW][NB], xr[RPW][NB], bi[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int i = r0 + r;
      const bool on = i < n && valid;
      bi[r] = on ? ldro(bv + ((size_t)t * n + i) * kWarp) : R(0);
#pragma unroll
      for (int k = 0; k < NB; ++k) {
        wr[r][k] = (on && t > 0 && k < n) ? ldro(W + ((size_t)i * n + k) * kWarp) : R(0);
        xr[r][k] = (on && k <= i) ? ldro(X + (size_t)LI(i, k) * kWarp) : R(0);
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      R u = bi[r];
#pragma unroll
      for (int k = 0; k < NB; ++k) u = fma(-wr[r][k], vsh[k][lane], u);
      ush[r0 + r][lane] = u;
    }
    __syncthreads();
    R y[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      R acc = R(0);
#pragma unroll
      for (int c = 0; c < NB; ++c) acc = fma(xr[r][c], ush[c][lane], acc);
      y[r] = acc;
      if (r0 + r < n && valid) xv[((size_t)t * n + r0 + r) * kWarp] = acc;
    }
    __syncthreads();  // every read of ush / vsh of this stage is done
#pragma unroll
    for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = y[r];
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = R(0);
  __syncthreads();
  // backward: x_t = L_t^-T (y_t - W_t^T x_{t+1}); thread row k needs column k
  // of W_t and column k of L_t^-1
  for (int t = T - 1; t >= 0; --t) {
    const R* W = F + (woff + (size_t)(t < T - 1 ? t : 0) * nn) * kWarp;
    const R* X = F + (size_t)t * trin * kWarp;
    R wc[RPW][NB], xc[RPW][NB], yi[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int k = r0 + r;
      const bool on = k < n && valid;
      yi[r] = on ? xv[((size_t)t * n + k) * kWarp] : R(0);
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        wc[r][i] = (on && t < T - 1 && i < n) ? ldro(W + ((size_t)i * n + k) * kWarp) : R(0);
        xc[r][i] = (on && i >= k && i < n) ? ldro(X + (size_t)LI(i, k) * kWarp) : R(0);
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      R u = yi[r];
#pragma unroll
      for (int i = 0; i < NB; ++i) u = fma(-wc[r][i], vsh[i][lane], u);
      ush[r0 + r][lane] = u;
    }
    __syncthreads();
    R x[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      R acc = R(0);
#pragma unroll
      for (int i = 0; i < NB; ++i) acc = fma(xc[r][i], ush[i][lane], acc);
      x[r] = acc;
      if (r0 + r < n && valid) xv[((size_t)t * n + r0 + r) * kWarp] = acc;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = x[r];
  }
}

// ---------------------------------------------------------------------------
// Solve with the stage data staged in shared memory: the same block shape and
// arithmetic as solve_kernel, but each stage's factor blocks and vector (L_t^-1,
// the W block the stage reads, and b_t or y_t) are copied by the whole block
// with 16-byte cp.async two stages ahead into one of two buffers, so no
// thread waits on global memory inside a stage.  Buffer layout: L_t^-1 (tri(n)
// values), W (n^2), the stage vector (n), each x 32 lanes.
// ---------------------------------------------------------------------------
__host__ __device__ constexpr size_t solve_stage_elems(int n) { return tri(n) + (size_t)n * n + n; }

template <int NB, typename R>
__global__ void __launch_bounds__(32 * kSolveWarps) solve_staged_kernel(const R* __restrict__ factor,
                                                                        const R* __restrict__ rhs,
                                                                        R* __restrict__ x_out, int Nb, int T,
                                                                        int n) {
  constexpr int RPW = NB / kSolveWarps;
  constexpr int V = 16 / sizeof(R);
  extern __shared__ __align__(16) unsigned char il_smem[];
  __shared__ R ush[NB][kWarp];
  __shared__ R vsh[NB][kWarp];
  const int lane = threadIdx.x & (kWarp - 1), w = threadIdx.x / kWarp;
  const size_t grp = blockIdx.x;
  const bool valid = grp * kWarp + lane < (size_t)Nb;
  const size_t trin = tri(n), nn = (size_t)n * n;
  const size_t woff = (size_t)T * trin;
  const size_t SE = solve_stage_elems(n);
  const R* F = factor + grp * op_elems(T, n) * kWarp;
  const R* bv = rhs + grp * (size_t)T * n * kWarp;
  R* xv = x_out + grp * (size_t)T * n * kWarp;
  R* const buf0 = reinterpret_cast<R*>(il_smem);
  R* const buf1 = buf0 + SE * kWarp;
  auto copy = [&](R* dst, const R* src, size_t elems) {
    const size_t chunks = elems * kWarp / V;
    for (size_t c = threadIdx.x; c < chunks; c += 32 * kSolveWarps) cp_async16(dst + c * V, src + c * V);
  };
  // stage t's data into dst: forward reads W_{t-1} and b_t, backward W_t and y_t
  auto fetch = [&](R* dst, int t, bool fwd) {
    copy(dst, F + (size_t)t * trin * kWarp, trin);
    const int wt = fwd ? t - 1 : t;
    if (wt >= 0 && wt < T - 1) copy(dst + trin * kWarp, F + (woff + (size_t)wt * nn) * kWarp, nn);
    copy(dst + (trin + nn) * kWarp, (fwd ? bv : xv) + (size_t)t * n * kWarp, n);
  };
  const int r0 = w * RPW;
#pragma unroll
  for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = R(0);
  fetch(buf0, 0, true);
  cp_async_commit();
  fetch(buf1, 1, true);
  cp_async_commit();
  // forward: y_t = L_t^-1 (b_t - W_{t-1} y_{t-1})
  for (int t = 0; t < T; ++t) {
    const R* B = (t & 1) ? buf1 : buf0;
    cp_async_wait<1>();
    __syncthreads();
    const R* X = B + lane;
    const R* W = B + trin * kWarp + lane;
    const R* vb = B + (trin + nn) * kWarp + lane;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int i = r0 + r;
      const bool on = i < n && valid;
      R u = on ? vb[(size_t)i * kWarp] : R(0);
      if (t > 0) {
#pragma unroll
        for (int k = 0; k < NB; ++k)
          if (on && k < n) u = fma(-W[((size_t)i * n + k) * kWarp], vsh[k][lane], u);
      }
      ush[i][lane] = u;
    }
    __syncthreads();
    R y[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int i = r0 + r;
      const bool on = i < n && valid;
      R acc = R(0);
#pragma unroll
      for (int c = 0; c < NB; ++c)
        if (on && c <= i) acc = fma(X[(size_t)LI(i, c) * kWarp], ush[c][lane], acc);
      y[r] = acc;
      if (on) xv[((size_t)t * n + i) * kWarp + lane] = acc;
    }
    __syncthreads();  // every read of ush, vsh and this stage's buffer is done; y_t is stored
#pragma unroll
    for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = y[r];
    if (t + 2 < T) fetch(const_cast<R*>(B), t + 2, true);
    cp_async_commit();
  }
  cp_async_wait<0>();
  __syncthreads();
#pragma unroll
  for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = R(0);
  fetch(buf0, T - 1, false);
  cp_async_commit();
  fetch(buf1, T - 2, false);
  cp_async_commit();
  // backward: x_t = L_t^-T (y_t - W_t^T x_{t+1}); thread row k needs column k
  // of W_t and of L_t^-1
  for (int t = T - 1; t >= 0; --t) {
    const R* B = ((T - 1 - t) & 1) ? buf1 : buf0;
    cp_async_wait<1>();
    __syncthreads();
    const R* X = B + lane;
    const R* W = B + trin * kWarp + lane;
    const R* yb = B + (trin + nn) * kWarp + lane;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int k = r0 + r;
      const bool on = k < n && valid;
      R u = on ? yb[(size_t)k * kWarp] : R(0);
      if (t < T - 1) {
#pragma unroll
        for (int i = 0; i < NB; ++i)
          if (on && i < n) u = fma(-W[((size_t)i * n + k) * kWarp], vsh[i][lane], u);
      }
      ush[k][lane] = u;
    }
    __syncthreads();
    R x[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int k = r0 + r;
      const bool on = k < n && valid;
      R acc = R(0);
#pragma unroll
      for (int i = 0; i < NB; ++i)
        if (on && i >= k && i < n) acc = fma(X[(size_t)LI(i, k) * kWarp], ush[i][lane], acc);
      x[r] = acc;
      if (on) xv[((size_t)t * n + k) * kWarp + lane] = acc;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RPW; ++r) vsh[r0 + r][lane] = x[r];
    if (t - 2 >= 0) fetch(const_cast<R*>(B), t - 2, false);
    cp_async_commit();
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Layout conversion: [Nb][E] problem-major <-> interleaved, through a 32 x 32
// shared-memory tile (coalesced on both sides).  With a gather map, element e
// of the interleaved array takes the problem-major element src(e).
// ---------------------------------------------------------------------------
struct IdentityMap {
  __device__ size_t operator()(size_t e) const { return e; }
};
// Reference-layout S [T][n][3n] -> operator format (Theta lower packed, Phi).
struct SchurMap {
  int T, n;
  __device__ size_t operator()(size_t e) const {
    const size_t trin = tri(n);
    const size_t n3 = 3 * (size_t)n;
    if (e < (size_t)T * trin) {
      const size_t t = e / trin;
      size_t r = e - t * trin;
      size_t i = (size_t)((sqrtf(8.f * (float)r + 1.f) - 1.f) * 0.5f);
      while (i * (i + 1) / 2 > r) --i;
      while ((i + 1) * (i + 2) / 2 <= r) ++i;
      const size_t j = r - i * (i + 1) / 2;
      return (t * n + i) * n3 + n + j;  // Theta_t[i][j] = S[t][i][n + j]
    }
    const size_t e2 = e - (size_t)T * trin;
    const size_t nn = (size_t)n * n;
    const size_t t = e2 / nn, rem = e2 - t * nn;
    const size_t i = rem / n, k = rem - i * n;
    return ((t + 1) * n + i) * n3 + k;  // Phi_t[i][k] = S[t+1][i][k]
  }
};

template <typename R, class Map>
__global__ void __launch_bounds__(256) interleave_kernel(const R* __restrict__ in, R* out, int Nb, size_t E_in,
                                                         size_t E, Map map) {
  __shared__ R tile[32][33];
  const size_t grp = blockIdx.y;
  const size_t e0 = (size_t)blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int r = ty; r < 32; r += 8) {
    const size_t b = grp * 32 + r, e = e0 + tx;
    tile[r][tx] = (b < (size_t)Nb && e < E) ? in[b * E_in + map(e)] : R(0);
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const size_t e = e0 + r;
    if (e < E) out[(grp * E + e) * 32 + tx] = tile[tx][r];
  }
}

template <typename R>
__global__ void __launch_bounds__(256) deinterleave_kernel(const R* __restrict__ in, R* out, int Nb, size_t E) {
  __shared__ R tile[32][33];
  const size_t grp = blockIdx.y;
  const size_t e0 = (size_t)blockIdx.x * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int r = ty; r < 32; r += 8) {
    const size_t e = e0 + r;
    tile[r][tx] = e < E ? in[(grp * E + e) * 32 + tx] : R(0);
  }
  __syncthreads();
  for (int r = ty; r < 32; r += 8) {
    const size_t b = grp * 32 + r, e = e0 + tx;
    if (b < (size_t)Nb && e < E) out[b * E + e] = tile[tx][r];
  }
}

inline bool grid_ok(int Nb, size_t E) { return groups(Nb) <= 65535 && (E + 31) / 32 <= 0x7fffffffu; }

template <typename R, class Map>
int interleave(int Nb, size_t E_in, size_t E, const R* in, R* out, Map map, cudaStream_t st) {
  if (Nb < 0) return TMPC_ERR_BAD_DIMS;
  if (Nb == 0 || E == 0) return TMPC_OK;
  if (!in || !out) return TMPC_ERR_NULL_ARG;
  if (!grid_ok(Nb, E)) return TMPC_ERR_BAD_DIMS;
  dim3 grid((unsigned)((E + 31) / 32), (unsigned)groups(Nb)), block(32, 8);
  interleave_kernel<R, Map><<<grid, block, 0, st>>>(in, out, Nb, E_in, E, map);
  return (int)cudaPeekAtLastError();
}

template <typename R>
int deinterleave(int Nb, size_t E, const R* in, R* out, cudaStream_t st) {
  if (Nb < 0) return TMPC_ERR_BAD_DIMS;
  if (Nb == 0 || E == 0) return TMPC_OK;
  if (!in || !out) return TMPC_ERR_NULL_ARG;
  if (!grid_ok(Nb, E)) return TMPC_ERR_BAD_DIMS;
  dim3 grid((unsigned)((E + 31) / 32), (unsigned)groups(Nb)), block(32, 8);
  deinterleave_kernel<R><<<grid, block, 0, st>>>(in, out, Nb, E);
  return (int)cudaPeekAtLastError();
}

template <typename R>
constexpr int max_nb() {
  return sizeof(R) == 4 ? 16 : 12;
}

template <typename R, class F>
int dispatch_il(int n, F&& f) {
  if (n <= 4) return f(std::integral_constant<int, 4>{});
  if (n <= 8) return f(std::integral_constant<int, 8>{});
  if (n <= 12) return f(std::integral_constant<int, 12>{});
  if constexpr (max_nb<R>() >= 16) {
    if (n <= 16) return f(std::integral_constant<int, 16>{});
  }
  return TMPC_ERR_UNSUPPORTED;
}

int check(const TmpcDims* d) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 2 || d->n < 1) return TMPC_ERR_BAD_DIMS;
  return TMPC_OK;
}

template <typename R>
int factor(const TmpcDims* d, const R* ops, R* fac, int32_t* status, cudaStream_t st) {
  int rc = check(d);
  if (rc) return rc;
  if (d->n > max_nb<R>()) return TMPC_ERR_UNSUPPORTED;
  if (d->Nb == 0) return TMPC_OK;
  if (!ops || !fac) return TMPC_ERR_NULL_ARG;
  return dispatch_il<R>(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    // The staged kernel needs 16-byte aligned operator / factor arrays and its
    // stage buffers within one block's shared memory; otherwise the factor
    // reads straight from global memory.  Two Phi / W buffers (Phi_{t+1}
    // fetched a whole stage ahead) where they still leave eight warps per SM
    // (n = 9 fp32), else one buffer (Phi_t fetched during the stage's
    // Cholesky) for twice the resident warps: measured faster at every other
    // size (n = 9 fp64, n = 12 and 16 fp32, 16,384 and 65,536 problems).
    const bool dbl = 8 * staged_smem_elems<R>(d->n, true) * sizeof(R) <= kSmemPerSm;
    const size_t smem = staged_smem_elems<R>(d->n, dbl) * sizeof(R);
    const bool aligned = ((reinterpret_cast<uintptr_t>(ops) | reinterpret_cast<uintptr_t>(fac)) & 15) == 0;
    if (aligned && (long)smem <= max_dyn_smem()) {
      auto k = dbl ? factor_staged_kernel<NB, R, true> : factor_staged_kernel<NB, R, false>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
      k<<<(unsigned)groups(d->Nb), kWarp, smem, st>>>(ops, fac, status, d->Nb, d->T, d->n);
      return (int)cudaPeekAtLastError();
    }
    const int grid = (int)((groups(d->Nb) * kWarp + kFactorThreads - 1) / kFactorThreads);
    factor_kernel<NB, R><<<grid, kFactorThreads, 0, st>>>(ops, fac, status, d->Nb, d->T, d->n);
    return (int)cudaPeekAtLastError();
  });
}

template <typename R>
int solve(const TmpcDims* d, const R* fac, const R* rhs, R* x, cudaStream_t st) {
  int rc = check(d);
  if (rc) return rc;
  if (d->n > max_nb<R>()) return TMPC_ERR_UNSUPPORTED;
  if (d->Nb == 0) return TMPC_OK;
  if (!fac || !rhs || !x) return TMPC_ERR_NULL_ARG;
  return dispatch_il<R>(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    const int grid = (int)groups(d->Nb);  // one block of kSolveWarps warps per group of 32 problems
    // Staged solve where the arrays are 16-byte aligned and two stage buffers
    // fit one block's shared memory (1.3-2.2x faster than solve_kernel at
    // n = 9 to 16); otherwise the loads go straight to global memory.
    const size_t smem = 2 * solve_stage_elems(d->n) * kWarp * sizeof(R);
    const bool aligned =
        ((reinterpret_cast<uintptr_t>(fac) | reinterpret_cast<uintptr_t>(rhs) | reinterpret_cast<uintptr_t>(x)) & 15) == 0;
    if (aligned && (long)smem <= max_dyn_smem()) {
      auto k = solve_staged_kernel<NB, R>;
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return (int)e;
      k<<<grid, 32 * kSolveWarps, smem, st>>>(fac, rhs, x, d->Nb, d->T, d->n);
      return (int)cudaPeekAtLastError();
    }
    solve_kernel<NB, R><<<grid, 32 * kSolveWarps, 0, st>>>(fac, rhs, x, d->Nb, d->T, d->n);
    return (int)cudaPeekAtLastError();
  });
}

}  // namespace il
}  // namespace tmpc

extern "C" {

size_t tmpc_interleaved_elems(int32_t Nb, int64_t elems_per_problem) {
  if (Nb <= 0 || elems_per_problem <= 0) return 0;
  return tmpc::il::groups(Nb) * tmpc::il::kWarp * (size_t)elems_per_problem;
}

int64_t tmpc_riccati_il_elems_per_problem(const TmpcDims* dims) {
  if (tmpc::il::check(dims)) return 0;
  return (int64_t)tmpc::il::op_elems(dims->T, dims->n);
}

int32_t tmpc_interleave_f32(int32_t Nb, int64_t elems, const float* src, float* dst, tmpc_stream_t stream) {
  if (elems < 0) return TMPC_ERR_BAD_DIMS;
  return tmpc::il::interleave<float>(Nb, (size_t)elems, (size_t)elems, src, dst, tmpc::il::IdentityMap{},
                                     (cudaStream_t)stream);
}
int32_t tmpc_interleave_f64(int32_t Nb, int64_t elems, const double* src, double* dst, tmpc_stream_t stream) {
  if (elems < 0) return TMPC_ERR_BAD_DIMS;
  return tmpc::il::interleave<double>(Nb, (size_t)elems, (size_t)elems, src, dst, tmpc::il::IdentityMap{},
                                      (cudaStream_t)stream);
}
int32_t tmpc_deinterleave_f32(int32_t Nb, int64_t elems, const float* src, float* dst, tmpc_stream_t stream) {
  if (elems < 0) return TMPC_ERR_BAD_DIMS;
  return tmpc::il::deinterleave<float>(Nb, (size_t)elems, src, dst, (cudaStream_t)stream);
}
int32_t tmpc_deinterleave_f64(int32_t Nb, int64_t elems, const double* src, double* dst, tmpc_stream_t stream) {
  if (elems < 0) return TMPC_ERR_BAD_DIMS;
  return tmpc::il::deinterleave<double>(Nb, (size_t)elems, src, dst, (cudaStream_t)stream);
}

int32_t tmpc_schur_interleave_f32(const TmpcDims* dims, const float* S, float* ops, tmpc_stream_t stream) {
  int rc = tmpc::il::check(dims);
  if (rc) return rc;
  const size_t Es = (size_t)dims->T * dims->n * 3 * dims->n;
  return tmpc::il::interleave<float>(dims->Nb, Es, tmpc::il::op_elems(dims->T, dims->n), S, ops,
                                     tmpc::il::SchurMap{dims->T, dims->n}, (cudaStream_t)stream);
}
int32_t tmpc_schur_interleave_f64(const TmpcDims* dims, const double* S, double* ops, tmpc_stream_t stream) {
  int rc = tmpc::il::check(dims);
  if (rc) return rc;
  const size_t Es = (size_t)dims->T * dims->n * 3 * dims->n;
  return tmpc::il::interleave<double>(dims->Nb, Es, tmpc::il::op_elems(dims->T, dims->n), S, ops,
                                      tmpc::il::SchurMap{dims->T, dims->n}, (cudaStream_t)stream);
}

int32_t tmpc_riccati_factor_il_f32(const TmpcDims* dims, const float* ops, float* factor, int32_t* status,
                                   tmpc_stream_t stream) {
  return tmpc::il::factor<float>(dims, ops, factor, status, (cudaStream_t)stream);
}
int32_t tmpc_riccati_factor_il_f64(const TmpcDims* dims, const double* ops, double* factor, int32_t* status,
                                   tmpc_stream_t stream) {
  return tmpc::il::factor<double>(dims, ops, factor, status, (cudaStream_t)stream);
}
int32_t tmpc_riccati_solve_il_f32(const TmpcDims* dims, const float* factor, const float* rhs, float* x,
                                  tmpc_stream_t stream) {
  return tmpc::il::solve<float>(dims, factor, rhs, x, (cudaStream_t)stream);
}
int32_t tmpc_riccati_solve_il_f64(const TmpcDims* dims, const double* factor, const double* rhs, double* x,
                                  tmpc_stream_t stream) {
  return tmpc::il::solve<double>(dims, factor, rhs, x, (cudaStream_t)stream);
}

}  // extern "C"
