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
    // Cholesky in registers (right-looking)
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
    // L_t^-1 in place, column by column from the last: with X = L^-1,
    // X[j][j] = 1 / L[j][j] and X[i][j] = -X[j][j] sum_{k=j+1..i} X[i][k] L[k][j]
    // (rows i taken from the bottom up, so the L[k][j], k <= i, they read
    // are not yet overwritten).
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
