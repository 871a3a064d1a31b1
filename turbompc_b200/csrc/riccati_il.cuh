#pragma once
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
__global__ void __launch_bounds__(kWarp) factor_staged_kernel(const R* ops, R* factor, int32_t* status,
                                                              const int* gate, int Nb, int T, int n) {
  constexpr int TR = NB * (NB + 1) / 2;
  extern __shared__ __align__(16) unsigned char il_smem[];
  if (gate && *gate == 0) return;  // nothing to refactor
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
// Layout conversion: [Nb][E] problem-major <-> interleaved, through a 32 x 32
// shared-memory tile (coalesced on both sides).  With a gather map, element e
// of the interleaved array takes the problem-major element src(e).  With
// skip, groups whose skip flag is set are left unconverted.
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

// Each block converts kConvTiles consecutive 32-element tiles of one group
// (all loads of the block issued before its stores).
constexpr int kConvTiles = 4;

template <typename R, class Map>
__global__ void __launch_bounds__(256) interleave_kernel(const R* __restrict__ in, R* out, int Nb, size_t E_in,
                                                         size_t E, Map map, const int* skip) {
  __shared__ R tile[kConvTiles][32][33];
  const size_t grp = blockIdx.y;
  if (skip && skip[grp]) return;
  const size_t e0 = (size_t)blockIdx.x * 32 * kConvTiles;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int k = 0; k < kConvTiles; ++k)
#pragma unroll
    for (int r = ty; r < 32; r += 8) {
      const size_t b = grp * 32 + r, e = e0 + (size_t)k * 32 + tx;
      tile[k][r][tx] = (b < (size_t)Nb && e < E) ? in[b * E_in + map(e)] : R(0);
    }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kConvTiles; ++k)
#pragma unroll
    for (int r = ty; r < 32; r += 8) {
      const size_t e = e0 + (size_t)k * 32 + r;
      if (e < E) out[(grp * E + e) * 32 + tx] = tile[k][tx][r];
    }
}

template <typename R>
__global__ void __launch_bounds__(256) deinterleave_kernel(const R* __restrict__ in, R* out, int Nb, size_t E) {
  __shared__ R tile[kConvTiles][32][33];
  const size_t grp = blockIdx.y;
  const size_t e0 = (size_t)blockIdx.x * 32 * kConvTiles;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int k = 0; k < kConvTiles; ++k)
#pragma unroll
    for (int r = ty; r < 32; r += 8) {
      const size_t e = e0 + (size_t)k * 32 + r;
      tile[k][r][tx] = e < E ? in[(grp * E + e) * 32 + tx] : R(0);
    }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kConvTiles; ++k)
#pragma unroll
    for (int r = ty; r < 32; r += 8) {
      const size_t b = grp * 32 + r, e = e0 + (size_t)k * 32 + tx;
      if (b < (size_t)Nb && e < E) out[b * E + e] = tile[k][tx][r];
    }
}

inline bool grid_ok(int Nb, size_t E) {
  return groups(Nb) <= 65535 && (E + 32 * kConvTiles - 1) / (32 * kConvTiles) <= 0x7fffffffu;
}

template <typename R, class Map>
int interleave(int Nb, size_t E_in, size_t E, const R* in, R* out, Map map, cudaStream_t st,
               const int* skip = nullptr) {
  if (Nb < 0) return TMPC_ERR_BAD_DIMS;
  if (Nb == 0 || E == 0) return TMPC_OK;
  if (!in || !out) return TMPC_ERR_NULL_ARG;
  if (!grid_ok(Nb, E)) return TMPC_ERR_BAD_DIMS;
  dim3 grid((unsigned)((E + 32 * kConvTiles - 1) / (32 * kConvTiles)), (unsigned)groups(Nb)), block(32, 8);
  interleave_kernel<R, Map><<<grid, block, 0, st>>>(in, out, Nb, E_in, E, map, skip);
  return (int)cudaPeekAtLastError();
}

template <typename R>
int deinterleave(int Nb, size_t E, const R* in, R* out, cudaStream_t st) {
  if (Nb < 0) return TMPC_ERR_BAD_DIMS;
  if (Nb == 0 || E == 0) return TMPC_OK;
  if (!in || !out) return TMPC_ERR_NULL_ARG;
  if (!grid_ok(Nb, E)) return TMPC_ERR_BAD_DIMS;
  dim3 grid((unsigned)((E + 32 * kConvTiles - 1) / (32 * kConvTiles)), (unsigned)groups(Nb)), block(32, 8);
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

// Factor launch: the staged kernel where the arrays are 16-byte aligned and its
// stage buffers fit one block's shared memory, else factor_kernel (global
// memory; no gate).  Two Phi / W buffers (Phi_{t+1}
// fetched a whole stage ahead) where they still leave eight warps per SM
// (n = 9 fp32), else one buffer (Phi_t fetched during the stage's Cholesky)
// for twice the resident warps: measured faster at every other size (n = 9
// fp64, n = 12 and 16 fp32, 16,384 and 65,536 problems).
template <int NB, typename R>
int launch_factor(int Nb, int T, int n, const R* ops, R* fac, int32_t* status, const int* gate, cudaStream_t st) {
  const bool dbl = 8 * staged_smem_elems<R>(n, true) * sizeof(R) <= kSmemPerSm;
  const size_t smem = staged_smem_elems<R>(n, dbl) * sizeof(R);
  const bool aligned = ((reinterpret_cast<uintptr_t>(ops) | reinterpret_cast<uintptr_t>(fac)) & 15) == 0;
  if (aligned && (long)smem <= max_dyn_smem()) {
    auto k = dbl ? factor_staged_kernel<NB, R, true> : factor_staged_kernel<NB, R, false>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    k<<<(unsigned)groups(Nb), kWarp, smem, st>>>(ops, fac, status, gate, Nb, T, n);
    return (int)cudaPeekAtLastError();
  }
  if (gate) return TMPC_ERR_UNSUPPORTED;
  const int grid = (int)((groups(Nb) * kWarp + kFactorThreads - 1) / kFactorThreads);
  factor_kernel<NB, R><<<grid, kFactorThreads, 0, st>>>(ops, fac, status, Nb, T, n);
  return (int)cudaPeekAtLastError();
}

}  // namespace il
}  // namespace tmpc
