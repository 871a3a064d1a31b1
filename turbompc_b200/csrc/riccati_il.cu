// Stand-alone entry points of the batch-interleaved block-Cholesky solve: the
// solve kernels, the factor / solve dispatch and the C ABI (kernels and
// layout shared with admm_il.cu are in riccati_il.cuh).
#include "riccati_il.cuh"

namespace tmpc {
namespace il {

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
    return launch_factor<NB, R>(d->Nb, d->T, d->n, ops, fac, status, nullptr, st);
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
