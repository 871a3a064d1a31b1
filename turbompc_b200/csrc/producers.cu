// QP producers of the benchmark problems that are not dynamics rows, batched
// over (problem, stage), one thread per pair:
//
//  * spherical obstacle rows (turbompc/problems/obstacle_avoidance.py:16-52,
//    linearised as get_inequalities_linearized_matrices does,
//    optimal_control_problem.py:580-626):
//        g_k  = 1 - ||p - c_k|| / (r_k + 0.001),  p = x[:dim]
//        G_k  = dg_k/dz = -(p - c_k) / ||p - c_k|| / (r_k + 0.001) on the first
//               dim columns, 0 elsewhere
//        l_k  = -1e9 - (g_k - G_k z),  u_k = 0 - (g_k - G_k z)
//    every row multiplied by row_scale (1 / mean(state_diff[:dim]) under
//    variable rescaling, else 1); the distance is clamped at 1e-12;
//  * the learned (MLP) stage cost of benchmark configuration 5,
//    s * w2 . tanh(W1 z + b1) on every stage, quadratised exactly and added
//    to the tracking blocks in place:
//        a = W1 z + b1, th = tanh(a), d = 1 - th^2
//        grad = s W1^T (w2 * d),   H = s W1^T diag(w2 * (-2 th d)) W1
//        D_t += H,   q_t += grad - H z
//    (get_cost_linearized_blocks, optimal_control_problem.py:1068-1174, for a
//    stage-separable cost: q = gradient - Hessian z);
//  * the inequality rows at an iterate, g_t = G_t z_t (+ slack), optionally
//    clamped to [l, u] (the initial z_g of admm.py:1051-1088, and the g of
//    the SQP's active-set identification, turbompc_solver.py:1387-1439).
#include <cuda_runtime.h>
#include <math.h>

#include "tmpc_common.cuh"

namespace tmpc {
namespace prod {

template <typename R>
__global__ void __launch_bounds__(256) obstacle_kernel(const R* __restrict__ states, const R* __restrict__ centers,
                                                      const R* __restrict__ radii, R row_scale, R* G, R* lo, R* hi,
                                                      int Nb, int T, int nx, int n, int K, int dim) {
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t total = (size_t)Nb * T * K;
  if (idx >= total) return;
  const int k = (int)(idx % K);
  const size_t bt = idx / K;
  const int b = (int)(bt / T);
  const R* x = states + bt * nx;
  const R* c = centers + ((size_t)b * K + k) * dim;
  const R rk = radii[(size_t)b * K + k] + R(0.001);
  R d2 = R(0);
  for (int i = 0; i < dim; ++i) {
    const R v = x[i] - c[i];
    d2 += v * v;
  }
  const R dist = sqrt(d2);
  const R dc = dist > R(1e-12) ? dist : R(1e-12);
  const R g = R(1) - dist / rk;
  R* Grow = G + idx * n;
  R gz = R(0);
  for (int j = 0; j < n; ++j) {
    R v = R(0);
    if (j < dim) {
      v = -(x[j] - c[j]) / dc / rk;
      gz += v * x[j];
    }
    Grow[j] = v * row_scale;
  }
  const R off = g - gz;
  lo[idx] = (R(-1e9) - off) * row_scale;
  hi[idx] = (R(0) - off) * row_scale;
}

// One thread per (problem, stage); W1 (H x n), b1, w2 staged in shared memory.
template <int NB, typename R>
__global__ void __launch_bounds__(128) mlp_kernel(const R* __restrict__ states, const R* __restrict__ controls,
                                                 const R* __restrict__ W1, const R* __restrict__ b1,
                                                 const R* __restrict__ w2, R s, R* D, R* q, int Nb, int T, int nx,
                                                 int nu, int H) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  R* sW = reinterpret_cast<R*>(smem_raw);
  const int n = nx + nu;
  R* sb = sW + H * n;
  R* sw = sb + H;
  for (int e = threadIdx.x; e < H * n; e += blockDim.x) sW[e] = W1[e];
  for (int e = threadIdx.x; e < H; e += blockDim.x) {
    sb[e] = b1[e];
    sw[e] = w2[e];
  }
  __syncthreads();
  const size_t bt = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (bt >= (size_t)Nb * T) return;
  R z[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    z[i] = R(0);
    if (i < nx) z[i] = states[bt * nx + i];
    else if (i < n) z[i] = controls[bt * nu + (i - nx)];
  }
  constexpr int TR = NB * (NB + 1) / 2;
  R h[TR], g[NB];
#pragma unroll
  for (int e = 0; e < TR; ++e) h[e] = R(0);
#pragma unroll
  for (int i = 0; i < NB; ++i) g[i] = R(0);
  for (int k = 0; k < H; ++k) {
    const R* wk = sW + k * n;
    R a = sb[k];
#pragma unroll
    for (int i = 0; i < NB; ++i)
      if (i < n) a = fma(wk[i], z[i], a);
    const R th = tanh(a);
    const R d = R(1) - th * th;
    const R gc = s * sw[k] * d;
    const R hc = s * sw[k] * (R(-2) * th * d);
    R w[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) w[i] = i < n ? wk[i] : R(0);
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      g[i] = fma(gc, w[i], g[i]);
      const R hw = hc * w[i];
#pragma unroll
      for (int j = 0; j <= i; ++j) h[i * (i + 1) / 2 + j] = fma(hw, w[j], h[i * (i + 1) / 2 + j]);
    }
  }
  R* Dt = D + bt * n * n;
  R* qt = q + bt * n;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    if (i < n) {
      R hz = R(0);
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        if (j < n) {
          const R hij = j <= i ? h[i * (i + 1) / 2 + j] : h[j * (j + 1) / 2 + i];
          Dt[i * n + j] += hij;
          hz = fma(hij, z[j], hz);
        }
      }
      qt[i] += g[i] - hz;
    }
  }
}

int check(const TmpcDims* d) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 1 || d->n < 1 || d->nx < 1 || d->nx > d->n) return TMPC_ERR_BAD_DIMS;
  return TMPC_OK;
}

template <typename R>
int obstacle_rows(const TmpcDims* d, int dim, int K, const R* states, const R* centers, const R* radii,
                  double row_scale, R* G, R* lo, R* hi, cudaStream_t st) {
  int rc = check(d);
  if (rc) return rc;
  if (K < 0 || dim < 1 || dim > d->nx) return TMPC_ERR_BAD_DIMS;
  const size_t total = (size_t)d->Nb * d->T * K;
  if (total == 0) return TMPC_OK;
  if (!states || !centers || !radii || !G || !lo || !hi) return TMPC_ERR_NULL_ARG;
  const unsigned grid = (unsigned)((total + 255) / 256);
  obstacle_kernel<R><<<grid, 256, 0, st>>>(states, centers, radii, (R)row_scale, G, lo, hi, d->Nb, d->T, d->nx, d->n,
                                           K, dim);
  return (int)cudaPeekAtLastError();
}

template <typename R>
int mlp_cost_blocks(const TmpcDims* d, int H, const R* states, const R* controls, const R* W1, const R* b1,
                    const R* w2, double scale, R* D, R* q, cudaStream_t st) {
  int rc = check(d);
  if (rc) return rc;
  if (H < 1) return TMPC_ERR_BAD_DIMS;
  if (d->n > 16) return TMPC_ERR_UNSUPPORTED;
  const size_t total = (size_t)d->Nb * d->T;
  if (total == 0) return TMPC_OK;
  if (!states || !controls || !W1 || !b1 || !w2 || !D || !q) return TMPC_ERR_NULL_ARG;
  const size_t smem = (size_t)H * (d->n + 2) * sizeof(R);
  if ((long)smem > max_dyn_smem()) return TMPC_ERR_SMEM;
  const unsigned grid = (unsigned)((total + 127) / 128);
  auto launch = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    kern<<<grid, 128, smem, st>>>(states, controls, W1, b1, w2, (R)scale, D, q, d->Nb, d->T, d->nx, d->n - d->nx, H);
    return (int)cudaPeekAtLastError();
  };
  if (d->n <= 8) return launch(mlp_kernel<8, R>);
  if (d->n <= 12) return launch(mlp_kernel<12, R>);
  return launch(mlp_kernel<16, R>);
}

// Thread per inequality row (problem, stage, row): the row's n entries
// against the stage's n values of z (two contiguous runs per thread).
template <typename R>
__global__ void __launch_bounds__(256) ineq_rows_kernel(const R* __restrict__ G, const R* __restrict__ z,
                                                       const R* __restrict__ slack, const R* __restrict__ lo,
                                                       const R* __restrict__ hi, R* out, size_t rows, int m,
                                                       int n) {
  const size_t r = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const R* g = G + r * n;
  const R* x = z + (r / m) * n;
  R s = R(0);
#pragma unroll 4
  for (int k = 0; k < n; ++k) s = fma(g[k], x[k], s);
  if (slack) s += slack[r];
  if (lo) s = fmin(fmax(s, lo[r]), hi[r]);
  out[r] = s;
}

template <typename R>
int ineq_rows(const TmpcDims* d, const R* G, const R* z, const R* slack, const R* lo, const R* hi, R* out,
              cudaStream_t st) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 1 || d->n < 1 || d->m < 0) return TMPC_ERR_BAD_DIMS;  // nx, n0 unused
  const size_t rows = (size_t)d->Nb * d->T * d->m;
  if (rows == 0) return TMPC_OK;
  if (!G || !z || !out || (lo == nullptr) != (hi == nullptr)) return TMPC_ERR_NULL_ARG;
  ineq_rows_kernel<R><<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(G, z, slack, lo, hi, out, rows, d->m, d->n);
  return (int)cudaPeekAtLastError();
}

}  // namespace prod
}  // namespace tmpc

extern "C" {

int32_t tmpc_obstacle_rows_f32(const TmpcDims* dims, int32_t dim, int32_t n_obstacles, const float* states,
                               const float* centers, const float* radii, double row_scale, float* G, float* l,
                               float* u, tmpc_stream_t stream) {
  return tmpc::prod::obstacle_rows<float>(dims, dim, n_obstacles, states, centers, radii, row_scale, G, l, u,
                                          (cudaStream_t)stream);
}
int32_t tmpc_obstacle_rows_f64(const TmpcDims* dims, int32_t dim, int32_t n_obstacles, const double* states,
                               const double* centers, const double* radii, double row_scale, double* G, double* l,
                               double* u, tmpc_stream_t stream) {
  return tmpc::prod::obstacle_rows<double>(dims, dim, n_obstacles, states, centers, radii, row_scale, G, l, u,
                                           (cudaStream_t)stream);
}
int32_t tmpc_mlp_cost_blocks_f32(const TmpcDims* dims, int32_t hidden, const float* states, const float* controls,
                                 const float* W1, const float* b1, const float* w2, double scale, float* D, float* q,
                                 tmpc_stream_t stream) {
  return tmpc::prod::mlp_cost_blocks<float>(dims, hidden, states, controls, W1, b1, w2, scale, D, q,
                                            (cudaStream_t)stream);
}
int32_t tmpc_mlp_cost_blocks_f64(const TmpcDims* dims, int32_t hidden, const double* states,
                                 const double* controls, const double* W1, const double* b1, const double* w2,
                                 double scale, double* D, double* q, tmpc_stream_t stream) {
  return tmpc::prod::mlp_cost_blocks<double>(dims, hidden, states, controls, W1, b1, w2, scale, D, q,
                                             (cudaStream_t)stream);
}
int32_t tmpc_ineq_rows_f32(const TmpcDims* dims, const float* G, const float* z, const float* slack, const float* l,
                           const float* u, float* g_out, tmpc_stream_t stream) {
  return tmpc::prod::ineq_rows<float>(dims, G, z, slack, l, u, g_out, (cudaStream_t)stream);
}
int32_t tmpc_ineq_rows_f64(const TmpcDims* dims, const double* G, const double* z, const double* slack,
                           const double* l, const double* u, double* g_out, tmpc_stream_t stream) {
  return tmpc::prod::ineq_rows<double>(dims, G, z, slack, l, u, g_out, (cudaStream_t)stream);
}

}  // extern "C"
