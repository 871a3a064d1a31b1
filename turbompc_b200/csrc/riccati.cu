// Standalone batched block-tridiagonal Cholesky factor / solve entry points
// (the direct linear-system backend; replaces cudss_blktridi_cuda,
// turbompc/solvers/linear_systems_solvers/csrc/cudss_ffi.cc:76-98).
#include "riccati.cuh"
#include "tmpc_common.cuh"

namespace tmpc {

constexpr int kRicWarps = 4;
// Lanes per problem: NB <= 16 runs two problems per warp (16-lane groups);
// one problem per warp would leave at least half of every warp idle.
template <int NB>
constexpr int ric_group() {
  return NB <= 16 ? 16 : 32;
}
// Warps per block: up to 4 within 40 KB of static shared memory (one
// scratch area per group).
template <int NB, typename R>
constexpr int ric_warps() {
  constexpr int per = riccati_scratch_elems<NB>() * (int)sizeof(R) * (32 / ric_group<NB>());
  constexpr int w = 40960 / per;
  return w < 1 ? 1 : (w > kRicWarps ? kRicWarps : w);
}

// Factor straight from the reference-layout S (no copy into the factor
// slots first).  One group of ric_group<NB>() lanes per problem.
template <int NB, typename R>
__device__ __forceinline__ void riccati_factor_body(const R* __restrict__ S, R* factor, int32_t* status, int Nb,
                                                    int T, int n) {
  using Gm = Geo<NB, R>;
  constexpr int G = ric_group<NB>();
  constexpr int GPB = ric_warps<NB, R>() * (32 / G);  // groups (problems) per block
  __shared__ __align__(16) R Msh[GPB][riccati_scratch_elems<NB>()];
  const int grp = threadIdx.x / G, gl = threadIdx.x & (G - 1);
  const int first_in_warp = blockIdx.x * GPB + (threadIdx.x >> 5) * (32 / G);
  if (first_in_warp >= Nb) return;  // the whole warp is past the batch
  int b = blockIdx.x * GPB + grp;
  const bool valid = b < Nb;  // a spare half-warp repeats the last problem without storing
  if (!valid) b = Nb - 1;
  const size_t opn = Gm::op_elems(T);
  const FactorView<NB, R> F{factor + (size_t)b * opn, T};
  const RefSrc<R> src{S + (size_t)b * T * n * 3 * n, n};  // Theta / Phi read straight from S
  const bool ok = riccati_factor_warp<NB, R, RefSrc<R>, G>(F, Msh[grp], n, src, valid);
  if (gl == 0 && status && valid) status[b] = ok ? 0 : TMPC_STATUS_SINGULAR_BLOCK;
}

template <int NB, typename R>
__global__ void __launch_bounds__(32 * kRicWarps) riccati_factor_kernel(const R* __restrict__ S, R* factor,
                                                                        int32_t* status, int Nb, int T, int n) {
  riccati_factor_body<NB, R>(S, factor, status, Nb, T, n);
}

// The fp32 32-wide factor capped at 128 registers (4 resident blocks of 4
// warps per SM instead of 3 at 137 registers): 8 % faster at n = 32, T = 129
// on B200 (latency-bound: the extra warps hide more of the dependent chains).
// The other instances keep the compiler's own register choice; asking them for
// a minimum block count measured slower.
__global__ void __launch_bounds__(32 * kRicWarps, 4) riccati_factor_kernel_f32_nb32(const float* __restrict__ S,
                                                                                    float* factor, int32_t* status,
                                                                                    int Nb, int T, int n) {
  riccati_factor_body<32, float>(S, factor, status, Nb, T, n);
}

// One group of ric_group<NB>() lanes per problem (32 / G problems per
// one-warp block); each group stages its b / y / x in shared memory as [T][VSTR].
template <int NB, typename R>
__global__ void __launch_bounds__(32) riccati_solve_kernel(const R* __restrict__ factor, const R* __restrict__ rhs,
                                                           R* x_out, int Nb, int T, int n) {
  using Gm = Geo<NB, R>;
  constexpr int G = ric_group<NB>();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int grp = threadIdx.x / G, gl = threadIdx.x & (G - 1);
  int b = blockIdx.x * (32 / G) + grp;
  const bool valid = b < Nb;  // a spare half-warp solves the last problem again and stores nothing
  if (!valid) b = Nb - 1;
  const size_t VS = (size_t)T * Gm::VSTR;
  R* sm = reinterpret_cast<R*>(smem_raw) + grp * 3 * VS;
  R* bb = sm;
  R* y = sm + VS;
  R* x = sm + 2 * VS;
  for (size_t e = gl; e < 3 * VS; e += G) sm[e] = R(0);
  __syncwarp();
  for (int e = gl; e < T * n; e += G) {
    const int t = e / n, j = e - t * n;
    bb[t * Gm::VSTR + j] = rhs[(size_t)b * T * n + e];
  }
  __syncwarp();
  const FactorView<NB, R> F{const_cast<R*>(factor) + (size_t)b * Gm::op_elems(T), T};
  riccati_solve_warp<NB, R, true, G>(F, bb, y, x);
  if (!valid) return;
  for (int e = gl; e < T * n; e += G) {
    const int t = e / n, j = e - t * n;
    x_out[(size_t)b * T * n + e] = x[t * Gm::VSTR + j];
  }
}

template <typename R>
int riccati_factor(const TmpcDims* d, const R* S, void* factor, int32_t* status, cudaStream_t st) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 2 || d->n < 1) return TMPC_ERR_BAD_DIMS;
  if (d->Nb == 0) return TMPC_OK;
  if (!S || !factor) return TMPC_ERR_NULL_ARG;
  if ((reinterpret_cast<uintptr_t>(factor) & 15) != 0) return TMPC_ERR_WORKSPACE;  // 128-bit stores of W
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    constexpr int WPB = ric_warps<NB, R>();  // the kernel indexes its scratch by group: launch exactly WPB warps
    constexpr int GPB = WPB * (32 / ric_group<NB>());
    const int grid = (d->Nb + GPB - 1) / GPB;
    if constexpr (NB == 32 && sizeof(R) == 4) {
      // (the casts are no-ops here: R is float; they keep the fp64 instance compiling)
      riccati_factor_kernel_f32_nb32<<<grid, 32 * WPB, 0, st>>>(reinterpret_cast<const float*>(S),
                                                                static_cast<float*>(factor), status, d->Nb, d->T,
                                                                d->n);
    } else {
      riccati_factor_kernel<NB, R><<<grid, 32 * WPB, 0, st>>>(S, static_cast<R*>(factor), status, d->Nb, d->T, d->n);
    }
    return (int)cudaPeekAtLastError();
  });
}

template <typename R>
int riccati_solve(const TmpcDims* d, const void* factor, const R* rhs, R* x, cudaStream_t st) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 2 || d->n < 1) return TMPC_ERR_BAD_DIMS;
  if (d->Nb == 0) return TMPC_OK;
  if (!factor || !rhs || !x) return TMPC_ERR_NULL_ARG;
  return dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    constexpr int GPB = 32 / ric_group<NB>();  // problems per one-warp block
    const size_t smem = GPB * 3 * (size_t)d->T * Geo<NB, R>::VSTR * sizeof(R);
    if ((long)smem > max_dyn_smem()) return (int)TMPC_ERR_SMEM;
    auto k = riccati_solve_kernel<NB, R>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    k<<<(d->Nb + GPB - 1) / GPB, 32, smem, st>>>(static_cast<const R*>(factor), rhs, x, d->Nb, d->T, d->n);
    return (int)cudaPeekAtLastError();
  });
}

}  // namespace tmpc

extern "C" {

size_t tmpc_riccati_factor_bytes(const TmpcDims* d, int32_t dtype_bytes) {
  if (!d || d->Nb < 0 || d->T < 2 || d->n < 1) return 0;
  size_t out = 0;
  tmpc::dispatch_nb(d->n, [&](auto tag) {
    constexpr int NB = decltype(tag)::value;
    out = dtype_bytes == 8 ? (size_t)d->Nb * tmpc::Geo<NB, double>::op_elems(d->T) * sizeof(double)
                           : (size_t)d->Nb * tmpc::Geo<NB, float>::op_elems(d->T) * sizeof(float);
    return 0;
  });
  return out;
}

int32_t tmpc_riccati_factor_f32(const TmpcDims* dims, const float* S, void* factor, int32_t* status_out,
                                tmpc_stream_t stream) {
  return tmpc::riccati_factor<float>(dims, S, factor, status_out, (cudaStream_t)stream);
}
int32_t tmpc_riccati_factor_f64(const TmpcDims* dims, const double* S, void* factor, int32_t* status_out,
                                tmpc_stream_t stream) {
  return tmpc::riccati_factor<double>(dims, S, factor, status_out, (cudaStream_t)stream);
}
int32_t tmpc_riccati_solve_f32(const TmpcDims* dims, const void* factor, const float* rhs, float* x_out,
                               tmpc_stream_t stream) {
  return tmpc::riccati_solve<float>(dims, factor, rhs, x_out, (cudaStream_t)stream);
}
int32_t tmpc_riccati_solve_f64(const TmpcDims* dims, const void* factor, const double* rhs, double* x_out,
                               tmpc_stream_t stream) {
  return tmpc::riccati_solve<double>(dims, factor, rhs, x_out, (cudaStream_t)stream);
}

}  // extern "C"
