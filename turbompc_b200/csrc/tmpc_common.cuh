// Shared device-side building blocks of the B200 inner solve.
//
// Layout conventions (all per problem, problem-major in HBM):
//   * QP inputs arrive in the reference layout (see include/tmpc_b200.h).
//   * Block vectors live on chip as [T][VSTR] with the NB-padded stage block
//     in the first NB entries; entries n..NB-1 are kept exactly zero.
//   * The Schur operator S and the preconditioner Phiinv are held in a
//     "packed" form: T diagonal blocks as the upper triangle (row-major,
//     NB-padded, symmetric) followed by N sub-diagonal blocks
//     L_t = M(t+1, t) stored full and row-major.  Every block is padded so
//     that its byte stride is an odd multiple of 16: eight consecutive
//     threads reading the same offset of eight consecutive blocks with
//     128-bit loads then hit eight distinct 16-byte bank groups.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "tmpc_b200.h"

namespace tmpc {

constexpr int kMaxThreads = 512;

// Threads per CTA of the per-problem kernels: 512 for block sizes up to 16;
// 256 for larger blocks, whose register-resident block tasks need up to 255
// registers per thread.
__host__ __device__ constexpr int max_threads_for(int nb) { return nb <= 16 ? 512 : 256; }
// One thread per matvec task (T diagonal + 4N quarter blocks), rounded to warps.
inline int cta_threads(int T, int maxt) {
  int th = ((T + 4 * (T - 1)) + 31) / 32 * 32;
  if (th < 64) th = 64;
  if (th > maxt) th = maxt;
  return th;
}

__host__ __device__ constexpr int tri_size(int nb) { return nb * (nb + 1) / 2; }

// Smallest element count >= elems whose byte size is an odd multiple of 16.
__host__ __device__ constexpr int skew_stride(int elems, int esize) {
  int chunks = (elems * esize + 15) / 16;
  if ((chunks & 1) == 0) chunks += 1;
  return chunks * 16 / esize;
}

// Packed upper-triangle index of (i, j), i <= j, in an nb x nb block.
__host__ __device__ constexpr int tri_index(int i, int j, int nb) {
  return i * nb - (i * (i - 1)) / 2 + (j - i);
}
// Row / column of packed index idx (runtime loops; used outside hot loops).
__host__ __device__ inline int tri_row(int idx, int nb) {
  int i = 0;
  while (idx >= nb - i) {
    idx -= nb - i;
    ++i;
  }
  return i;
}
__host__ __device__ inline int tri_col(int idx, int nb) {
  int i = 0;
  while (idx >= nb - i) {
    idx -= nb - i;
    ++i;
  }
  return i + idx;
}

// Layout of the per-CTA reduction region ("red") of the fused ADMM kernels:
// [0, 352) an 11 x 32 table of per-warp partial maxima for the residual check
// (also the block_sum slots of the packed PCG), residual scalars at 352, the
// register-resident kernel's dot-product slots at 368.
constexpr int kRedSc = 352;
constexpr int kRedSlots = 368;
constexpr int kRedSize = 400;

template <int NB, typename R>
struct Geo {
  static constexpr int VEC = 16 / (int)sizeof(R);                // elements per 128-bit load
  static constexpr int TRI = tri_size(NB);
  static constexpr int DSTR = skew_stride(TRI, sizeof(R));       // diagonal block stride
  static constexpr int OSTR = skew_stride(NB * NB, sizeof(R));   // sub-diagonal block stride
  static constexpr int VSTR = skew_stride(NB, sizeof(R));        // block-vector row stride
  static_assert(NB % VEC == 0, "NB must be a multiple of the 128-bit vector width");
  __host__ __device__ static size_t op_elems(int T) { return (size_t)T * DSTR + (size_t)(T - 1) * OSTR; }
};

// Host-side block size selection: the smallest compiled NB >= n.
inline int pick_nb(int n) {
  if (n <= 8) return 8;
  if (n <= 12) return 12;
  if (n <= 16) return 16;
  if (n <= 24) return 24;
  if (n <= 32) return 32;
  return -1;
}

// 128-bit load of VEC consecutive elements into w[].
template <typename R>
__device__ __forceinline__ void ld128(R* w, const R* p) {
  if constexpr (sizeof(R) == 4) {
    float4 v = *reinterpret_cast<const float4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
    double2 v = *reinterpret_cast<const double2*>(p);
    w[0] = v.x; w[1] = v.y;
  }
}
template <typename R>
__device__ __forceinline__ void st128(R* p, const R* w) {
  if constexpr (sizeof(R) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(w[0], w[1], w[2], w[3]);
  } else {
    *reinterpret_cast<double2*>(p) = make_double2(w[0], w[1]);
  }
}
// Read-only global 128-bit load through the non-coherent path.
template <typename R>
__device__ __forceinline__ void ldg128(R* w, const R* p) {
  if constexpr (sizeof(R) == 4) {
    float4 v = __ldg(reinterpret_cast<const float4*>(p));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else {
    double2 v = __ldg(reinterpret_cast<const double2*>(p));
    w[0] = v.x; w[1] = v.y;
  }
}
template <bool SMEM, typename R>
__device__ __forceinline__ void ldop(R* w, const R* p) {
  if constexpr (SMEM) ld128(w, p); else ldg128(w, p);
}

template <typename R>
__device__ __forceinline__ R warp_sum(R v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
template <typename R>
__device__ __forceinline__ R warp_max(R v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum returned to every thread.  `slots` holds >= 32 entries and
// must not be reused until after the caller's next __syncthreads().
// Deterministic: fixed reduction order independent of timing.
template <typename R>
__device__ __forceinline__ R block_sum(R v, R* slots) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) slots[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  R s = R(0);
  for (int w = 0; w < nw; ++w) s += slots[w];
  return s;
}
template <typename R>
__device__ __forceinline__ R block_max(R v, R* slots) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) slots[wid] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  R s = R(0);
  for (int w = 0; w < nw; ++w) s = fmax(s, slots[w]);
  return s;
}

// Per-problem views of the reference-layout QP.
template <typename R>
struct QPView {
  const R* D;   // [T][n][n]
  const R* E;   // [N][n][n]
  const R* q;   // [T][n]
  const R* A0;  // [n0][n]
  const R* Am;  // [N][nx][n]
  const R* Ap;  // [N][nx][n]
  const R* c0;  // [n0]
  const R* c;   // [N][nx]
  const R* G;   // [T][m][n]
  const R* l;   // [T][m]
  const R* u;   // [T][m]
};

template <typename R>
__device__ __forceinline__ QPView<R> qp_view(const TmpcQP& qp, int b, int T, int n, int nx, int n0, int m) {
  const int N = T - 1;
  QPView<R> v;
  v.D = static_cast<const R*>(qp.D) + (size_t)b * T * n * n;
  v.E = static_cast<const R*>(qp.E) + (size_t)b * N * n * n;
  v.q = qp.q ? static_cast<const R*>(qp.q) + (size_t)b * T * n : nullptr;
  v.A0 = n0 > 0 ? static_cast<const R*>(qp.A0) + (size_t)b * n0 * n : nullptr;
  v.Am = static_cast<const R*>(qp.A_minus) + (size_t)b * N * nx * n;
  v.Ap = static_cast<const R*>(qp.A_plus) + (size_t)b * N * nx * n;
  v.c0 = (n0 > 0 && qp.c0) ? static_cast<const R*>(qp.c0) + (size_t)b * n0 : nullptr;
  v.c = qp.c ? static_cast<const R*>(qp.c) + (size_t)b * N * nx : nullptr;
  v.G = m > 0 ? static_cast<const R*>(qp.G) + (size_t)b * T * m * n : nullptr;
  v.l = (m > 0 && qp.l) ? static_cast<const R*>(qp.l) + (size_t)b * T * m : nullptr;
  v.u = (m > 0 && qp.u) ? static_cast<const R*>(qp.u) + (size_t)b * T * m : nullptr;
  return v;
}

int check_dims(const TmpcDims* d);  // capi.cu
int max_dyn_smem();                 // capi.cu: opt-in shared memory per block of the current device
int max_sm_smem();                  // capi.cu: shared memory per SM of the current device

// Calls f(std::integral_constant<int, NB>) for the compiled block size of n.
template <typename F>
int dispatch_nb(int n, F&& f) {
  switch (pick_nb(n)) {
    case 8: return f(std::integral_constant<int, 8>{});
    case 12: return f(std::integral_constant<int, 12>{});
    case 16: return f(std::integral_constant<int, 16>{});
    case 24: return f(std::integral_constant<int, 24>{});
    case 32: return f(std::integral_constant<int, 32>{});
  }
  return TMPC_ERR_UNSUPPORTED;
}

// Asynchronous 16-byte global -> shared copies (cp.async, cached in L2 only),
// committed in groups and waited for by group count; no registers are held
// while the copies are in flight.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(a), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

}  // namespace tmpc
