// Register-resident fused ADMM kernel (16-wide stage blocks, fp32): launcher.
#include "admm_rows.cuh"

namespace tmpc {

bool admm_rows_ok(int T, int n, int nx, int n0, int m) {
  if (!admm_rows_applicable(T, n, nx, n0, m)) return false;
  // The kernel must fit on one SM (registers of rows_threads(T) threads + shared memory).
  const size_t smem = admm_rows_smem_bytes(T, n, nx, n0, m);
  auto k = rows_cap(T) == 52 ? admm_rows_kernel<52> : admm_rows_kernel<64>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, rows_threads(T), smem) != cudaSuccess) return false;
  return blocks >= 1;
}

int launch_admm_rows(const AdmmParams<float>& P, cudaStream_t st) {
  if (!admm_rows_applicable(P.T, P.n, P.nx, P.n0, P.m)) return TMPC_ERR_UNSUPPORTED;
  const size_t smem = admm_rows_smem_bytes(P.T, P.n, P.nx, P.n0, P.m);
  auto k = rows_cap(P.T) == 52 ? admm_rows_kernel<52> : admm_rows_kernel<64>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  k<<<P.Nb, rows_threads(P.T), smem, st>>>(P);
  return (int)cudaPeekAtLastError();
}

}  // namespace tmpc

#ifdef TMPC_ROWS_PROFILE
extern "C" int32_t tmpc_debug_rows_profile(unsigned long long* out16, int32_t reset) {
  cudaError_t e = cudaMemcpyFromSymbol(out16, tmpc::g_rows_prof, sizeof(unsigned long long) * 16);
  if (e == cudaSuccess && reset) {
    unsigned long long z[16] = {};
    e = cudaMemcpyToSymbol(tmpc::g_rows_prof, z, sizeof(z));
  }
  return (int32_t)e;
}
#endif
