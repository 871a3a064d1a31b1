// Library-level C ABI entry points (version, error strings) and host helpers.
#include <cuda_runtime.h>

#include "tma.cuh"
#include "tmpc_common.cuh"

namespace tmpc {

int check_dims(const TmpcDims* d) {
  if (!d) return TMPC_ERR_NULL_ARG;
  if (d->Nb < 0 || d->T < 2 || d->n < 1 || d->nx < 1 || d->nx > d->n || d->n0 < 0 || d->m < 0)
    return TMPC_ERR_BAD_DIMS;
  return TMPC_OK;
}

int max_dyn_smem() {
  int dev = 0, v = 48 * 1024;
  if (cudaGetDevice(&dev) != cudaSuccess) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 48 * 1024;
  return v;
}

int max_sm_smem() {
  int dev = 0, v = 100 * 1024;
  if (cudaGetDevice(&dev) != cudaSuccess) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev) != cudaSuccess) v = 100 * 1024;
  return v;
}

}  // namespace tmpc

extern "C" {

int32_t tmpc_version(void) { return 100; }

uint32_t tmpc_set_transfer_poll_limit(uint32_t polls) { return tmpc::transfer_poll_limit().exchange(polls); }

const char* tmpc_error_string(int32_t code) {
  switch (code) {
    case TMPC_OK: return "ok";
    case TMPC_ERR_NULL_ARG: return "null pointer argument";
    case TMPC_ERR_BAD_DIMS: return "invalid dimensions";
    case TMPC_ERR_UNSUPPORTED:
      return "unsupported configuration (block size n beyond the entry point's limit: 96 for the fused PCG "
             "solve and the reference-layout assembly / PCG, 32 for the other operator formats and the direct "
             "solve; or an unknown option)";
    case TMPC_ERR_WORKSPACE: return "workspace or factor buffer missing, too small or not 16-byte aligned";
    case TMPC_ERR_SMEM: return "problem does not fit the shared-memory budget of one CTA";
    case TMPC_ERR_SCRATCH_LIMIT:
      return "batch needs more scratch than the fixed device buffer of tmpc_admm_solve_fixed_scratch_f64 holds "
             "(64 MiB); split the batch or use tmpc_admm_solve_f64 with a workspace";
  }
  if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
  return "unknown error";
}

}  // extern "C"
