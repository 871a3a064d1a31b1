// Fused ADMM solve for callers that cannot allocate device memory.
//
// tmpc_admm_solve_f64 takes a caller-owned workspace for problems whose
// Schur operators do not fit in one CTA's shared memory.  Some callers cannot
// provide one: code running inside a framework or runtime that owns every
// allocation (a custom-call handler that may only use the buffers it is
// given, a stream-captured region, an embedded controller with a fixed memory
// plan) must not call cudaMalloc.  This file gives them one entry point whose
// scratch lives in a fixed, statically allocated device array.
//
// The array below is part of the library image: every GPU that loads the
// library holds its kTmpcFixedScratchBytes until the process exits.  In host
// code its name is only a host-side stand-in, never a device address, so the
// address is looked up with cudaGetSymbolAddress once per device (with that
// device current) on the first call made on that device, and cached.  The
// cached address belongs to the device's primary context: after
// cudaDeviceReset (or anything else that destroys that context) it is stale,
// and the process must not call this entry point on that device again.
#include <mutex>

#include "launchers.cuh"

namespace tmpc {

constexpr size_t kTmpcFixedScratchBytes = size_t(64) << 20;  // 64 MiB per device
static __device__ __align__(256) unsigned char g_fixed_scratch[kTmpcFixedScratchBytes];

template <typename R>
int admm_solve(const TmpcDims* d, const TmpcQP* qp, const TmpcAdmmState* in, const TmpcAdmmState* out,
               const R* slack_weight, const TmpcAdmmConfig* cfg, R* x_out, uint32_t* iters_out, int32_t* status_out,
               void* ws, size_t ws_bytes, cudaStream_t st);  // admm_fused.cu
template <typename R>
size_t admm_ws_bytes_cfg(const TmpcDims& d, const TmpcAdmmConfig* cfg);  // admm_fused.cu

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices] = {};

// Device address of g_fixed_scratch on the current device (set-up on first use).
int fixed_scratch_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return TMPC_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fixed_scratch);
    if (e != cudaSuccess) return (int)e;
    g_ptr[dev] = p;
  }
  *out = g_ptr[dev];
  return TMPC_OK;
}
}  // namespace

}  // namespace tmpc

extern "C" int32_t tmpc_admm_solve_fixed_scratch_f64(const TmpcDims* dims, const TmpcQP* qp,
                                                     const TmpcAdmmState* state_in, const TmpcAdmmState* state_out,
                                                     const double* slack_weight, const TmpcAdmmConfig* cfg,
                                                     double* x_out, uint32_t* iters_out, int32_t* status_out,
                                                     tmpc_stream_t stream) {
  int rc = tmpc::check_dims(dims);
  if (rc) return rc;
  const size_t need = tmpc::admm_ws_bytes_cfg<double>(*dims, cfg);
  if (need > tmpc::kTmpcFixedScratchBytes) return TMPC_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  if (need > 0) {
    rc = tmpc::fixed_scratch_ptr(&ws);
    if (rc) return rc;
  }
  // Every scratch byte the kernel reads is written earlier in the same call
  // (the operators are re-assembled on entry), so nothing needs clearing.
  return tmpc::admm_solve<double>(dims, qp, state_in, state_out, slack_weight, cfg, x_out, iters_out, status_out,
                                  ws, need, (cudaStream_t)stream);
}
