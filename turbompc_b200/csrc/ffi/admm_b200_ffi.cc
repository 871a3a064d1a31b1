// XLA FFI handlers that put the b200 fused ADMM solve behind the reference's
// FFI target contracts, so the reference's Python adapters can call them
// unchanged after registering these symbols under its target names:
//   `admm_fused_cuda` / `admm_fused_cuda_f64` (turbompc/solvers/admm/csrc/
//     admm_ffi.cc:150-274; adapter admm/admm_ffi_backend.py:271-430): the same
//     21 operands, 17 attributes and 12 results, in the same order -> the
//     b200 PCG solve (AdmmB200Cuda[F64]);
//   `admm_cudss_cuda` / `admm_cudss_cuda_f64` (admm/csrc/admm_cudss_ffi.cc:
//     142-256, the reference's default forward backend): 20 operands, 15
//     attributes and 10 results -> the b200 direct (block-Cholesky) solve
//     (AdmmB200DirectCuda[F64]).  That contract has no workspace result (the
//     reference's cuDSS path keeps process-global caches), so the handler
//     takes its workspace and status words from XLA's scratch allocator.
//
// Compiled only where the jaxlib FFI headers exist (python -m
// turbompc_b200.build --ffi <jaxlib include dir>); neither this build
// environment nor the GPU image has them, so without them this file compiles
// to nothing.
//
// Mapping onto the C ABI (include/tmpc_b200.h, tmpc_admm_solve_f32/f64):
//   * S and Phiinv are not read: the b200 kernel assembles the Schur operator
//     and its preconditioner from the QP on the GPU (for the same rho_bar,
//     sigma and rho_f_factor the reference used to build them).
//   * The S_work and Phiinv_work results ([Nb, T, n, 4n] and [Nb, T, n, 3n],
//     owned by XLA) are the kernel's workspace when its operators do not fit
//     on chip, and hold the per-problem status words (int32, at the start of
//     Phiinv_work).  Their contents are unspecified afterwards, as in the
//     reference.
//   * kernel_ns_out is zero-filled (the reference writes raw clock64 cycles).
//   * x_out and x_blocks_out both receive the primal solution.
// Errors: bad shapes -> InvalidArgument; a launch error -> Internal, with the
// library's message (the reference's pcg_ffi.cc:37-78, 108-111 convention).
#if defined(__has_include)
#if __has_include("xla/ffi/api/ffi.h")
#define TMPC_HAVE_XLA_FFI 1
#endif
#endif

#ifdef TMPC_HAVE_XLA_FFI

#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "tmpc_b200.h"
#include "xla/ffi/api/c_api.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

template <ffi::DataType DT>
using Buf = ffi::Buffer<DT>;
using BufU32 = ffi::Buffer<ffi::DataType::U32>;

template <typename R>
struct Api;
template <>
struct Api<float> {
  static int32_t solve(const TmpcDims* d, const TmpcQP* qp, const TmpcAdmmState* in, const TmpcAdmmState* out,
                       const void* sw, const TmpcAdmmConfig* cfg, void* x, uint32_t* it, int32_t* st, void* ws,
                       size_t wsb, void* stream) {
    return tmpc_admm_solve_f32(d, qp, in, out, static_cast<const float*>(sw), cfg, static_cast<float*>(x), it, st,
                               ws, wsb, stream);
  }
};
template <>
struct Api<double> {
  static int32_t solve(const TmpcDims* d, const TmpcQP* qp, const TmpcAdmmState* in, const TmpcAdmmState* out,
                       const void* sw, const TmpcAdmmConfig* cfg, void* x, uint32_t* it, int32_t* st, void* ws,
                       size_t wsb, void* stream) {
    return tmpc_admm_solve_f64(d, qp, in, out, static_cast<const double*>(sw), cfg, static_cast<double*>(x), it,
                               st, ws, wsb, stream);
  }
};

template <ffi::DataType DT, typename R>
ffi::Error AdmmB200Impl(cudaStream_t stream, Buf<DT> S, Buf<DT> /*Phiinv*/, Buf<DT> D, Buf<DT> E, Buf<DT> q,
                        Buf<DT> A0, Buf<DT> A_minus, Buf<DT> A_plus, Buf<DT> G, Buf<DT> l, Buf<DT> u, Buf<DT> c0,
                        Buf<DT> c_dyn, Buf<DT> x0, Buf<DT> z_g0, Buf<DT> y_g0, Buf<DT> y_f_0, Buf<DT> y_f_dyn,
                        Buf<DT> xi_g0, Buf<DT> rho_bar, Buf<DT> slack_weight, int64_t max_iter,
                        int64_t pcg_max_iter, int64_t check_every, double eps_abs, double eps_rel, double sigma,
                        double rho_f_factor, double alpha, double pcg_eps, int64_t nx, int64_t n0, int64_t m,
                        int64_t use_slack, int64_t adapt_rho_every, double adaptive_rho_tolerance, double rho_min,
                        double rho_max, ffi::Result<Buf<DT>> x_out, ffi::Result<BufU32> iters_out,
                        ffi::Result<Buf<DT>> x_blocks_out, ffi::Result<Buf<DT>> z_g_out,
                        ffi::Result<Buf<DT>> y_g_out, ffi::Result<Buf<DT>> y_f_0_out,
                        ffi::Result<Buf<DT>> y_f_dyn_out, ffi::Result<Buf<DT>> xi_g_out,
                        ffi::Result<Buf<DT>> rho_bar_out, ffi::Result<Buf<DT>> kernel_ns_out,
                        ffi::Result<Buf<DT>> S_work, ffi::Result<Buf<DT>> Phiinv_work) {
  // Batch and block sizes from S: [Nb, T, n, 3n] or [T, n, 3n] (one problem).
  const auto sd = S.dimensions();
  TmpcDims d{};
  if (sd.size() == 4) {
    d.Nb = static_cast<int32_t>(sd[0]);
    d.T = static_cast<int32_t>(sd[1]);
    d.n = static_cast<int32_t>(sd[2]);
  } else if (sd.size() == 3) {
    d.Nb = 1;
    d.T = static_cast<int32_t>(sd[0]);
    d.n = static_cast<int32_t>(sd[1]);
  } else {
    return ffi::Error::InvalidArgument("S must be [T, n, 3n] or [Nb, T, n, 3n]");
  }
  d.nx = static_cast<int32_t>(nx);
  d.n0 = static_cast<int32_t>(n0);
  d.m = static_cast<int32_t>(m);
  if (sd[sd.size() - 1] != 3 * sd[sd.size() - 2])
    return ffi::Error::InvalidArgument("S's last dimension must be 3n");
  const int64_t N = d.T - 1;
  auto expect = [&](const auto& b, int64_t per, const char* name) -> std::string {
    return static_cast<int64_t>(b.element_count()) == per * d.Nb ? std::string() : std::string(name);
  };
  const char* bad = nullptr;
  std::string e;
  if (!(e = expect(D, (int64_t)d.T * d.n * d.n, "D")).empty() ||
      !(e = expect(E, N * d.n * d.n, "E")).empty() || !(e = expect(q, (int64_t)d.T * d.n, "q")).empty() ||
      !(e = expect(A0, (int64_t)d.n0 * d.n, "A0")).empty() ||
      !(e = expect(A_minus, N * d.nx * d.n, "A_minus")).empty() ||
      !(e = expect(A_plus, N * d.nx * d.n, "A_plus")).empty() ||
      !(e = expect(G, (int64_t)d.T * d.m * d.n, "G")).empty() ||
      !(e = expect(l, (int64_t)d.T * d.m, "l")).empty() || !(e = expect(u, (int64_t)d.T * d.m, "u")).empty() ||
      !(e = expect(c0, d.n0, "c0")).empty() || !(e = expect(c_dyn, N * d.nx, "c_dyn")).empty() ||
      !(e = expect(x0, (int64_t)d.T * d.n, "x0")).empty() || !(e = expect(rho_bar, 1, "rho_bar")).empty())
    bad = e.c_str();
  if (bad) return ffi::Error::InvalidArgument(std::string("operand ") + bad + " has the wrong size");

  TmpcQP qp{D.typed_data(), E.typed_data(), q.typed_data(), A0.typed_data(), A_minus.typed_data(),
            A_plus.typed_data(), c0.typed_data(), c_dyn.typed_data(), d.m ? G.typed_data() : nullptr,
            d.m ? l.typed_data() : nullptr, d.m ? u.typed_data() : nullptr};
  TmpcAdmmState in{x0.typed_data(), y_g0.typed_data(), y_f_0.typed_data(), y_f_dyn.typed_data(),
                   z_g0.typed_data(), xi_g0.typed_data(), rho_bar.typed_data()};
  TmpcAdmmState out{x_blocks_out->typed_data(), y_g_out->typed_data(), y_f_0_out->typed_data(),
                    y_f_dyn_out->typed_data(), z_g_out->typed_data(), xi_g_out->typed_data(),
                    rho_bar_out->typed_data()};
  TmpcAdmmConfig cfg{};
  cfg.max_iter = static_cast<int32_t>(max_iter);
  cfg.pcg_max_iter = static_cast<int32_t>(pcg_max_iter);
  cfg.check_every = static_cast<int32_t>(check_every);
  cfg.adapt_rho_every = static_cast<int32_t>(adapt_rho_every);
  cfg.eps_abs = eps_abs;
  cfg.eps_rel = eps_rel;
  cfg.sigma = sigma;
  cfg.rho_f_factor = rho_f_factor;
  cfg.alpha = alpha;
  cfg.pcg_eps = pcg_eps;
  cfg.adaptive_rho_tolerance = adaptive_rho_tolerance;
  cfg.rho_min = rho_min;
  cfg.rho_max = rho_max;
  cfg.use_slack = static_cast<int32_t>(use_slack != 0);
  cfg.linsys = TMPC_LINSYS_PCG;

  // Workspace: S_work; status words: the head of Phiinv_work.
  const size_t need = tmpc_admm_workspace_bytes(&d, static_cast<int32_t>(sizeof(R)), &cfg);
  const size_t have = S_work->element_count() * sizeof(R);
  if (need > have) return ffi::Error::InvalidArgument("S_work is smaller than the b200 workspace");
  if (Phiinv_work->element_count() * sizeof(R) < sizeof(int32_t) * static_cast<size_t>(d.Nb))
    return ffi::Error::InvalidArgument("Phiinv_work cannot hold the status words");
  int32_t* status = reinterpret_cast<int32_t*>(Phiinv_work->untyped_data());

  int32_t rc = Api<R>::solve(&d, &qp, &in, &out, use_slack ? slack_weight.typed_data() : nullptr, &cfg,
                             x_out->typed_data(), iters_out->typed_data(), status, need ? S_work->untyped_data() : nullptr,
                             need, stream);
  if (rc < 0) return ffi::Error::InvalidArgument(std::string("b200 ADMM: ") + tmpc_error_string(rc));
  if (rc > 0) return ffi::Error::Internal(std::string("b200 ADMM: ") + tmpc_error_string(rc));
  cudaError_t ce = cudaMemsetAsync(kernel_ns_out->untyped_data(), 0, kernel_ns_out->element_count() * sizeof(R),
                                   stream);
  if (ce != cudaSuccess) return ffi::Error::Internal(std::string("CUDA error: ") + cudaGetErrorString(ce));
  return ffi::Error::Success();
}

template <ffi::DataType DT, typename R>
XLA_FFI_Error* Call(XLA_FFI_CallFrame* frame) {
  static auto* handler = ffi::Ffi::Bind()
                             .Ctx<ffi::PlatformStream<cudaStream_t>>()
                             // S, Phiinv, D, E, q, A0, A_minus, A_plus, G, l, u, c0, c_dyn
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             // x0, z_g0, y_g0, y_f_0, y_f_dyn, xi_g0, rho_bar, slack_weight
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Attr<int64_t>("max_iter")
                             .Attr<int64_t>("pcg_max_iter")
                             .Attr<int64_t>("check_every")
                             .Attr<double>("eps_abs")
                             .Attr<double>("eps_rel")
                             .Attr<double>("sigma")
                             .Attr<double>("rho_f_factor")
                             .Attr<double>("alpha")
                             .Attr<double>("pcg_eps")
                             .Attr<int64_t>("nx")
                             .Attr<int64_t>("n0")
                             .Attr<int64_t>("m")
                             .Attr<int64_t>("use_slack")
                             .Attr<int64_t>("adapt_rho_every")
                             .Attr<double>("adaptive_rho_tolerance")
                             .Attr<double>("rho_min")
                             .Attr<double>("rho_max")
                             // x_out, iters_out, x_blocks, z_g, y_g, y_f_0, y_f_dyn, xi_g, rho_bar,
                             // kernel_ns, S_work, Phiinv_work
                             .Ret<Buf<DT>>().Ret<BufU32>().Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>()
                             .Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>()
                             .Ret<Buf<DT>>().Ret<Buf<DT>>()
                             .To(AdmmB200Impl<DT, R>)
                             .release();
  return handler->Call(frame);
}

// admm_cudss_cuda contract: S, D, E, q, A0, A_minus, A_plus, G, l, u, c0, c_dyn,
// x0, z_g0, y_g0, y_f_0, y_f_dyn, xi_g0, rho_bar, slack_weight; attributes
// max_iter, check_every, adapt_rho_every, eps_abs, eps_rel, sigma,
// rho_f_factor, alpha, adaptive_rho_tolerance, rho_min, rho_max, nx, n0, m,
// use_slack; results x_out, iters_out, x_blocks, z_g, y_g, y_f_0, y_f_dyn,
// xi_g, rho_bar, kernel_ns.
template <ffi::DataType DT, typename R>
ffi::Error AdmmB200DirectImpl(cudaStream_t stream, ffi::ScratchAllocator scratch, Buf<DT> S, Buf<DT> D, Buf<DT> E,
                              Buf<DT> q, Buf<DT> A0, Buf<DT> A_minus, Buf<DT> A_plus, Buf<DT> G, Buf<DT> l,
                              Buf<DT> u, Buf<DT> c0, Buf<DT> c_dyn, Buf<DT> x0, Buf<DT> z_g0, Buf<DT> y_g0,
                              Buf<DT> y_f_0, Buf<DT> y_f_dyn, Buf<DT> xi_g0, Buf<DT> rho_bar, Buf<DT> slack_weight,
                              int64_t max_iter, int64_t check_every, int64_t adapt_rho_every, double eps_abs,
                              double eps_rel, double sigma, double rho_f_factor, double alpha,
                              double adaptive_rho_tolerance, double rho_min, double rho_max, int64_t nx, int64_t n0,
                              int64_t m, int64_t use_slack, ffi::Result<Buf<DT>> x_out,
                              ffi::Result<BufU32> iters_out, ffi::Result<Buf<DT>> x_blocks_out,
                              ffi::Result<Buf<DT>> z_g_out, ffi::Result<Buf<DT>> y_g_out,
                              ffi::Result<Buf<DT>> y_f_0_out, ffi::Result<Buf<DT>> y_f_dyn_out,
                              ffi::Result<Buf<DT>> xi_g_out, ffi::Result<Buf<DT>> rho_bar_out,
                              ffi::Result<Buf<DT>> kernel_ns_out) {
  const auto sd = S.dimensions();
  TmpcDims d{};
  if (sd.size() == 4) {
    d.Nb = static_cast<int32_t>(sd[0]);
    d.T = static_cast<int32_t>(sd[1]);
    d.n = static_cast<int32_t>(sd[2]);
  } else if (sd.size() == 3) {
    d.Nb = 1;
    d.T = static_cast<int32_t>(sd[0]);
    d.n = static_cast<int32_t>(sd[1]);
  } else {
    return ffi::Error::InvalidArgument("S must be [T, n, 3n] or [Nb, T, n, 3n]");
  }
  d.nx = static_cast<int32_t>(nx);
  d.n0 = static_cast<int32_t>(n0);
  d.m = static_cast<int32_t>(m);
  const int64_t N = d.T - 1;
  auto ok = [&](const auto& b, int64_t per) { return static_cast<int64_t>(b.element_count()) == per * d.Nb; };
  if (!ok(D, (int64_t)d.T * d.n * d.n) || !ok(E, N * d.n * d.n) || !ok(q, (int64_t)d.T * d.n) ||
      !ok(A0, (int64_t)d.n0 * d.n) || !ok(A_minus, N * d.nx * d.n) || !ok(A_plus, N * d.nx * d.n) ||
      !ok(G, (int64_t)d.T * d.m * d.n) || !ok(l, (int64_t)d.T * d.m) || !ok(u, (int64_t)d.T * d.m) ||
      !ok(c0, d.n0) || !ok(c_dyn, N * d.nx) || !ok(x0, (int64_t)d.T * d.n) || !ok(rho_bar, 1))
    return ffi::Error::InvalidArgument("an operand has the wrong size");
  TmpcQP qp{D.typed_data(), E.typed_data(), q.typed_data(), A0.typed_data(), A_minus.typed_data(),
            A_plus.typed_data(), c0.typed_data(), c_dyn.typed_data(), d.m ? G.typed_data() : nullptr,
            d.m ? l.typed_data() : nullptr, d.m ? u.typed_data() : nullptr};
  TmpcAdmmState in{x0.typed_data(), y_g0.typed_data(), y_f_0.typed_data(), y_f_dyn.typed_data(),
                   z_g0.typed_data(), xi_g0.typed_data(), rho_bar.typed_data()};
  TmpcAdmmState out{x_blocks_out->typed_data(), y_g_out->typed_data(), y_f_0_out->typed_data(),
                    y_f_dyn_out->typed_data(), z_g_out->typed_data(), xi_g_out->typed_data(),
                    rho_bar_out->typed_data()};
  TmpcAdmmConfig cfg{};
  cfg.max_iter = static_cast<int32_t>(max_iter);
  cfg.pcg_max_iter = 1;
  cfg.check_every = static_cast<int32_t>(check_every);
  cfg.adapt_rho_every = static_cast<int32_t>(adapt_rho_every);
  cfg.eps_abs = eps_abs;
  cfg.eps_rel = eps_rel;
  cfg.sigma = sigma;
  cfg.rho_f_factor = rho_f_factor;
  cfg.alpha = alpha;
  cfg.pcg_eps = 0.0;
  cfg.adaptive_rho_tolerance = adaptive_rho_tolerance;
  cfg.rho_min = rho_min;
  cfg.rho_max = rho_max;
  cfg.use_slack = static_cast<int32_t>(use_slack != 0);
  cfg.linsys = TMPC_LINSYS_DIRECT;
  // workspace (256-byte aligned) followed by the per-problem status words
  const size_t need = tmpc_admm_workspace_bytes(&d, static_cast<int32_t>(sizeof(R)), &cfg);
  const size_t ws_bytes = (need + 255) & ~size_t(255);
  auto mem = scratch.Allocate(ws_bytes + sizeof(int32_t) * static_cast<size_t>(d.Nb), 256);
  if (!mem.has_value()) return ffi::Error::Internal("b200 direct ADMM: scratch allocation failed");
  void* ws = *mem;
  int32_t* status = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(ws) + ws_bytes);
  int32_t rc = Api<R>::solve(&d, &qp, &in, &out, use_slack ? slack_weight.typed_data() : nullptr, &cfg,
                             x_out->typed_data(), iters_out->typed_data(), status, need ? ws : nullptr, need, stream);
  if (rc < 0) return ffi::Error::InvalidArgument(std::string("b200 direct ADMM: ") + tmpc_error_string(rc));
  if (rc > 0) return ffi::Error::Internal(std::string("b200 direct ADMM: ") + tmpc_error_string(rc));
  cudaError_t ce = cudaMemsetAsync(kernel_ns_out->untyped_data(), 0, kernel_ns_out->element_count() * sizeof(R),
                                   stream);
  if (ce != cudaSuccess) return ffi::Error::Internal(std::string("CUDA error: ") + cudaGetErrorString(ce));
  return ffi::Error::Success();
}

template <ffi::DataType DT, typename R>
XLA_FFI_Error* CallDirect(XLA_FFI_CallFrame* frame) {
  static auto* handler = ffi::Ffi::Bind()
                             .Ctx<ffi::PlatformStream<cudaStream_t>>()
                             .Ctx<ffi::ScratchAllocator>()
                             // S, D, E, q, A0, A_minus, A_plus, G, l, u, c0, c_dyn
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Arg<Buf<DT>>().Arg<Buf<DT>>()
                             // x0, z_g0, y_g0, y_f_0, y_f_dyn, xi_g0, rho_bar, slack_weight
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Arg<Buf<DT>>().Arg<Buf<DT>>().Arg<Buf<DT>>()
                             .Attr<int64_t>("max_iter")
                             .Attr<int64_t>("check_every")
                             .Attr<int64_t>("adapt_rho_every")
                             .Attr<double>("eps_abs")
                             .Attr<double>("eps_rel")
                             .Attr<double>("sigma")
                             .Attr<double>("rho_f_factor")
                             .Attr<double>("alpha")
                             .Attr<double>("adaptive_rho_tolerance")
                             .Attr<double>("rho_min")
                             .Attr<double>("rho_max")
                             .Attr<int64_t>("nx")
                             .Attr<int64_t>("n0")
                             .Attr<int64_t>("m")
                             .Attr<int64_t>("use_slack")
                             // x_out, iters_out, x_blocks, z_g, y_g, y_f_0, y_f_dyn, xi_g, rho_bar, kernel_ns
                             .Ret<Buf<DT>>().Ret<BufU32>().Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>()
                             .Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>().Ret<Buf<DT>>()
                             .To(AdmmB200DirectImpl<DT, R>)
                             .release();
  return handler->Call(frame);
}

}  // namespace

extern "C" XLA_FFI_Error* AdmmB200Cuda(XLA_FFI_CallFrame* frame) {
  return Call<ffi::DataType::F32, float>(frame);
}
extern "C" XLA_FFI_Error* AdmmB200CudaF64(XLA_FFI_CallFrame* frame) {
  return Call<ffi::DataType::F64, double>(frame);
}
extern "C" XLA_FFI_Error* AdmmB200DirectCuda(XLA_FFI_CallFrame* frame) {
  return CallDirect<ffi::DataType::F32, float>(frame);
}
extern "C" XLA_FFI_Error* AdmmB200DirectCudaF64(XLA_FFI_CallFrame* frame) {
  return CallDirect<ffi::DataType::F64, double>(frame);
}

#endif  // TMPC_HAVE_XLA_FFI
