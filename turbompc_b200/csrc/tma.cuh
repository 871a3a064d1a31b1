// 1-D TMA bulk copies (cp.async.bulk, global -> shared) completed on an
// mbarrier, with a bounded wait: a wait that runs out of polls returns false
// instead of spinning forever, so a lost transfer cannot hang the GPU.
// No multicast form is used anywhere.
#pragma once

#include <stdint.h>

#include <atomic>

namespace tmpc {

// Polls a kernel spends waiting for its operators' bulk copies before it
// reports a transfer time-out (far longer than any copy takes), and the polls
// it then spends draining the copies still in flight before it returns.
constexpr uint32_t kTransferPolls = 1u << 26;
constexpr uint32_t kTransferDrainPolls = 1u << 26;

// Host-side poll limit passed to the kernels; tmpc_set_transfer_poll_limit
// changes it (a diagnostics hook: a limit of 0 makes every wait report a
// time-out after its copies have landed, which exercises the status path).
inline std::atomic<uint32_t>& transfer_poll_limit() {
  static std::atomic<uint32_t> v{kTransferPolls};
  return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Wait for phase `parity` of the barrier; gives up after max_polls polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t max_polls) {
  for (uint32_t i = 0; i < max_polls; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

}  // namespace tmpc
