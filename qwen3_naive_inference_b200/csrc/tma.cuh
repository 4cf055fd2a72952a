// mbarrier and TMA helpers of the tcgen05 GEMM kernels.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace {

// A wait that has not completed after this many SM clock cycles (~2 s at 1.9 GHz) is
// declared hung.  The bound is on elapsed clock64() time, not on a poll count, because a
// single try_wait may itself suspend for an implementation-defined interval.
constexpr long long WAIT_CYCLES = 4000000000ll;

// ---------------------------------------------------------------- PTX helpers
QB_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
QB_DEVICE void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
QB_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
QB_DEVICE bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false when it gave up (or another role already aborted).
QB_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 255) {
      if (*abort_flag) return false;
      if (clock64() - t0 > WAIT_CYCLES) break;
    }
  }
  *abort_flag = 1;
  qb_set_err(err, QB_DEVERR_TIMEOUT);
  return false;
}
// Bounded wait used on the way out: no abort check, same time limit.
QB_DEVICE void mbar_drain(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > WAIT_CYCLES) return;
}

QB_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

}  // namespace
