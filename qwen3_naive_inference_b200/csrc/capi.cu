// Library-wide entry points of the C ABI: version and status strings, the launch switch.
#include <atomic>

#include "common.cuh"

namespace {
std::atomic<int> g_pdl{1};
}  // namespace

bool qb_pdl_enabled() { return g_pdl.load(std::memory_order_relaxed) != 0; }

extern "C" int qb_set_pdl(int on) {
  g_pdl.store(on ? 1 : 0, std::memory_order_relaxed);
  return QB_OK;
}

extern "C" int qb_get_pdl(void) { return g_pdl.load(std::memory_order_relaxed); }

extern "C" int qb_abi_version(void) { return 2; }

extern "C" const char* qb_status_string(int status) {
  if (status == QB_OK) return "ok";
  if (status == QB_ERR_INVALID) return "invalid argument";
  if (status == QB_ERR_UNSUPPORTED) return "unsupported shape or configuration";
  if (status >= QB_ERR_CUDA_BASE) return cudaGetErrorString((cudaError_t)(status - QB_ERR_CUDA_BASE));
  return "unknown status";
}
