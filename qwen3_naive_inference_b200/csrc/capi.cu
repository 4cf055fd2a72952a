// Library-wide entry points of the C ABI: version and status strings.
#include "common.cuh"

extern "C" int qb_abi_version(void) { return 2; }

extern "C" const char* qb_status_string(int status) {
  if (status == QB_OK) return "ok";
  if (status == QB_ERR_INVALID) return "invalid argument";
  if (status == QB_ERR_UNSUPPORTED) return "unsupported shape or configuration";
  if (status >= QB_ERR_CUDA_BASE) return cudaGetErrorString((cudaError_t)(status - QB_ERR_CUDA_BASE));
  return "unknown status";
}
