// Shared device helpers for the sm_100a kernels of the GRPO step.
//
// Every kernel in this library is launched through an extern "C" entry point
// declared in include/qwen3b200.h.  Entry points take raw device pointers,
// explicit sizes and a cudaStream_t, never allocate, and return a status code
// (QB_OK == 0).  Data-dependent indices (page ids, slots, token ids) are
// bounds-checked on the device: a bad index skips the access and ORs a bit
// into the caller's `err` word instead of faulting.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/qwen3b200.h"

typedef __nv_bfloat16 bf16;

#define QB_DEVICE __device__ __forceinline__

// ---------------------------------------------------------------- launch glue
static inline int qb_launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? QB_OK : (QB_ERR_CUDA_BASE + (int)e);
}

// ---------------------------------------------------------------- programmatic dependent launch
// The tcgen05 kernels (GEMMs, training attention), whose prologue is long (barrier init, TMEM
// allocation, tensor-map prefetch), are launched with programmatic stream serialization when the
// library-wide switch is on: such a kernel may be scheduled as soon as every CTA of the kernel
// before it in the stream has passed qb_pdl_trigger(), so its launch and prologue overlap that
// kernel's run; qb_pdl_wait() then blocks until the kernel before has completed and its writes
// are visible.  Short kernels are launched with plain stream order (measured: the early launch
// costs them more than it hides) but still trigger at their start, so a GEMM after them starts
// early.  Both calls are no-ops in a kernel launched without the attribute.  Rules every kernel
// of the library follows:
//   * every thread calls qb_pdl_wait() before its first global access that depends on earlier
//     work (any read of an input another kernel may have written, and every global write), and
//     before it exits -- a kernel that could complete without waiting would let the kernel after
//     it pass its own wait while the kernel before is still running;
//   * a kernel that allocates TMEM calls qb_pdl_trigger() only after its allocation succeeded,
//     so the next kernel never holds TMEM this one still needs.
QB_DEVICE void qb_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
QB_DEVICE void qb_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Library-wide switch (qb_set_pdl in the C ABI); on by default.
bool qb_pdl_enabled();

// Launch `kern` on `st` with a cluster of `cluster_x` CTAs (1: none) and, when `early` and the
// switch is on, programmatic stream serialization.  Returns the launch status like
// qb_launch_status().
template <typename... KArgs, typename... Args>
static inline int qb_launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               int cluster_x, bool early, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (cluster_x > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = (unsigned)cluster_x;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  if (early && qb_pdl_enabled()) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  (void)cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  return qb_launch_status();  // the launch's own error (consumed here: callers return this value)
}
// Plain stream order (short kernels).
template <typename... KArgs, typename... Args>
static inline int qb_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                            int cluster_x, Args&&... args) {
  return qb_launch_ex(kern, grid, block, smem, st, cluster_x, false, static_cast<Args&&>(args)...);
}

#define QB_CHECK_ARG(cond)            \
  do {                                \
    if (!(cond)) return QB_ERR_INVALID; \
  } while (0)

// Device-side error flag bits (ORed into *err by kernels).
#define QB_DEVERR_PAGE 1      // block_table entry outside [0, num_blocks)
#define QB_DEVERR_SLOT 2      // slot_mapping entry outside the cache
#define QB_DEVERR_TOKEN 4     // token id outside [0, vocab)
#define QB_DEVERR_SHAPE 8     // per-row length inconsistent with the buffers
#define QB_DEVERR_TIMEOUT 16  // a bounded wait gave up

QB_DEVICE void qb_set_err(int* err, int bit) {
  if (err) atomicOr(err, bit);
}

// ---------------------------------------------------------------- numerics
QB_DEVICE float bf2f(bf16 x) { return __bfloat162float(x); }
QB_DEVICE bf16 f2bf(float x) { return __float2bfloat16_rn(x); }
QB_DEVICE float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

QB_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
QB_DEVICE float2 unpack_bf16x2(uint32_t u) {
  __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&u);
  return __bfloat1622float2(v);
}

// SiLU as the SwiGLU kernel and the GEMM's SwiGLU epilogue compute it (one definition, so the fused
// and unfused paths give the same bits): fp32 with the fast exponential and divide intrinsics (a
// few ulp of fp32, far below the bf16 rounding that follows; 1 + e^-g overflowing to inf gives 0).
QB_DEVICE float qb_silu(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// Requests the 128-byte line holding p into L1 (no register written).
QB_DEVICE void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

// QK-norm + RoPE arithmetic shared by the standalone kernel and the qkv GEMM's epilogue, with the
// fused multiply-adds written out so both give the same bits (a 128-wide head; RoPE pairs (j, j+64)).
// Sum of squares of eight consecutive elements of a head, in order.
QB_DEVICE float qk_sumsq8(const float (&v)[8]) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = fmaf(v[i], v[i], s);
  return s;
}
// The head's sum of squares from its sixteen 8-element partial sums p[g] (elements 8g..8g+7),
// combined in the order of a half-warp butterfly over offsets 8, 4, 2, 1.
QB_DEVICE float qk_sumsq_tree(const float (&p)[16]) {
  float t[8], u[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) t[i] = p[i] + p[i + 8];
#pragma unroll
  for (int i = 0; i < 4; ++i) u[i] = t[i] + t[i + 4];
  return (u[0] + u[2]) + (u[1] + u[3]);
}
QB_DEVICE float qk_rstd(float ss, float eps) { return rsqrtf(ss / 128.0f + eps); }
QB_DEVICE float qk_rope_lo(float x1, float x2, float c, float s) { return fmaf(x1, c, -(x2 * s)); }  // x1*c - x2*s
QB_DEVICE float qk_rope_hi(float x2, float x1, float c, float s) { return fmaf(x2, c, x1 * s); }     // x2*c + x1*s

QB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
QB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum for blockDim.x a multiple of 32 (<= 1024). `red` holds >= 32 floats.
QB_DEVICE float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = (threadIdx.x < (unsigned)nw) ? red[threadIdx.x] : 0.f;
  if (wid == 0) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  float r = red[0];
  __syncthreads();
  return r;
}

// ---------------------------------------------------------------- PTX wrappers
QB_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte async global->shared copy; src_bytes == 0 zero-fills the destination.
QB_DEVICE void cp_async_16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
// 4-byte copy (zero-filled when src_bytes == 0); no 16-byte alignment needed.
QB_DEVICE void cp_async_4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
QB_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
QB_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

QB_DEVICE void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
QB_DEVICE void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D = A(16x16, row) * B(16x8, col) + D, bf16 inputs, fp32 accumulate.
QB_DEVICE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Tiles of 128 bf16 per row (256 B = 16 chunks of 16 B) are stored with the
// 16-byte chunk index XORed by (row & 7): the eight rows read by one
// ldmatrix phase then fall into eight distinct bank groups.
QB_DEVICE uint32_t swz128(int row, int chunk) {
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

// ---------------------------------------------------------------- thread-block clusters
QB_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory byte in CTA `rank` of the cluster.
QB_DEVICE uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}
QB_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
