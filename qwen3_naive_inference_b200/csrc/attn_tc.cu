// Causal GQA attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
// Replaces the dense varlen branch of flash_attn_varlen_func used by the training / recompute
// forward (qwen3_naive.py:540-548 and the manual attention of Qwen3Attention.forward,
// :553-593) for packed sequences, Lq == Lk.
//
// One CTA owns 64 query positions of one sequence and one kv head.  Both query heads of the kv
// group are stacked into the 128 rows of one MMA tile (rows 0-63: head 2*kvh, rows 64-127: head
// 2*kvh+1), so each K/V tile is read from memory once for both heads.  Keys come in tiles of 64;
// two CTAs share an SM (96 KB of shared memory and 256 TMEM columns each), so one CTA's start-up
// and epilogue overlap the other's main loop.
//   warp 0     TMA producers: lane 0 loads Q once (4 boxes) and runs the K ring (K-major, released
//              as soon as S_j has read it), lane 1 the V ring (MN-major, two 64-wide d atoms,
//              released after P_j V_j); two stages each;
//   warp 1     allocates 256 TMEM columns; one thread issues tcgen05.mma:
//                S_b = Q K_j^T       (A, B from shared memory; fp32 S in TMEM columns [64 b, +64))
//                O  += P_{j-1} V_{j-1} (A = P from TMEM, aliasing S_{b'}; B = V, MN-major)
//              software-pipelined so that S_j is computed while the softmax works on S_{j-1};
//   warps 2-5  softmax, one thread per row (TMEM lane): causal mask, running max in the log2
//              domain, P = exp2(S - max) written back into TMEM as bf16 pairs, running row sum;
//              the O accumulator (TMEM columns [128, 256)) is rescaled in place only when a row's
//              max grows by more than 2^8 (otherwise the stale max keeps every P below 256); at
//              the end O / l is stored as bf16 and the log-sum-exp for the backward.
// Every mbarrier wait is bounded (~2 s): on timeout the kernel raises QB_DEVERR_TIMEOUT, all roles
// leave their loops, the producer drains its copies, the MMA issuer waits for its MMAs, TMEM is
// freed.  Every TMA load reads this GPU's memory; no cluster multicast.
#include "tcgen05.cuh"

namespace {

constexpr int AT_THREADS = 192;                      // producer warp, MMA warp, softmax warpgroup
constexpr int AT_QPOS = 64;                           // query positions per CTA (x 2 heads = 128 rows)
constexpr int AT_KEYS = 64;                           // keys per tile
constexpr int AT_Q_HALF = 128 * 64 * 2;               // Q sub-tile [128 rows x 64 d]: 16 KB
constexpr int AT_Q_BYTES = 2 * AT_Q_HALF;             // Q: d halves 0-63, 64-127
constexpr int AT_K_HALF = AT_KEYS * 64 * 2;           // K sub-tile [64 keys x 64 d]: 8 KB
constexpr int AT_KV_BYTES = 2 * AT_K_HALF;            // K or V tile: 16 KB
constexpr int AT_STAGE_BYTES = 2 * AT_KV_BYTES;       // K then V
constexpr int AT_STAGES = 2;
constexpr int AT_SMEM = AT_Q_BYTES + AT_STAGES * AT_STAGE_BYTES + 1024 /*align*/ + 160 /*barriers*/;
constexpr int AT_TMEM_COLS = 256;                     // S buffers [0,64), [64,128); O [128,256)
constexpr uint32_t AT_O_COL = 128;
constexpr float AT_RESCALE = 8.f;                     // rescale O only when a max grows by > 2^8

// kind::f16, D fp32, A/B bf16, M = 128; S: N = 64, both K-major; PV: N = 128, B (V) MN-major.
constexpr uint32_t IDESC_S = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t IDESC_PV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((128u >> 3) << 17) |
                              ((128u >> 4) << 24);

struct AttnTcParams {
  const int32_t* cu;     // [batch + 1] packed sequence starts (queries and keys alike)
  const int32_t* tiles;  // [n_tiles, 2]: (sequence, first query position of a 64-position tile)
  int tiles_per_seq;
  int hq, hkv;
  float scale_log2;      // softmax scale * log2(e)
  bf16* out;
  int64_t o_stride;
  float* lse;            // nullable [hq, total_q], natural log
  int64_t total_q;
  int* err;
};

__global__ void __launch_bounds__(AT_THREADS, 2)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, AttnTcParams p) {
  qb_pdl_wait();  // metadata and operands may come from the kernel before; also before any exit
  extern __shared__ uint8_t smem_raw[];
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int b = p.tiles ? p.tiles[2 * tile] : tile / p.tiles_per_seq;
  const int q_start = p.tiles ? p.tiles[2 * tile + 1] : (tile % p.tiles_per_seq) * AT_QPOS;
  const int s0 = p.cu[b], L = p.cu[b + 1] - s0;
  if (q_start >= L) return;  // uniform across the CTA, before any barrier or TMEM exists
  const int n_kv = min(L, q_start + AT_QPOS);
  const int n_tiles = (n_kv + AT_KEYS - 1) / AT_KEYS;
  const int h0 = 2 * kvh;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;  // SW128 atoms need 1024-byte alignment
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base;
  auto sK = [&](int s) { return base + AT_Q_BYTES + s * AT_STAGE_BYTES; };
  auto sV = [&](int s) { return base + AT_Q_BYTES + s * AT_STAGE_BYTES + AT_KV_BYTES; };
  const uint32_t bar0 = base + AT_Q_BYTES + AT_STAGES * AT_STAGE_BYTES;
  // q_full, k_full[2], k_empty[2], s_full[2], s_free[2], p_ready[2], o_done, o_last, done, v_full[2], v_empty[2]
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8 * (3 + s); };
  auto s_full = [&](int x) { return bar0 + 8 * (5 + x); };
  auto s_free = [&](int x) { return bar0 + 8 * (7 + x); };
  auto p_ready = [&](int x) { return bar0 + 8 * (9 + x); };
  auto v_full = [&](int s) { return bar0 + 8 * (14 + s); };
  auto v_empty = [&](int s) { return bar0 + 8 * (16 + s); };
  const uint32_t o_done = bar0 + 8 * 11, o_last = bar0 + 8 * 12, done_bar = bar0 + 8 * 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + AT_Q_BYTES + AT_STAGES * AT_STAGE_BYTES + 8 * 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
      mbar_init(s_full(s), 1);
      mbar_init(s_free(s), 1);
      mbar_init(p_ready(s), 128);
    }
    mbar_init(o_done, 1);
    mbar_init(o_last, 1);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tq)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tk)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tv)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(AT_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  qb_pdl_trigger();  // after the TMEM allocation: the next kernel cannot take it from this CTA

  if (warp == 0 && lane < 2) {
    // ------------------------------------------------------------ TMA producers
    // lane 0: Q, then the K ring (a K tile is released as soon as S_j has read it);
    // lane 1: the V ring (released after P_j V_j)
    if (lane == 0) {
      mbar_expect_tx(q_full, AT_Q_BYTES);
      for (int d = 0; d < 2; ++d)
        for (int hh = 0; hh < 2; ++hh)
          tma_load_2d(sQ + d * AT_Q_HALF + hh * (AT_Q_HALF / 2), &tq, (h0 + hh) * 128 + d * 64, s0 + q_start,
                      q_full);
    }
    uint32_t issued = 0, last_parity = 0;  // per stage: a load is in flight; its phase parity
    for (int j = 0; j < n_tiles && !*abort_flag; ++j) {
      const int st = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      const uint32_t empty = lane == 0 ? k_empty(st) : v_empty(st), full = lane == 0 ? k_full(st) : v_full(st);
      if (!mbar_wait(empty, ph ^ 1, abort_flag, p.err)) break;
      mbar_expect_tx(full, AT_KV_BYTES);
      const int key0 = s0 + j * AT_KEYS;
      for (int d = 0; d < 2; ++d) {
        if (lane == 0)
          tma_load_2d(sK(st) + d * AT_K_HALF, &tk, kvh * 128 + d * 64, key0, full);  // K-major halves
        else
          tma_load_2d(sV(st) + d * AT_K_HALF, &tv, kvh * 128 + d * 64, key0, full);  // MN atom d
      }
      issued |= 1u << st;
      last_parity = (last_parity & ~(1u << st)) | (ph << st);
    }
    // never leave with a copy in flight into this CTA's shared memory
    if (lane == 0) mbar_drain(q_full, 0);
    for (int st = 0; st < 2; ++st)
      if (issued & (1u << st)) mbar_drain(lane == 0 ? k_full(st) : v_full(st), (last_parity >> st) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    bool ok = mbar_wait(q_full, 0, abort_flag, p.err);
    for (int j = 0; ok && j <= n_tiles; ++j) {
      if (j < n_tiles) {
        const int st = j & 1, x = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(k_full(st), ph, abort_flag, p.err) || !mbar_wait(s_free(x), ph ^ 1, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)  // d = 128 in K-steps of 16: sub-tile k/4, 32 B each inside it
          umma_bf16(tmem + x * AT_KEYS, sw128_kmajor_desc(sQ + (k >> 2) * AT_Q_HALF + (k & 3) * 32),
                    sw128_kmajor_desc(sK(st) + (k >> 2) * AT_K_HALF + (k & 3) * 32), IDESC_S, k > 0);
        umma_commit(s_full(x));
        umma_commit(k_empty(st));  // the K tile is free once S_j has read it
      }
      if (j > 0) {
        const int i = j - 1, st = i & 1, x = i & 1;
        if (!mbar_wait(p_ready(x), (uint32_t)(i >> 1) & 1u, abort_flag, p.err) ||
            !mbar_wait(v_full(st), (uint32_t)(i >> 1) & 1u, abort_flag, p.err)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 64 keys in K-steps of 16: P columns x*64 + 8k; V rows 16k
          umma_bf16_ts(tmem + AT_O_COL, tmem + x * AT_KEYS + 8 * k, sw128_mnmajor_desc(sV(st) + k * 16 * 128),
                       IDESC_PV, (i > 0 || k > 0) ? 1u : 0u);
        umma_commit(i + 1 == n_tiles ? o_last : o_done);
        umma_commit(v_empty(st));
        umma_commit(s_free(x));
      }
    }
    // no MMA may still be reading shared memory or writing TMEM when the CTA leaves
    umma_commit(done_bar);
    mbar_drain(done_bar, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;       // TMEM lane = tile row
    const int hh = r >> 6, pos = q_start + (r & 63);
    const bool live = pos < L;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const int lim = live ? pos : -1;  // inclusive causal limit (dense: query i sees keys <= i)
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int x = j & 1;
      // tcgen05.ld/st below are warp-collective: every decision that leads to them is warp-uniform
      if (__any_sync(0xffffffffu, !mbar_wait(s_full(x), (uint32_t)(j >> 1) & 1u, abort_flag, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t v[64];
      tmem_ld32_nowait(t_lane + x * AT_KEYS, v);
      tmem_ld32_nowait(t_lane + x * AT_KEYS + 32, v + 32);
      tmem_ld_wait();
      const int k0 = j * AT_KEYS;
      const bool full = k0 + AT_KEYS - 1 <= lim;  // every key of the tile visible: no per-key mask
      if (!full) {  // the diagonal tile: keys past the row's limit drop out of the max and the sum
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (k0 + i > lim) v[i] = __float_as_uint(-INFINITY);
      }
      // row max over eight independent chains (a single chain would serialise 64 dependent maxes)
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = __uint_as_float(v[c]);
#pragma unroll
      for (int i = 8; i < 64; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(v[i]));
      float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      mt *= p.scale_log2;
      const bool need = mt > m_ref + AT_RESCALE || (m_ref == -INFINITY && mt > -INFINITY);
      float alpha = 1.f;
      if (need) {
        alpha = m_ref == -INFINITY ? 0.f : exp2f(m_ref - mt);
        m_ref = mt;
        l *= alpha;
      }
      // O holds P_0..P_{j-1} V: when any row of the warp moved its max, the warp waits for the last
      // of those products and rescales its 32 rows in TMEM together (the others by 1)
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        if (__any_sync(0xffffffffu, !mbar_wait(o_done, (uint32_t)(j - 1) & 1u, abort_flag, p.err))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          uint32_t o[32];
          tmem_ld32(t_lane + AT_O_COL + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_lane + AT_O_COL + c, o);
        }
      }
      // P = exp2(S - max) as bf16 pairs over the first 32 columns of this S buffer
      const float mref = m_ref == -INFINITY ? 0.f : m_ref;
      // masked keys hold -inf: exp2 gives 0 (a fully masked row has mref 0 and stays at 0)
      float rsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float a = fast_exp2(fmaf(__uint_as_float(v[2 * i]), p.scale_log2, -mref));
        const float bb = fast_exp2(fmaf(__uint_as_float(v[2 * i + 1]), p.scale_log2, -mref));
        rsum[i & 7] += a + bb;
        pk[i] = pack_bf16x2(a, bb);
      }
      const float rs = ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
      tmem_st32(t_lane + x * AT_KEYS, pk);
      l += rs;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_ready(x));
    }
    // epilogue: O / l -> bf16, and the row's log-sum-exp
    if (ok && __all_sync(0xffffffffu, mbar_wait(o_last, 0, abort_flag, p.err))) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = p.out + (int64_t)(s0 + pos) * p.o_stride + (h0 + hh) * 128;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t o[32];
        tmem_ld32(t_lane + AT_O_COL + c, o);
        if (live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv);
            reinterpret_cast<uint4*>(orow + c)[q] = w;
          }
        }
      }
      if (live && p.lse)
        p.lse[(int64_t)(h0 + hh) * p.total_q + s0 + pos] = l > 0.f ? (m_ref + log2f(l)) * 0.6931471805599453f
                                                                   : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AT_TMEM_COLS));
  }
}

// 2-D bf16 tensor map over rows of `ld` elements: inner extent `inner`, box {64, box_rows}, 128-byte
// swizzle, zero fill out of bounds.
bool at_tmap(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Dense causal attention forward on tcgen05 for packed sequences (Lq == Lk); called by
// qb_attn_varlen_fwd when block_tables is NULL, D == 128 and hq == 2 * hkv.
int attn_fwd_tc_launch(const void* q, int64_t q_stride, const void* k, const void* v, int64_t kv_stride,
                   const int32_t* cu_seqlens, int batch, const int32_t* tile_info, int n_tiles, int tiles_per_seq,
                   int hq, int hkv, float scale, void* out, int64_t o_stride, float* lse, int64_t total_q, int* err,
                   cudaStream_t st) {
  const auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (!al16(q) || !al16(k) || !al16(v) || q_stride % 8 || kv_stride % 8 || o_stride % 8 || !al16(out))
    return QB_ERR_INVALID;
  if (total_q <= 0 || n_tiles <= 0) return QB_OK;
  CUtensorMap tq, tk, tv;
  if (!at_tmap(&tq, q, (uint64_t)hq * 128, (uint64_t)total_q, (uint64_t)q_stride, 64) ||
      !at_tmap(&tk, k, (uint64_t)hkv * 128, (uint64_t)total_q, (uint64_t)kv_stride, AT_KEYS) ||
      !at_tmap(&tv, v, (uint64_t)hkv * 128, (uint64_t)total_q, (uint64_t)kv_stride, AT_KEYS))
    return QB_ERR_INVALID;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM) != cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  AttnTcParams p{cu_seqlens, tile_info, tiles_per_seq, hq, hkv, scale * 1.4426950408889634f,
                 (bf16*)out, o_stride, lse, total_q, err};
  (void)batch;
  return qb_launch_ex(attn_fwd_tc_kernel, dim3(dim3((unsigned)n_tiles, (unsigned)hkv)), dim3(AT_THREADS), AT_SMEM, st, 1, true, tq, tk, tv, p);
}

namespace {

// ================================================================ backward: dK, dV on tcgen05
// Gradient of the dense causal attention above w.r.t. K and V (the autograd of the reference's
// attention, qwen3_naive.py:553-593): for a 128-key tile of one kv head the CTA walks the query
// tiles at or after it, both query heads of the group stacked into 128 rows as in the forward:
//   S^T  = K Q_i^T ,  dP^T = V dO_i^T                      (M = 128 keys, N = 128 rows, K = d)
//   P^T  = exp2(S^T scale log2e - lse2[row]) (causal),  dS^T = P^T (dP^T - delta[row])
//   dV  += P^T dO_i ,  dK += dS^T Q_i                     (A = P^T / dS^T from TMEM, N = d)
// TMEM holds dV [0,128), dK [128,256), S^T [256,384) and dP^T [384,512); P^T and dS^T are written
// back as bf16 pairs over the first 64 columns of S^T and dP^T.  The K and V tiles stay in shared
// memory; Q_i and dO_i stream through a two-stage TMA ring; the rows' lse and delta are staged in
// shared memory by the softmax warps (loaded one item ahead).  dK is scaled by the softmax scale on
// the way out.  Bounded waits and teardown as in the forward; the four warps that share the
// staging barrier leave their loop together (a barrier reduction of their wait results).
constexpr int BT_THREADS = 192;
constexpr int BT_KEYS = 128;
constexpr int BT_HALF = 128 * 64 * 2;          // [128 rows x 64 d] bf16 sub-tile: 16 KB
constexpr int BT_TILE = 2 * BT_HALF;           // [128 x 128] tile: 32 KB
constexpr int BT_STAGE = 2 * BT_TILE;          // Q_i then dO_i
constexpr int BT_SMEM = 2 * BT_TILE + 2 * BT_STAGE + 2 * 2 * 128 * 4 /*lse2, delta x 2*/ + 1024 + 256;
constexpr uint32_t BT_DV = 0, BT_DK = 128, BT_S = 256, BT_DP = 384;
constexpr uint32_t IDESC_BT_KK = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t IDESC_BT_TS = IDESC_BT_KK | (1u << 16);  // B MN-major

struct AttnBwdTcParams {
  const int32_t* cu;
  const int32_t* tiles;   // [n_tiles, 2] (sequence, first row of a 64-row tile)
  int hq, hkv;
  float scale, scale_log2;
  const float* lse;       // [hq, total] natural log
  const float* delta;     // [hq, total] rowsum(dO * O)
  int64_t total;
  bf16* dk;
  bf16* dv;
  int64_t stride;         // row pitch of dq / dk / dv
  int* err;
};

// true in every calling thread when any of the `n` threads of named barrier `id` passes true
QB_DEVICE bool bar_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred q, o;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred o, 1, 128, q;\n\tselp.u32 %0, 1, 0, o;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v)
      : "memory");
  return r != 0;
}

__global__ void __launch_bounds__(BT_THREADS, 1)
attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                        AttnBwdTcParams p) {
  qb_pdl_wait();  // metadata and operands may come from the kernel before; also before any exit
  extern __shared__ uint8_t smem_raw[];
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int b = p.tiles[2 * tile], k_start = p.tiles[2 * tile + 1];
  if (k_start % BT_KEYS != 0) return;  // this 64-row tile is the second half of a 128-key tile
  const int s0 = p.cu[b], L = p.cu[b + 1] - s0;
  if (k_start >= L) return;
  const int n_items = (L - k_start + AT_QPOS - 1) / AT_QPOS;  // query tiles of 64 positions from k_start
  const int h0 = 2 * kvh;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sK = base, sV = base + BT_TILE;
  auto sQ = [&](int s) { return base + 2 * BT_TILE + s * BT_STAGE; };
  auto sDO = [&](int s) { return base + 2 * BT_TILE + s * BT_STAGE + BT_TILE; };
  float* sRow = reinterpret_cast<float*>(gbase + 2 * BT_TILE + 2 * BT_STAGE);  // [buf][lse2 128 | delta 128]
  const uint32_t bar0 = base + 2 * BT_TILE + 2 * BT_STAGE + 2 * 2 * 128 * 4;
  // kv_full, qd_full[2], qd_empty[2], s_full, pd_ready, st_free, done
  const uint32_t kv_full = bar0;
  auto qd_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto qd_empty = [&](int s) { return bar0 + 8 * (3 + s); };
  const uint32_t s_full = bar0 + 8 * 5, pd_ready = bar0 + 8 * 6, st_free = bar0 + 8 * 7, done_bar = bar0 + 8 * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + 2 * BT_TILE + 2 * BT_STAGE + 2 * 2 * 128 * 4 + 8 * 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(qd_full(s), 1);
      mbar_init(qd_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(pd_ready, 128);
    mbar_init(st_free, 1);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  qb_pdl_trigger();  // after the TMEM allocation: the next kernel cannot take it from this CTA

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ TMA producer
    mbar_expect_tx(kv_full, 2 * BT_TILE);
    for (int d = 0; d < 2; ++d) {
      tma_load_2d(sK + d * BT_HALF, &tk, kvh * 128 + d * 64, s0 + k_start, kv_full);
      tma_load_2d(sV + d * BT_HALF, &tv, kvh * 128 + d * 64, s0 + k_start, kv_full);
    }
    uint32_t issued = 0, last_parity = 0;
    for (int i = 0; i < n_items && !*abort_flag; ++i) {
      const int st = i & 1;
      const uint32_t ph = (uint32_t)(i >> 1) & 1u;
      if (!mbar_wait(qd_empty(st), ph ^ 1, abort_flag, p.err)) break;
      mbar_expect_tx(qd_full(st), BT_STAGE);
      const int row0 = s0 + k_start + i * AT_QPOS;
      for (int d = 0; d < 2; ++d)
        for (int hh = 0; hh < 2; ++hh) {
          tma_load_2d(sQ(st) + d * BT_HALF + hh * (BT_HALF / 2), &tq, (h0 + hh) * 128 + d * 64, row0, qd_full(st));
          tma_load_2d(sDO(st) + d * BT_HALF + hh * (BT_HALF / 2), &tdo, (h0 + hh) * 128 + d * 64, row0,
                      qd_full(st));
        }
      issued |= 1u << st;
      last_parity = (last_parity & ~(1u << st)) | (ph << st);
    }
    mbar_drain(kv_full, 0);
    for (int st = 0; st < 2; ++st)
      if (issued & (1u << st)) mbar_drain(qd_full(st), (last_parity >> st) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    auto issue_s_dp = [&](int i) {  // S^T = K Q_i^T, dP^T = V dO_i^T
      const int st = i & 1;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ko = (k >> 2) * BT_HALF + (k & 3) * 32;
        umma_bf16(tmem + BT_S, sw128_kmajor_desc(sK + ko), sw128_kmajor_desc(sQ(st) + ko), IDESC_BT_KK, k > 0);
        umma_bf16(tmem + BT_DP, sw128_kmajor_desc(sV + ko), sw128_kmajor_desc(sDO(st) + ko), IDESC_BT_KK, k > 0);
      }
      umma_commit(s_full);
    };
    bool ok = mbar_wait(kv_full, 0, abort_flag, p.err) && mbar_wait(qd_full(0), 0, abort_flag, p.err);
    if (ok) {
      tc_fence_after();
      issue_s_dp(0);
    }
    for (int i = 0; ok && i < n_items; ++i) {
      const int st = i & 1;
      if (!mbar_wait(pd_ready, (uint32_t)i & 1u, abort_flag, p.err)) break;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k) {  // 128 rows in K-steps of 16: P^T / dS^T columns 8k, Q / dO rows 16k
        umma_bf16_ts(tmem + BT_DV, tmem + BT_S + 8 * k, sw128_mn_desc(sDO(st) + k * 16 * 128, BT_HALF), IDESC_BT_TS,
                     (i > 0 || k > 0) ? 1u : 0u);
        umma_bf16_ts(tmem + BT_DK, tmem + BT_DP + 8 * k, sw128_mn_desc(sQ(st) + k * 16 * 128, BT_HALF), IDESC_BT_TS,
                     (i > 0 || k > 0) ? 1u : 0u);
      }
      umma_commit(qd_empty(st));
      umma_commit(st_free);
      if (i + 1 < n_items) {
        // S^T / dP^T are overwritten only after dV_i and dK_i have read P^T and dS^T
        if (!mbar_wait(st_free, (uint32_t)i & 1u, abort_flag, p.err) ||
            !mbar_wait(qd_full((i + 1) & 1), (uint32_t)((i + 1) >> 1) & 1u, abort_flag, p.err))
          break;
        tc_fence_after();
        issue_s_dp(i + 1);
      }
    }
    umma_commit(done_bar);
    mbar_drain(done_bar, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ P^T, dS^T and the epilogue
    const int quarter = warp & 3;
    const int kr = quarter * 32 + lane;  // TMEM lane = key row of the tile
    const int kpos = k_start + kr;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const int t = kr;                    // this thread also stages row t's lse2 / delta
    const int thh = t >> 6;
    auto fetch = [&](int i, float& l2, float& dl) {
      const int pos = k_start + i * AT_QPOS + (t & 63);
      if (pos < L) {
        const int64_t idx = (int64_t)(h0 + thh) * p.total + s0 + pos;
        l2 = p.lse[idx] * 1.4426950408889634f;
        dl = p.delta[idx];
      } else {
        l2 = INFINITY;
        dl = 0.f;
      }
    };
    float nl2, ndl;
    fetch(0, nl2, ndl);
    bool ok = true;
    for (int i = 0; i < n_items; ++i) {
      float* rowbuf = sRow + (i & 1) * 256;
      rowbuf[t] = nl2;
      rowbuf[128 + t] = ndl;
      asm volatile("bar.sync 1, 128;" ::: "memory");  // this item's rows are staged
      if (i + 1 < n_items) fetch(i + 1, nl2, ndl);    // in flight while this item is processed
      // every thread of the warpgroup leaves together if any wait gave up (they share the
      // named barriers above and below)
      const bool failed = !mbar_wait(s_full, (uint32_t)i & 1u, abort_flag, p.err) || *abort_flag;
      __syncwarp();  // bar.red is warp-aligned: reconverge after the spin
      if (bar_any(failed)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int q_start = k_start + i * AT_QPOS;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t sv[32], dv[32], pk[16], dk[16];
        tmem_ld32_nowait(t_lane + BT_S + c, sv);
        tmem_ld32_nowait(t_lane + BT_DP + c, dv);
        tmem_ld_wait();
        const float4* l4 = reinterpret_cast<const float4*>(rowbuf + c);
        const float4* d4 = reinterpret_cast<const float4*>(rowbuf + 128 + c);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 l = l4[q], dl = d4[q];
          const float lv[4] = {l.x, l.y, l.z, l.w}, dlv[4] = {dl.x, dl.y, dl.z, dl.w};
          float pv[4], dsv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int r = c + 4 * q + e;                 // tile row: head r >> 6, position q_start + (r & 63)
            const int qpos = q_start + (r & 63);
            const bool vis = kpos <= qpos && qpos < L;   // (kpos < L follows)
            const float pe = vis ? fast_exp2(fmaf(__uint_as_float(sv[4 * q + e]), p.scale_log2, -lv[e])) : 0.f;
            pv[e] = pe;
            dsv[e] = pe * (__uint_as_float(dv[4 * q + e]) - dlv[e]);
          }
          pk[2 * q] = pack_bf16x2(pv[0], pv[1]);
          pk[2 * q + 1] = pack_bf16x2(pv[2], pv[3]);
          dk[2 * q] = pack_bf16x2(dsv[0], dsv[1]);
          dk[2 * q + 1] = pack_bf16x2(dsv[2], dsv[3]);
        }
        tmem_st16(t_lane + BT_S + c / 2, pk);
        tmem_st16(t_lane + BT_DP + c / 2, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(pd_ready);
    }
    // epilogue: dK (x scale) and dV of this key row
    if (ok && __all_sync(0xffffffffu, mbar_wait(done_bar, 0, abort_flag, p.err))) {
      tc_fence_after();
      const bool live = kpos < L;
      bf16* dkrow = p.dk + (int64_t)(s0 + kpos) * p.stride + kvh * 128;
      bf16* dvrow = p.dv + (int64_t)(s0 + kpos) * p.stride + kvh * 128;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t a[32], v[32];
        tmem_ld32_nowait(t_lane + BT_DK + c, a);
        tmem_ld32_nowait(t_lane + BT_DV + c, v);
        tmem_ld_wait();
        if (live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 wk, wv;
            wk.x = pack_bf16x2(__uint_as_float(a[8 * q + 0]) * p.scale, __uint_as_float(a[8 * q + 1]) * p.scale);
            wk.y = pack_bf16x2(__uint_as_float(a[8 * q + 2]) * p.scale, __uint_as_float(a[8 * q + 3]) * p.scale);
            wk.z = pack_bf16x2(__uint_as_float(a[8 * q + 4]) * p.scale, __uint_as_float(a[8 * q + 5]) * p.scale);
            wk.w = pack_bf16x2(__uint_as_float(a[8 * q + 6]) * p.scale, __uint_as_float(a[8 * q + 7]) * p.scale);
            wv.x = pack_bf16x2(__uint_as_float(v[8 * q + 0]), __uint_as_float(v[8 * q + 1]));
            wv.y = pack_bf16x2(__uint_as_float(v[8 * q + 2]), __uint_as_float(v[8 * q + 3]));
            wv.z = pack_bf16x2(__uint_as_float(v[8 * q + 4]), __uint_as_float(v[8 * q + 5]));
            wv.w = pack_bf16x2(__uint_as_float(v[8 * q + 6]), __uint_as_float(v[8 * q + 7]));
            reinterpret_cast<uint4*>(dkrow + c)[q] = wk;
            reinterpret_cast<uint4*>(dvrow + c)[q] = wv;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

}  // namespace

// dK, dV of the dense causal attention on tcgen05 (packed sequences, Lq == Lk, hq == 2 hkv, d 128);
// called by qb_attn_varlen_bwd after its delta kernel.  q/k/v/dk/dv share `stride`, o/dout `o_stride`.
int attn_bwd_dkdv_tc_launch(const void* q, const void* k, const void* v, int64_t stride, const void* dout,
                            int64_t o_stride, const float* lse, const float* delta, const int32_t* cu_seqlens,
                            const int32_t* tile_info, int n_tiles, int hq, int hkv, float scale, int64_t total,
                            void* dk, void* dv, int* err, cudaStream_t st) {
  const auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (!al16(q) || !al16(k) || !al16(v) || !al16(dout) || !al16(dk) || !al16(dv) || stride % 8 || o_stride % 8)
    return QB_ERR_INVALID;
  if (total <= 0 || n_tiles <= 0) return QB_OK;
  CUtensorMap tq, tk, tv, tdo;
  if (!at_tmap(&tq, q, (uint64_t)hq * 128, (uint64_t)total, (uint64_t)stride, 64) ||
      !at_tmap(&tk, k, (uint64_t)hkv * 128, (uint64_t)total, (uint64_t)stride, BT_KEYS) ||
      !at_tmap(&tv, v, (uint64_t)hkv * 128, (uint64_t)total, (uint64_t)stride, BT_KEYS) ||
      !at_tmap(&tdo, dout, (uint64_t)hq * 128, (uint64_t)total, (uint64_t)o_stride, 64))
    return QB_ERR_INVALID;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BT_SMEM) !=
        cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  AttnBwdTcParams p{cu_seqlens, tile_info, hq, hkv, scale, scale * 1.4426950408889634f, lse, delta, total,
                    (bf16*)dk, (bf16*)dv, stride, err};
  return qb_launch_ex(attn_bwd_dkdv_tc_kernel, dim3(dim3((unsigned)n_tiles, (unsigned)hkv)), dim3(BT_THREADS), BT_SMEM, st, 1, true, tq, tk, tv, tdo, p);
}

namespace {

// ================================================================ backward: dQ on tcgen05
// For 64 query positions x both query heads of a kv group (128 rows, as in the forward) the CTA walks
// the 128-key tiles at or before them:
//   S = Q K_j^T ,  dP = dO V_j^T                 (M = 128 rows, N = 128 keys, K = d; A, B in smem)
//   dS = exp2(S scale log2e - lse2) (dP - delta) (causal; each thread holds one row's lse and delta)
//   dQ += dS K_j                                  (A = dS from TMEM, B = K_j read MN-major, N = d)
// TMEM: dQ [0,128), S [128,256), dP [256,384); dS is written as bf16 pairs over dP's first 64
// columns.  Q and dO stay in shared memory; K and V stream through two-stage rings (V released
// after dP_j, K after dQ_j).  dQ is scaled by the softmax scale on the way out.
constexpr int DQ_THREADS = 192;
constexpr int DQ_SMEM_TC = 2 * BT_TILE /*Q, dO*/ + 2 * BT_TILE /*K ring*/ + 2 * BT_TILE /*V ring*/ + 1024 + 256;
constexpr uint32_t DQ_ACC = 0, DQ_S = 128, DQ_DP = 256;

__global__ void __launch_bounds__(DQ_THREADS, 1)
attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                      AttnBwdTcParams p, bf16* dq) {
  qb_pdl_wait();  // metadata and operands may come from the kernel before; also before any exit
  extern __shared__ uint8_t smem_raw[];
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int b = p.tiles[2 * tile], q_start = p.tiles[2 * tile + 1];
  const int s0 = p.cu[b], L = p.cu[b + 1] - s0;
  if (q_start >= L) return;
  const int n_kv = min(L, q_start + AT_QPOS);
  const int n_tiles = (n_kv + BT_KEYS - 1) / BT_KEYS;
  const int h0 = 2 * kvh;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sQ = base, sDO = base + BT_TILE;
  auto sK = [&](int s) { return base + 2 * BT_TILE + s * BT_TILE; };
  auto sV = [&](int s) { return base + 4 * BT_TILE + s * BT_TILE; };
  const uint32_t bar0 = base + 6 * BT_TILE;
  // q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full, ds_ready, st_free, done
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8 * (3 + s); };
  auto v_full = [&](int s) { return bar0 + 8 * (5 + s); };
  auto v_empty = [&](int s) { return bar0 + 8 * (7 + s); };
  const uint32_t s_full = bar0 + 8 * 9, ds_ready = bar0 + 8 * 10, st_free = bar0 + 8 * 11, done_bar = bar0 + 8 * 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + 6 * BT_TILE + 8 * 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(ds_ready, 128);
    mbar_init(st_free, 1);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  qb_pdl_trigger();  // after the TMEM allocation: the next kernel cannot take it from this CTA

  if (warp == 0 && lane < 2) {
    // ------------------------------------------------------------ TMA producers: lane 0 Q, dO and K; lane 1 V
    if (lane == 0) {
      mbar_expect_tx(q_full, 2 * BT_TILE);
      for (int d = 0; d < 2; ++d)
        for (int hh = 0; hh < 2; ++hh) {
          tma_load_2d(sQ + d * BT_HALF + hh * (BT_HALF / 2), &tq, (h0 + hh) * 128 + d * 64, s0 + q_start, q_full);
          tma_load_2d(sDO + d * BT_HALF + hh * (BT_HALF / 2), &tdo, (h0 + hh) * 128 + d * 64, s0 + q_start, q_full);
        }
    }
    uint32_t issued = 0, last_parity = 0;
    for (int j = 0; j < n_tiles && !*abort_flag; ++j) {
      const int st = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      const uint32_t empty = lane == 0 ? k_empty(st) : v_empty(st), full = lane == 0 ? k_full(st) : v_full(st);
      if (!mbar_wait(empty, ph ^ 1, abort_flag, p.err)) break;
      mbar_expect_tx(full, BT_TILE);
      for (int d = 0; d < 2; ++d)
        tma_load_2d((lane == 0 ? sK(st) : sV(st)) + d * BT_HALF, lane == 0 ? &tk : &tv, kvh * 128 + d * 64,
                    s0 + j * BT_KEYS, full);
      issued |= 1u << st;
      last_parity = (last_parity & ~(1u << st)) | (ph << st);
    }
    if (lane == 0) mbar_drain(q_full, 0);
    for (int st = 0; st < 2; ++st)
      if (issued & (1u << st)) mbar_drain(lane == 0 ? k_full(st) : v_full(st), (last_parity >> st) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    auto issue_s_dp = [&](int j) {  // S = Q K_j^T, dP = dO V_j^T
      const int st = j & 1;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ko = (k >> 2) * BT_HALF + (k & 3) * 32;
        umma_bf16(tmem + DQ_S, sw128_kmajor_desc(sQ + ko), sw128_kmajor_desc(sK(st) + ko), IDESC_BT_KK, k > 0);
        umma_bf16(tmem + DQ_DP, sw128_kmajor_desc(sDO + ko), sw128_kmajor_desc(sV(st) + ko), IDESC_BT_KK, k > 0);
      }
      umma_commit(s_full);
      umma_commit(v_empty(st));
    };
    bool ok = mbar_wait(q_full, 0, abort_flag, p.err) && mbar_wait(k_full(0), 0, abort_flag, p.err) &&
              mbar_wait(v_full(0), 0, abort_flag, p.err);
    if (ok) {
      tc_fence_after();
      issue_s_dp(0);
    }
    for (int j = 0; ok && j < n_tiles; ++j) {
      const int st = j & 1;
      if (!mbar_wait(ds_ready, (uint32_t)j & 1u, abort_flag, p.err)) break;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 8; ++k)  // 128 keys in K-steps of 16: dS columns 8k, K rows 16k (read MN-major)
        umma_bf16_ts(tmem + DQ_ACC, tmem + DQ_DP + 8 * k, sw128_mn_desc(sK(st) + k * 16 * 128, BT_HALF), IDESC_BT_TS,
                     (j > 0 || k > 0) ? 1u : 0u);
      umma_commit(k_empty(st));
      umma_commit(st_free);
      if (j + 1 < n_tiles) {
        const int sn = (j + 1) & 1;
        const uint32_t pn = (uint32_t)((j + 1) >> 1) & 1u;
        if (!mbar_wait(st_free, (uint32_t)j & 1u, abort_flag, p.err) || !mbar_wait(k_full(sn), pn, abort_flag, p.err) ||
            !mbar_wait(v_full(sn), pn, abort_flag, p.err))
          break;
        tc_fence_after();
        issue_s_dp(j + 1);
      }
    }
    umma_commit(done_bar);
    mbar_drain(done_bar, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ dS and the epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int hh = r >> 6, pos = q_start + (r & 63);
    const bool live = pos < L;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    float l2 = INFINITY, dl = 0.f;
    if (live) {
      const int64_t idx = (int64_t)(h0 + hh) * p.total + s0 + pos;
      l2 = p.lse[idx] * 1.4426950408889634f;
      dl = p.delta[idx];
    }
    const int lim = live ? pos : -1;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      // tcgen05.ld/st below are warp-collective: the warp leaves together
      if (__any_sync(0xffffffffu, !mbar_wait(s_full, (uint32_t)j & 1u, abort_flag, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = j * BT_KEYS;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t sv[32], dv[32], pk[16];
        tmem_ld32_nowait(t_lane + DQ_S + c, sv);
        tmem_ld32_nowait(t_lane + DQ_DP + c, dv);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k = k0 + c + 2 * i;
          const float p0 = k <= lim ? fast_exp2(fmaf(__uint_as_float(sv[2 * i]), p.scale_log2, -l2)) : 0.f;
          const float p1 = k + 1 <= lim ? fast_exp2(fmaf(__uint_as_float(sv[2 * i + 1]), p.scale_log2, -l2)) : 0.f;
          pk[i] = pack_bf16x2(p0 * (__uint_as_float(dv[2 * i]) - dl), p1 * (__uint_as_float(dv[2 * i + 1]) - dl));
        }
        tmem_st16(t_lane + DQ_DP + c / 2, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    if (ok && __all_sync(0xffffffffu, mbar_wait(done_bar, 0, abort_flag, p.err))) {
      tc_fence_after();
      bf16* qrow = dq + (int64_t)(s0 + pos) * p.stride + (h0 + hh) * 128;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t a[32];
        tmem_ld32(t_lane + DQ_ACC + c, a);
        if (live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(a[8 * q + 0]) * p.scale, __uint_as_float(a[8 * q + 1]) * p.scale);
            w.y = pack_bf16x2(__uint_as_float(a[8 * q + 2]) * p.scale, __uint_as_float(a[8 * q + 3]) * p.scale);
            w.z = pack_bf16x2(__uint_as_float(a[8 * q + 4]) * p.scale, __uint_as_float(a[8 * q + 5]) * p.scale);
            w.w = pack_bf16x2(__uint_as_float(a[8 * q + 6]) * p.scale, __uint_as_float(a[8 * q + 7]) * p.scale);
            reinterpret_cast<uint4*>(qrow + c)[q] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}

}  // namespace

// dQ of the dense causal attention on tcgen05 (same shapes as attn_bwd_dkdv_tc_launch).
int attn_bwd_dq_tc_launch(const void* q, const void* k, const void* v, int64_t stride, const void* dout,
                          int64_t o_stride, const float* lse, const float* delta, const int32_t* cu_seqlens,
                          const int32_t* tile_info, int n_tiles, int hq, int hkv, float scale, int64_t total, void* dq,
                          int* err, cudaStream_t st) {
  const auto al16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  if (!al16(q) || !al16(k) || !al16(v) || !al16(dout) || !al16(dq) || stride % 8 || o_stride % 8)
    return QB_ERR_INVALID;
  if (total <= 0 || n_tiles <= 0) return QB_OK;
  CUtensorMap tq, tk, tv, tdo;
  if (!at_tmap(&tq, q, (uint64_t)hq * 128, (uint64_t)total, (uint64_t)stride, 64) ||
      !at_tmap(&tk, k, (uint64_t)hkv * 128, (uint64_t)total, (uint64_t)stride, BT_KEYS) ||
      !at_tmap(&tv, v, (uint64_t)hkv * 128, (uint64_t)total, (uint64_t)stride, BT_KEYS) ||
      !at_tmap(&tdo, dout, (uint64_t)hq * 128, (uint64_t)total, (uint64_t)o_stride, 64))
    return QB_ERR_INVALID;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_dq_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM_TC) !=
        cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  AttnBwdTcParams p{cu_seqlens, tile_info, hq, hkv, scale, scale * 1.4426950408889634f, lse, delta, total,
                    nullptr, nullptr, stride, err};
  return qb_launch_ex(attn_bwd_dq_tc_kernel, dim3((unsigned)n_tiles, (unsigned)hkv), dim3(DQ_THREADS), DQ_SMEM_TC,
                      st, 1, true, tq, tk, tv, tdo, p, (bf16*)dq);
}
