// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), sm_100a.
//
//   C[M, N] (=|+=) A[M, K] . B[N, K]^T      A, B bf16 K-major (nn.Linear weight layout)
//
// Persistent kernel, one CTA per SM, 192 threads:
//   warp 0     TMA producer: 128x64 A and BNx64 B tiles into a STAGES-deep ring of
//              128B-swizzled shared-memory stages (mbarrier full/empty pairs);
//   warp 1     allocates 2*BN TMEM columns; one thread issues tcgen05.mma (M=128,
//              N=BN, K=16) into a double-buffered fp32 accumulator and commits
//              stage releases / tile completion to mbarriers;
//   warps 2-5  epilogue: tcgen05.ld of the accumulator (each warp owns 32 TMEM lanes =
//              32 rows), conversion and global stores, then release of the buffer so
//              the next tile's MMAs overlap this tile's stores.
// Products whose 256x256 tiles fill every SM pair run on gemm_pair_kernel instead: a cluster
// of two CTAs issues tcgen05.mma.cta_group::2 (M = 256, N = 256), each CTA loading half of the
// operands (see its comment).
// Every mbarrier wait is bounded: on timeout the kernel raises QB_DEVERR_TIMEOUT, all
// roles leave their loops, the producer waits (bounded) for its own copies, TMEM is
// freed and the kernel returns.  Each CTA issues its own TMA loads from this GPU's memory.
#include "tcgen05.cuh"

namespace {

constexpr int BM = 128, BK = 64;
constexpr int THREADS = 192;
// ---------------------------------------------------------------- kernel
struct GemmParams {
  void* C;
  int64_t ldc;
  int M, N, K;
  int tiles_m, tiles_n;
  int vec_ok;  // every output row starts on a 16-byte boundary: 16-byte stores allowed
  int* err;
  // MODE 3 (lm_head log-prob) only:
  const int64_t* targets;  // [M] target column of each row
  float2* lse_part;        // [M, n_part]: per N tile, (max, sum of exp) of the row in the log2 domain
  float* tgt_logit;        // [M] fp32 logit at the target column
  int n_part;              // row pitch of lse_part (= number of N tiles of the launch)
  int b_static;            // B is written by no kernel still in flight: it may be read before the PDL wait
  int ksplit;              // pair kernel, MODE 2: K split over this many pairs per tile (atomic adds to C)
  // MODE 4 (gate_up projection -> SwiGLU): B is the [2*half, K] gate_up weight (gate rows, then up
  // rows); an N tile of width BN holds BN/2 gate columns and the same BN/2 up columns; C receives
  // silu(gate) * up [M, N = half], C2 (nullable) the bf16 gate_up itself [M, 2*half] for a backward.
  void* C2;
  int64_t ld2;
  int half;
  // MODE 5 (qkv projection -> QK-norm + RoPE, + paged KV store): the output columns are 128-wide
  // heads, q heads [0, hq), k heads [hq, hq+hkv), then v; C (nullable) receives the rotated q/k and
  // the v columns, C2 (nullable) the bf16 projection itself.
  struct QkEpilogue {
    const int64_t* positions;  // [M]
    const float* cos_sin;      // [max_pos, 128]: cos | sin
    int64_t max_pos;
    const bf16* qw;            // q_norm / k_norm weights [128]
    const bf16* kw;
    float eps;
    int hq, hkv;
    bf16* q_out;               // nullable [M, hq, 128] rotated q
    bf16* k_cache;             // nullable [num_slots, hkv, 128]: rotated k of row r at slots[r]
    bf16* v_cache;             //                                   raw v
    const int32_t* slots;      // [M], -1 skips the store
    int64_t num_slots;
    float* q_rstd;             // nullable [M, hq] / [M, hkv] for a backward
    float* k_rstd;
  } qk;
};

// One epilogue thread's 32 consecutive fp32 accumulator columns of output row `row`, starting
// at column `col` (< N): bf16 store, fp32 store or fp32 accumulate by MODE.
template <int MODE>
QB_DEVICE void store_row32(const GemmParams& p, int row, int col, const uint32_t (&r)[32]) {
    const bool full = col + 32 <= p.N && p.vec_ok;
    if (MODE == 0) {
      bf16* dst = reinterpret_cast<bf16*>(p.C) + (int64_t)row * p.ldc + col;
      if (full) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(r[8 * q + 0]), __uint_as_float(r[8 * q + 1]));
          v.y = pack_bf16x2(__uint_as_float(r[8 * q + 2]), __uint_as_float(r[8 * q + 3]));
          v.z = pack_bf16x2(__uint_as_float(r[8 * q + 4]), __uint_as_float(r[8 * q + 5]));
          v.w = pack_bf16x2(__uint_as_float(r[8 * q + 6]), __uint_as_float(r[8 * q + 7]));
          reinterpret_cast<uint4*>(dst)[q] = v;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col + i < p.N) dst[i] = f2bf(__uint_as_float(r[i]));
      }
    } else {
      float* dst = reinterpret_cast<float*>(p.C) + (int64_t)row * p.ldc + col;
      if (full) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 v = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
          if (MODE == 2) {
            const float4 o = reinterpret_cast<const float4*>(dst)[q];
            v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
          }
          reinterpret_cast<float4*>(dst)[q] = v;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col + i < p.N) dst[i] = (MODE == 2 ? dst[i] : 0.f) + __uint_as_float(r[i]);
      }
    }
}

// MODE 2 with K split over several CTAs: this thread's 32 fp32 columns added to C atomically (16-byte
// vector adds where the row is aligned), since the splits of a tile finish in any order.
QB_DEVICE void red_row32(const GemmParams& p, int row, int col, const uint32_t (&r)[32]) {
  float* dst = reinterpret_cast<float*>(p.C) + (int64_t)row * p.ldc + col;
  if (col + 32 <= p.N && p.vec_ok) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      atomicAdd(reinterpret_cast<float4*>(dst) + q, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                                __uint_as_float(r[4 * q + 2]),
                                                                __uint_as_float(r[4 * q + 3])));
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col + i < p.N) atomicAdd(dst + i, __uint_as_float(r[i]));
  }
}

// MODE 3 (lm_head -> log-softmax -> gather): the epilogue thread that holds row `row` of a tile
// folds each 32-column chunk of fp32 logits into a running (max, sum of exp) pair in the log2
// domain, keeps the target column's logit when the chunk holds it, and stores the bf16 logits
// only when the caller asked for them (p.C != nullptr).  Logits never leave the SM otherwise.
struct LseAcc {
  float m2, s, tv;
  bool has_t;
};

QB_DEVICE void lse_fold32(const GemmParams& p, int row, int col, int64_t tgt, const uint32_t (&r)[32], LseAcc& a) {
  constexpr float L2E = 1.4426950408889634f;  // log2(e)
  if (p.C) store_row32<0>(p, row, col, r);
  const int nvalid = p.N - col < 32 ? p.N - col : 32;
  float cm = -INFINITY;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < nvalid) cm = fmaxf(cm, __uint_as_float(r[i]));
  if ((uint64_t)(tgt - col) < 32u) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (col + i == tgt) a.tv = __uint_as_float(r[i]);
    a.has_t = true;
  }
  const float cm2 = cm * L2E;
  if (cm2 > a.m2) {
    a.s *= exp2f(a.m2 - cm2);
    a.m2 = cm2;
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i)
    if (i < nvalid) s += exp2f(fmaf(__uint_as_float(r[i]), L2E, -a.m2));
  a.s += s;
}

// Folds the accumulator rows of one tile (this thread's row, BN columns from TMEM column `tcol`).
template <int BN>
QB_DEVICE void lse_tile(const GemmParams& p, uint32_t taddr, int row, bool row_ok, int n0, int n_tile) {
  LseAcc a{-INFINITY, 0.f, 0.f, false};
  const int64_t tgt = (row_ok && p.targets) ? p.targets[row] : -1;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(taddr + c, r);  // warp-collective: every lane loads before any lane skips
    const int col = n0 + c;
    if (!row_ok || col >= p.N) continue;
    lse_fold32(p, row, col, tgt, r, a);
  }
  if (row_ok) {
    p.lse_part[(int64_t)row * p.n_part + n_tile] = make_float2(a.m2, a.s);
    if (a.has_t) p.tgt_logit[row] = a.tv;
  }
}

// MODE 4: this thread's row of a tile whose TMEM columns [0, BN/2) hold gate and [BN/2, BN) the
// matching up columns.  Both are rounded to bf16 first -- the values the unfused path stores and
// its SwiGLU kernel reads -- so the result has the same bits as gate_up GEMM + SwiGLU kernel.
template <int BN>
QB_DEVICE void swiglu_tile(const GemmParams& p, uint32_t taddr, int row, bool row_ok, int n0) {
  constexpr int H = BN / 2;
#pragma unroll 1
  for (int c = 0; c < H; c += 32) {
    uint32_t g[32], u[32];
    tmem_ld32(taddr + c, g);  // warp-collective: every lane loads before any lane skips
    tmem_ld32(taddr + H + c, u);
    const int col = n0 + c;
    if (!row_ok || col >= p.N) continue;
    const bool full = col + 32 <= p.N && p.vec_ok;
    bf16* dst = reinterpret_cast<bf16*>(p.C) + (int64_t)row * p.ldc + col;
    bf16* gdst = p.C2 ? reinterpret_cast<bf16*>(p.C2) + (int64_t)row * p.ld2 + col : nullptr;
    uint32_t gp[16], up[16], hp[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      gp[i] = pack_bf16x2(__uint_as_float(g[2 * i]), __uint_as_float(g[2 * i + 1]));
      up[i] = pack_bf16x2(__uint_as_float(u[2 * i]), __uint_as_float(u[2 * i + 1]));
      const float2 gf = unpack_bf16x2(gp[i]), uf = unpack_bf16x2(up[i]);
      hp[i] = pack_bf16x2(qb_silu(gf.x) * uf.x, qb_silu(gf.y) * uf.y);
    }
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        reinterpret_cast<uint4*>(dst)[q] = make_uint4(hp[4 * q], hp[4 * q + 1], hp[4 * q + 2], hp[4 * q + 3]);
        if (gdst) {
          reinterpret_cast<uint4*>(gdst)[q] = make_uint4(gp[4 * q], gp[4 * q + 1], gp[4 * q + 2], gp[4 * q + 3]);
          reinterpret_cast<uint4*>(gdst + p.half)[q] =
              make_uint4(up[4 * q], up[4 * q + 1], up[4 * q + 2], up[4 * q + 3]);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (col + i >= p.N) break;
        const uint32_t w = i & 1 ? 16 : 0;
        dst[i] = __ushort_as_bfloat16((unsigned short)(hp[i >> 1] >> w));
        if (gdst) {
          gdst[i] = __ushort_as_bfloat16((unsigned short)(gp[i >> 1] >> w));
          gdst[p.half + i] = __ushort_as_bfloat16((unsigned short)(up[i >> 1] >> w));
        }
      }
    }
  }
}

// MODE 5: this thread's row of a tile of whole 128-wide heads.  The projection is rounded to bf16
// (the value the unfused path stores), then QK-norm and RoPE follow the standalone kernel's
// arithmetic step for step (its half-warp reduction order included), so the bits are the same.
QB_DEVICE void st_head(bf16* dst, const uint32_t (&x)[64]) {
#pragma unroll
  for (int q = 0; q < 16; ++q)
    reinterpret_cast<uint4*>(dst)[q] = make_uint4(x[4 * q], x[4 * q + 1], x[4 * q + 2], x[4 * q + 3]);
}

// MODE 5, before this thread's accumulator row is ready: its token's rotation-table row (512 B)
// into L1, so the epilogue's table reads do not wait on L2.
QB_DEVICE void qknorm_prefetch(const GemmParams& p, int row) {
  if (row >= p.M) return;
  int64_t pos = p.qk.positions[row];
  if (pos < 0 || pos >= p.qk.max_pos) pos = 0;
  const float* cs = p.qk.cos_sin + pos * 128;
#pragma unroll
  for (int q = 0; q < 4; ++q) prefetch_l1(cs + q * 32);
}

template <int BN>
QB_DEVICE void qknorm_tile(const GemmParams& p, uint32_t taddr, int row, bool row_ok, int n0) {
  static_assert(BN % 128 == 0, "whole heads per tile");
  const GemmParams::QkEpilogue& e = p.qk;
#pragma unroll 1
  for (int hh = 0; hh < BN / 128; ++hh) {
    uint32_t x[64];  // the head's 128 values as bf16 pairs
#pragma unroll
    for (int c = 0; c < 128; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + hh * 128 + c, r);  // warp-collective: every lane loads before any lane skips
#pragma unroll
      for (int i = 0; i < 16; ++i) x[c / 2 + i] = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    }
    const int col = n0 + hh * 128;
    if (!row_ok || col >= p.N) continue;
    const int head = col / 128;
    const bool is_q = head < e.hq, is_v = head >= e.hq + e.hkv;
    if (p.C2) st_head(reinterpret_cast<bf16*>(p.C2) + (int64_t)row * p.ld2 + col, x);
    int64_t slot = -1;
    if (e.k_cache) {
      slot = e.slots[row];
      if (slot >= e.num_slots || slot < -1) {
        qb_set_err(p.err, QB_DEVERR_SLOT);
        slot = -1;
      }
    }
    bf16* out = p.C ? reinterpret_cast<bf16*>(p.C) + (int64_t)row * p.ldc + col : nullptr;
    if (is_v) {  // v: the projection itself (and into the cache)
      if (out) st_head(out, x);
      if (slot >= 0) st_head(e.v_cache + (slot * e.hkv + (head - e.hq - e.hkv)) * 128, x);
      continue;
    }
    int64_t pos = e.positions[row];
    if (pos < 0 || pos >= e.max_pos) {
      qb_set_err(p.err, QB_DEVERR_SHAPE);
      pos = 0;
    }
    float part[16];
#pragma unroll
    for (int g = 0; g < 16; ++g) {
      float v8[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(x[4 * g + i]);
        v8[2 * i] = f.x;
        v8[2 * i + 1] = f.y;
      }
      part[g] = qk_sumsq8(v8);
    }
    const float rstd = qk_rstd(qk_sumsq_tree(part), e.eps);
    const bf16* w = is_q ? e.qw : e.kw;
    const float* cs = e.cos_sin + pos * 128;
#pragma unroll
    for (int j = 0; j < 64; j += 4) {  // RoPE pairs (j+i, j+i+64), i < 4: 16-byte table loads
      const float4 c = *reinterpret_cast<const float4*>(cs + j), sn = *reinterpret_cast<const float4*>(cs + 64 + j);
      const uint2 wlr = *reinterpret_cast<const uint2*>(w + j), whr = *reinterpret_cast<const uint2*>(w + 64 + j);
      const float cc[4] = {c.x, c.y, c.z, c.w}, ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const float2 lo = unpack_bf16x2(x[j / 2 + h2]), hi = unpack_bf16x2(x[32 + j / 2 + h2]);
        const float2 wl = unpack_bf16x2(h2 ? wlr.y : wlr.x), wh = unpack_bf16x2(h2 ? whr.y : whr.x);
        const float c0 = cc[2 * h2], c1 = cc[2 * h2 + 1], s0 = ss[2 * h2], s1 = ss[2 * h2 + 1];
        const float xl0 = round_bf16((lo.x * rstd) * wl.x), xl1 = round_bf16((lo.y * rstd) * wl.y);
        const float xh0 = round_bf16((hi.x * rstd) * wh.x), xh1 = round_bf16((hi.y * rstd) * wh.y);
        x[j / 2 + h2] = pack_bf16x2(qk_rope_lo(xl0, xh0, c0, s0), qk_rope_lo(xl1, xh1, c1, s1));
        x[32 + j / 2 + h2] = pack_bf16x2(qk_rope_hi(xh0, xl0, c0, s0), qk_rope_hi(xh1, xl1, c1, s1));
      }
    }
    if (is_q) {
      if (e.q_rstd) e.q_rstd[(int64_t)row * e.hq + head] = rstd;
      if (e.q_out) st_head(e.q_out + ((int64_t)row * e.hq + head) * 128, x);
    } else {
      if (e.k_rstd) e.k_rstd[(int64_t)row * e.hkv + (head - e.hq)] = rstd;
      if (slot >= 0) st_head(e.k_cache + (slot * e.hkv + (head - e.hq)) * 128, x);
    }
    if (out) st_head(out, x);
  }
}

template <int BN, int STAGES, int MODE, bool A_MN, bool B_MN>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int ACC_STRIDE = BN <= 128 ? BN : 256;  // TMEM columns between the two accumulators
  static constexpr int TMEM_COLS = 2 * ACC_STRIDE;          // double-buffered (power of two)
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static constexpr uint32_t IDESC = (1u << 4)            // D fp32
                                    | (1u << 7)          // A bf16
                                    | (1u << 10)         // B bf16
                                    | ((A_MN ? 1u : 0u) << 15) | ((B_MN ? 1u : 0u) << 16)
                                    | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};

// Loads one operand tile of ROWS (M or N) x BK into a stage: one {64, ROWS} box for a K-major
// operand, ROWS/64 {64, 64} boxes (one per 64-wide MN atom) for an MN-major operand.
template <bool MN_MAJOR, int ROWS>
QB_DEVICE void load_operand(uint32_t dst, const CUtensorMap* map, int k0, int mn0, uint32_t bar) {
  if (MN_MAJOR) {
#pragma unroll
    for (int a = 0; a < ROWS / 64; ++a) tma_load_2d(dst + a * 64 * 128, map, mn0 + a * 64, k0, bar);
  } else {
    tma_load_2d(dst, map, k0, mn0, bar);
  }
}

// The B rows of N tile `tile_n` (BN rows x 64 K): one box, or in MODE 4 the tile's BN/2 gate rows
// and the same BN/2 up rows (`half` rows further) as two boxes of BN/2 rows.
template <int MODE, bool B_MN, int BN>
QB_DEVICE void load_b(uint32_t sb, const CUtensorMap* map, int k0, int tile_n, int half, uint32_t bar) {
  if constexpr (MODE == 4) {
    static_assert(!B_MN, "the SwiGLU epilogue reads K-major weights");
    load_operand<B_MN, BN / 2>(sb, map, k0, tile_n * (BN / 2), bar);
    load_operand<B_MN, BN / 2>(sb + (BN / 2) * BK * 2, map, k0, half + tile_n * (BN / 2), bar);
  } else {
    load_operand<B_MN, BN>(sb, map, k0, tile_n * BN, bar);
  }
}

template <int BN, int STAGES, int MODE, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    GemmParams p) {
  using Cfg = GemmCfg<BN, STAGES, MODE, A_MN, B_MN>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;  // SW128 atoms need 1024-byte alignment
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + STAGES * Cfg::STAGE_BYTES;
  // barrier block: full[S], empty[S], tfull[2], tempty[2], then tmem base (u32) and abort flag
  auto full_bar = [&](int s) { return bar0 + 8 * s; };
  auto empty_bar = [&](int s) { return bar0 + 8 * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8 * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8 * (2 * STAGES + 2 + a); };
  const uint32_t done_bar = bar0 + 8 * (2 * STAGES + 4);  // completion of every MMA this CTA issued
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + STAGES * Cfg::STAGE_BYTES + 8 * (2 * STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = p.tiles_m * p.tiles_n;
  const int kblocks = (p.K + BK - 1) / BK;  // a K tail is zero-filled by TMA

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4 * 32);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
  }
  if (warp == 1) {  // TMEM allocation is warp-collective
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(Cfg::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  qb_pdl_trigger();  // after the TMEM allocation: the next kernel cannot take it from this CTA
  // With a static B (weights no kernel in flight writes), the producer requests the B halves of
  // its first tile's first ring stages before waiting for the kernel before: their DRAM trip
  // overlaps that kernel's tail.  Each such stage expects its full bytes, so it completes only
  // once the A half, requested after the wait, has landed too.
  int pre = 0;
  uint32_t issued = 0;  // producer: per-stage bit, a load is in flight
  if (warp == 0 && lane == 0 && p.b_static && (int)blockIdx.x < n_tiles) {
    const int tile_n = (int)blockIdx.x / p.tiles_m;
    pre = kblocks < STAGES ? kblocks : STAGES;
    for (int s = 0; s < pre; ++s) {
      mbar_expect_tx(full_bar(s), Cfg::STAGE_BYTES);
      load_b<MODE, B_MN, BN>(base + s * Cfg::STAGE_BYTES + Cfg::A_BYTES, &tmap_b, s * BK, tile_n, p.half, full_bar(s));
      issued |= 1u << s;
    }
  }
  qb_pdl_wait();  // A, and C in MODE 2, may come from the kernel before

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t last_parity = 0;  // per-stage bit: the phase parity of its load in flight
    for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
      const int m0 = (t % p.tiles_m) * BM, tile_n = t / p.tiles_m;
      for (int kb = 0; kb < kblocks; ++kb) {
        // the first `pre` stages of the first tile: fresh barriers, B already requested
        const bool pre_b = t == (int)blockIdx.x && kb < pre;
        if (!pre_b && !mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) break;
        const uint32_t sa = base + stage * Cfg::STAGE_BYTES, sb = sa + Cfg::A_BYTES;
        if (!pre_b) mbar_expect_tx(full_bar(stage), Cfg::STAGE_BYTES);
        load_operand<A_MN, BM>(sa, &tmap_a, kb * BK, m0, full_bar(stage));
        if (!pre_b) load_b<MODE, B_MN, BN>(sb, &tmap_b, kb * BK, tile_n, p.half, full_bar(stage));
        issued |= 1u << stage;
        last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
    // never leave with a copy in flight into this CTA's shared memory
    for (int s = 0; s < STAGES; ++s)
      if (issued & (1u << s)) mbar_drain(full_bar(s), (last_parity >> s) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
      if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1, abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t d = tmem + acc * Cfg::ACC_STRIDE;
      bool ok = true;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = base + stage * Cfg::STAGE_BYTES, sb = sa + Cfg::A_BYTES;
#pragma unroll
        for (int j = 0; j < BK / 16; ++j)
          umma_bf16(d, operand_desc<A_MN>(sa, j), operand_desc<B_MN>(sb, j), Cfg::IDESC, (kb | j) != 0);
        umma_commit(empty_bar(stage));  // stage reusable once these MMAs have read it
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      umma_commit(tfull_bar(acc));  // accumulator complete
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    // no MMA may still be reading shared memory or writing TMEM when the CTA leaves
    umma_commit(done_bar);
    mbar_drain(done_bar, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes [32*quarter, 32*quarter+32)
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < n_tiles && !*abort_flag; t += gridDim.x) {
      const int m0 = (t % p.tiles_m) * BM, n0 = (t / p.tiles_m) * (MODE == 4 ? BN / 2 : BN);
      if constexpr (MODE == 5) qknorm_prefetch(p, m0 + row_in_tile);
      // tcgen05.ld is warp-collective: the warp leaves (or goes on) together
      if (__any_sync(0xffffffffu, !mbar_wait(tfull_bar(acc), acc_phase, abort_flag, p.err))) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      if constexpr (MODE == 3) {
        lse_tile<BN>(p, tmem + ((uint32_t)(quarter * 32) << 16) + acc * Cfg::ACC_STRIDE, row, row_ok, n0,
                     t / p.tiles_m);
      } else if constexpr (MODE == 4) {
        swiglu_tile<BN>(p, tmem + ((uint32_t)(quarter * 32) << 16) + acc * Cfg::ACC_STRIDE, row, row_ok, n0);
      } else if constexpr (MODE == 5) {
        qknorm_tile<BN>(p, tmem + ((uint32_t)(quarter * 32) << 16) + acc * Cfg::ACC_STRIDE, row, row_ok, n0);
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + acc * Cfg::ACC_STRIDE + c, r);
          const int col = n0 + c;
          if (!row_ok || col >= p.N) continue;
          store_row32<MODE>(p, row, col, r);
        }
      }
      tc_fence_before();
      mbar_arrive(tempty_bar(acc));  // accumulator free for the tile after next
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Cfg::TMEM_COLS));
  }
}

// ---------------------------------------------------------------- CTA-pair kernel (cta_group::2)
// A cluster of two CTAs on two SMs computes a 256 x PBN tile (PBN = 256, 192 or 128).  Per 64-deep
// K block each CTA loads its own 128 rows of A and its own PBN/2-row half of B (N) into its ring,
// signalling the stage barrier of the even CTA (the leader), whose one thread issues
// tcgen05.mma.cta_group::2 (M = 256, N = PBN) reading both CTAs' stages; each CTA's TMEM receives
// its 128 rows of the accumulator (double-buffered).  Each SM pulls (128 + PBN/2) rows of operands
// per K block for a 128 x PBN share of the product, against (128 + PBN) rows for the same share
// on one CTA.  The dispatcher uses PBN = 256, for products that fill every SM pair; the narrower
// tiles pull fewer bytes per SM but measured slower on the decode step's M = 512 products, whose
// time is latency rather than operand traffic.  The leader's commits release both CTAs' stages
// and accumulators (one commit per CTA's barrier); each CTA's epilogue drains its own TMEM rows
// and tells the leader through a remote arrive.  Every wait is bounded; each CTA loads from this
// GPU's memory only.
constexpr int P_HALF_BYTES = 128 * BK * 2;  // 16 KB: 128 rows x 64 K of A (this CTA's rows)

template <int PBN>
struct PairShape {
  static constexpr int B_ROWS = PBN / 2;                       // this CTA's rows of B
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static constexpr int STAGE_BYTES = P_HALF_BYTES + B_BYTES;
  static constexpr int STAGES = (200 * 1024) / STAGE_BYTES;  // 6 / 7 / 8 stages
  static constexpr int ACC_STRIDE = PBN <= 128 ? PBN : 256;   // TMEM columns between the accumulators
  static constexpr int TMEM_COLS = 2 * ACC_STRIDE;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

template <bool A_MN, bool B_MN, int PBN>
struct PairCfg {
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((A_MN ? 1u : 0u) << 15) |
                                    ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(PBN >> 3) << 17) |
                                    ((uint32_t)(256 >> 4) << 24);
};

// Arrivals on a barrier of either CTA of the pair, with the default (CTA-scope release)
// semantics: the data they guard arrives by TMA transaction counts or is TMEM read back with
// tcgen05.wait, so no cluster-wide fence is needed (one would stall the producer on its own
// copies in flight).
QB_DEVICE void mbar_expect_tx_remote(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
QB_DEVICE void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Bounded wait on a barrier of this CTA that the other CTA of the pair may signal.
QB_DEVICE bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
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
// TMA load into this CTA's shared memory whose completion is counted on a barrier of either CTA
// of the pair; each CTA fetches only its own half of the operands.
QB_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
// ROWS rows (M or N) x 64 K of one operand: one K-major box, or ROWS/64 MN-major 64-wide atoms.
template <bool MN_MAJOR, int ROWS>
QB_DEVICE void load_half(uint32_t dst, const CUtensorMap* map, int k0, int mn0, uint32_t bar) {
  if constexpr (MN_MAJOR) {
    static_assert(ROWS % 64 == 0, "MN-major operands load whole 64-wide atoms");
#pragma unroll
    for (int a = 0; a < ROWS / 64; ++a) tma_load_2d_pair(dst + a * 64 * 128, map, mn0 + a * 64, k0, bar);
  } else {
    tma_load_2d_pair(dst, map, k0, mn0, bar);
  }
}
QB_DEVICE void umma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive (once) on a barrier of either CTA when the pair's prior MMAs have completed.
QB_DEVICE void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

template <int MODE, bool A_MN, bool B_MN, int PBN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                 GemmParams p) {
  using Sh = PairShape<PBN>;
  constexpr int P_STAGES = Sh::STAGES;
  constexpr int P_STAGE_BYTES = Sh::STAGE_BYTES;
  constexpr int P_TMEM_COLS = Sh::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;  // the same offset in both CTAs of the pair
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + P_STAGES * P_STAGE_BYTES;
  // full[S] (leader: one expect_tx arrive per CTA), empty[S], tfull[2], tempty[2] (leader: 256
  // epilogue threads of both CTAs), done, then tmem base and abort flag
  auto full_bar = [&](int s) { return bar0 + 8 * s; };
  auto empty_bar = [&](int s) { return bar0 + 8 * (P_STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8 * (2 * P_STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8 * (2 * P_STAGES + 2 + a); };
  const uint32_t done_bar = bar0 + 8 * (2 * P_STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + P_STAGES * P_STAGE_BYTES + 8 * (2 * P_STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank(), peer = rank ^ 1;
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  constexpr int TN = MODE == 4 ? PBN / 2 : PBN;  // output columns of an N tile
  static_assert(MODE != 4 || !B_MN, "the SwiGLU epilogue reads K-major weights");
  const int tiles_m = (p.M + 255) / 256, tiles_n = (p.N + TN - 1) / TN;
  const int n_tiles = tiles_m * tiles_n;
  const int kblocks = (p.K + BK - 1) / BK;
  // work units: (tile, K split), split-major; a unit covers K blocks [kb0, kb1) of its tile
  const int ksplit = MODE == 2 && p.ksplit > 1 ? p.ksplit : 1;
  const int n_units = n_tiles * ksplit;
  auto unit_kb = [&](int u, int& kb0, int& kb1) {
    const int sp = u / n_tiles;
    kb0 = sp * kblocks / ksplit;
    kb1 = (sp + 1) * kblocks / ksplit;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(full_bar(s), 2);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 2 * 4 * 32);
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
  }
  if (warp == 1) {  // both CTAs of the pair allocate together
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(P_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // barriers and TMEM of both CTAs exist before either uses the other's
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  qb_pdl_trigger();  // after the TMEM allocation: the next kernel cannot take it from this CTA
  qb_pdl_wait();     // operands and C may come from the kernel before

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer (each CTA)
    int stage = 0;
    uint32_t phase = 0;
    for (int u = pair; u < n_units && !*abort_flag; u += n_pairs) {
      const int t = u % n_tiles;
      int kb0, kb1;
      unit_kb(u, kb0, kb1);
      // this CTA's half of B: rows [rank * PBN/2, ...) of the tile; in MODE 4 the even CTA takes the
      // tile's gate rows and the odd CTA the same rows of up
      const int m0 = (t % tiles_m) * 256 + (int)rank * 128,
                n0 = MODE == 4 ? (rank ? p.half : 0) + (t / tiles_m) * TN : (t / tiles_m) * PBN + (int)rank * Sh::B_ROWS;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1, abort_flag, p.err)) break;
        const uint32_t sa = base + stage * P_STAGE_BYTES, sb = sa + P_HALF_BYTES;
        const uint32_t lf = cluster_addr(full_bar(stage), 0);
        mbar_expect_tx_remote(lf, P_STAGE_BYTES);
        load_half<A_MN, 128>(sa, &tmap_a, kb * BK, m0, lf);
        load_half<B_MN, Sh::B_ROWS>(sb, &tmap_b, kb * BK, n0, lf);
        if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1 && lane == 0 && leader) {
    // ------------------------------------------------------------ MMA issuer (leader)
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < n_units && !*abort_flag; u += n_pairs) {
      if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1, abort_flag, p.err)) break;
      tc_fence_after();
      const uint32_t d = tmem + acc * Sh::ACC_STRIDE;
      int kb0, kb1;
      unit_kb(u, kb0, kb1);
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_cluster(full_bar(stage), phase, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = base + stage * P_STAGE_BYTES, sb = sa + P_HALF_BYTES;
#pragma unroll
        for (int j = 0; j < BK / 16; ++j)
          umma_pair(d, operand_desc<A_MN>(sa, j), operand_desc<B_MN>(sb, j), PairCfg<A_MN, B_MN, PBN>::IDESC,
                    (kb != kb0 || j != 0));
        umma_commit_pair(empty_bar(stage));  // both CTAs' stage is free once these MMAs read it
        umma_commit_pair(cluster_addr(empty_bar(stage), peer));
        if (++stage == P_STAGES) { stage = 0; phase ^= 1; }
      }
      if (!ok) break;
      umma_commit_pair(tfull_bar(acc));  // both CTAs' accumulator rows are complete
      umma_commit_pair(cluster_addr(tfull_bar(acc), peer));
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    umma_commit_pair(done_bar);
    mbar_drain(done_bar, 0);
    if (*abort_flag) {  // copies the producers may still have in flight land before the CTAs leave
      for (int s = 0; s < P_STAGES; ++s) mbar_drain(full_bar(s), s < stage ? phase ^ 1 : phase);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue (each CTA, its 128 rows)
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t leader_tempty0 = cluster_addr(tempty_bar(0), 0), leader_tempty1 = cluster_addr(tempty_bar(1), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = pair; u < n_units && !*abort_flag; u += n_pairs) {
      const int t = u % n_tiles;
      const int m0 = (t % tiles_m) * 256 + (int)rank * 128, n0 = (t / tiles_m) * TN;
      if constexpr (MODE == 5) qknorm_prefetch(p, m0 + row_in_tile);
      // tcgen05.ld is warp-collective: the warp leaves (or goes on) together
      if (__any_sync(0xffffffffu, !mbar_wait_cluster(tfull_bar(acc), acc_phase, abort_flag, p.err))) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      if constexpr (MODE == 3) {
        lse_tile<PBN>(p, tmem + ((uint32_t)(quarter * 32) << 16) + acc * Sh::ACC_STRIDE, row, row_ok, n0,
                      t / tiles_m);
      } else if constexpr (MODE == 4) {
        swiglu_tile<PBN>(p, tmem + ((uint32_t)(quarter * 32) << 16) + acc * Sh::ACC_STRIDE, row, row_ok, n0);
      } else if constexpr (MODE == 5) {
        qknorm_tile<PBN>(p, tmem + ((uint32_t)(quarter * 32) << 16) + acc * Sh::ACC_STRIDE, row, row_ok, n0);
      } else {
#pragma unroll 1
        for (int c = 0; c < PBN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + acc * Sh::ACC_STRIDE + c, r);
          const int col = n0 + c;
          if (!row_ok || col >= p.N) continue;
          if (MODE == 2 && ksplit > 1)
            red_row32(p, row, col, r);
          else
            store_row32<MODE>(p, row, col, r);
        }
      }
      tc_fence_before();
      mbar_arrive_remote(acc == 0 ? leader_tempty0 : leader_tempty1);  // the leader may reuse it
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // neither CTA leaves while the other may still signal its barriers or TMEM
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P_TMEM_COLS));
  }
}

// ---------------------------------------------------------------- split-K clusters
// Skinny products with few output tiles and a long K (the decode step's o_proj and down_proj at
// M = 512: 32 tiles of 128 x 128 over K = 2048 / 3072) leave most SMs idle, and each busy SM
// pulls the whole K extent of its tile through its own port.  A cluster of S CTAs computes one
// 128 x 128 tile instead, CTA r over K blocks [r*KB/S, (r+1)*KB/S), so S SMs share the tile's
// loads.  The fp32 partials are summed in distributed shared memory: the tile's 128 rows are cut
// into S slices, CTA j owns slice j, and every other CTA pushes its partial rows of slice j into
// a receive buffer of CTA j with st.async, counted in bytes on CTA j's receive barrier; the
// owner's epilogue warps add them to their own accumulator rows and store the result (any MODE).
// One tile per cluster and one cluster per S SMs at most: the host launches this only when every
// cluster is resident at once.  Every wait is bounded; each CTA loads from this GPU's memory.
constexpr int S_STAGES = 4;
constexpr int S_BN = 128;
constexpr int S_STAGE_BYTES = (BM + S_BN) * BK * 2;  // 32 KB
constexpr int S_ROW = S_BN + 4;  // receive-buffer row pitch in floats: 16-byte pad, conflict-free v4 reads

template <int S>
struct SplitCfg {
  static constexpr int SLICE_ROWS = BM / S;                             // rows each CTA finishes
  static constexpr int RECV_BYTES = (S - 1) * SLICE_ROWS * S_ROW * 4;   // one slot per other CTA
  static constexpr uint32_t RECV_TX = (S - 1) * SLICE_ROWS * S_BN * 4;  // bytes pushed to each owner
  static constexpr int SMEM = S_STAGES * S_STAGE_BYTES + RECV_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

// Stores four fp32 words into another CTA's shared memory; the bytes count on that CTA's barrier.
QB_DEVICE void st_async_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "r"(a), "r"(b), "r"(c), "r"(d), "r"(bar)
               : "memory");
}

// Bounded wait for the partial rows the other CTAs pushed (cluster-scope acquire: the bytes were
// written by other CTAs' st.async).
QB_DEVICE bool recv_wait(uint32_t bar, volatile int* abort_flag, int* err) {
  const long long t0 = clock64();
  for (uint32_t i = 0;; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar)
        : "memory");
    if (ok) return true;
    if ((i & 255) == 255) {
      if (*abort_flag) return false;
      if (clock64() - t0 > WAIT_CYCLES) break;
    }
  }
  *abort_flag = 1;
  qb_set_err(err, QB_DEVERR_TIMEOUT);
  return false;
}

template <int S, int MODE, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(THREADS, 1)
gemm_split_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                  GemmParams p) {
  using Cfg = GemmCfg<S_BN, S_STAGES, MODE, A_MN, B_MN>;
  using Sc = SplitCfg<S>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023) & ~1023u;  // the same offset in every CTA of the cluster
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t recv = base + S_STAGES * S_STAGE_BYTES;
  const uint32_t bar0 = recv + Sc::RECV_BYTES;
  // barrier block: full[S_STAGES], empty[S_STAGES], tfull, recv, done, then tmem base and abort flag
  auto full_bar = [&](int s) { return bar0 + 8 * s; };
  auto empty_bar = [&](int s) { return bar0 + 8 * (S_STAGES + s); };
  const uint32_t tfull_bar = bar0 + 8 * (2 * S_STAGES);
  const uint32_t recv_bar = tfull_bar + 8;
  const uint32_t done_bar = recv_bar + 8;
  const int bar_off = S_STAGES * S_STAGE_BYTES + Sc::RECV_BYTES + 8 * (2 * S_STAGES + 3);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + bar_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = (int)cluster_rank();
  const int tile = blockIdx.x / S;
  const int m0 = (tile % p.tiles_m) * BM, n0 = (tile / p.tiles_m) * S_BN;
  const int kblocks = (p.K + BK - 1) / BK;  // >= S (host check): every CTA gets a K block
  const int kb0 = rank * kblocks / S, kb1 = (rank + 1) * kblocks / S;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S_STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(recv_bar, 1);
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // the receive phase completes once the other CTAs' partial rows have all landed
    mbar_expect_tx(recv_bar, Sc::RECV_TX);
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(S_BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();  // every CTA's receive barrier exists before any CTA pushes into it
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  qb_pdl_trigger();  // after the TMEM allocation: the next kernel cannot take it from this CTA
  // A static B's first ring stages are requested before the wait for the kernel before (as in
  // gemm_tcgen05_kernel); each such stage completes once its A half, requested after, lands too.
  int pre = 0;
  uint32_t issued = 0;  // producer: per-stage bit, a load is in flight
  if (warp == 0 && lane == 0 && p.b_static) {
    pre = kb1 - kb0 < S_STAGES ? kb1 - kb0 : S_STAGES;
    for (int s = 0; s < pre; ++s) {
      mbar_expect_tx(full_bar(s), S_STAGE_BYTES);
      load_operand<B_MN, S_BN>(base + s * S_STAGE_BYTES + BM * BK * 2, &tmap_b, (kb0 + s) * BK, n0, full_bar(s));
      issued |= 1u << s;
    }
  }
  qb_pdl_wait();  // A, and C in MODE 2, may come from the kernel before

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t last_parity = 0;
    for (int kb = kb0; kb < kb1 && !*abort_flag; ++kb) {
      const bool pre_b = kb - kb0 < pre;  // fresh barrier, B already requested
      if (!pre_b && !mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.err)) break;
      const uint32_t sa = base + stage * S_STAGE_BYTES, sb = sa + BM * BK * 2;
      if (!pre_b) mbar_expect_tx(full_bar(stage), S_STAGE_BYTES);
      load_operand<A_MN, BM>(sa, &tmap_a, kb * BK, m0, full_bar(stage));
      if (!pre_b) load_operand<B_MN, S_BN>(sb, &tmap_b, kb * BK, n0, full_bar(stage));
      issued |= 1u << stage;
      last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == S_STAGES) { stage = 0; phase ^= 1; }
    }
    for (int s = 0; s < S_STAGES; ++s)
      if (issued & (1u << s)) mbar_drain(full_bar(s), (last_parity >> s) & 1);
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait(full_bar(stage), phase, abort_flag, p.err)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sa = base + stage * S_STAGE_BYTES, sb = sa + BM * BK * 2;
#pragma unroll
      for (int j = 0; j < BK / 16; ++j)
        umma_bf16(tmem, operand_desc<A_MN>(sa, j), operand_desc<B_MN>(sb, j), Cfg::IDESC, ((kb - kb0) | j) != 0);
      umma_commit(empty_bar(stage));
      if (++stage == S_STAGES) { stage = 0; phase ^= 1; }
    }
    if (ok) umma_commit(tfull_bar);
    umma_commit(done_bar);
    mbar_drain(done_bar, 0);
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue: push or reduce
    const int quarter = warp & 3;                   // TMEM lanes [32*quarter, 32*quarter+32)
    const int owner = quarter / (4 / S);            // CTA that finishes these 32 rows
    const int slice_row = (quarter % (4 / S)) * 32 + lane;  // row within the owner's slice
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    if (__all_sync(0xffffffffu, mbar_wait(tfull_bar, 0, abort_flag, p.err))) {  // warp-uniform (tcgen05.ld)
      tc_fence_after();
      if (owner != rank) {
        const int slot = (rank - owner - 1 + S) % S;  // this CTA's slot in the owner's buffer
        const uint32_t dst = cluster_addr(recv + (uint32_t)((slot * Sc::SLICE_ROWS + slice_row) * S_ROW * 4),
                                          (uint32_t)owner);
        const uint32_t rbar = cluster_addr(recv_bar, (uint32_t)owner);
#pragma unroll 1
        for (int c = 0; c < S_BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(t_lane + c, r);
#pragma unroll
          for (int v = 0; v < 8; ++v)
            st_async_v4(dst + (uint32_t)(c + 4 * v) * 4, r[4 * v], r[4 * v + 1], r[4 * v + 2], r[4 * v + 3], rbar);
        }
      } else if (__all_sync(0xffffffffu, recv_wait(recv_bar, abort_flag, p.err))) {
        const int row = m0 + quarter * 32 + lane;
        const bool row_ok = row < p.M;
        const float* slots = reinterpret_cast<const float*>(gbase + S_STAGES * S_STAGE_BYTES) + slice_row * S_ROW;
#pragma unroll 1
        for (int c = 0; c < S_BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(t_lane + c, r);
#pragma unroll
          for (int sl = 0; sl < S - 1; ++sl) {
            const float4* src = reinterpret_cast<const float4*>(slots + sl * Sc::SLICE_ROWS * S_ROW + c);
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 x = src[v];
              r[4 * v] = __float_as_uint(__uint_as_float(r[4 * v]) + x.x);
              r[4 * v + 1] = __float_as_uint(__uint_as_float(r[4 * v + 1]) + x.y);
              r[4 * v + 2] = __float_as_uint(__uint_as_float(r[4 * v + 2]) + x.z);
              r[4 * v + 3] = __float_as_uint(__uint_as_float(r[4 * v + 3]) + x.w);
            }
          }
          const int col = n0 + c;
          if (row_ok && col < p.N) store_row32<MODE>(p, row, col, r);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while another may still push into its receive buffer
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S_BN));
  }
}

// ---------------------------------------------------------------- host side
// 2-D bf16 tensor map: inner dim `inner` (contiguous), outer dim `outer`, row pitch ld elements,
// box {64, box_outer}, 128-byte swizzle, zero fill out of bounds.
bool make_tmap(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Operand map: K-major [rows, K] -> box {64 along K, rows_tile}; MN-major stored [K, rows] ->
// box {64 along MN, 64 along K} (one box per 64-wide MN atom).
bool operand_tmap(CUtensorMap* map, const void* ptr, bool mn_major, uint64_t rows, uint64_t K, uint64_t ld,
                  uint32_t rows_tile) {
  return mn_major ? make_tmap(map, ptr, rows, K, ld, BK) : make_tmap(map, ptr, K, rows, ld, rows_tile);
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int BN, int STAGES, int MODE, bool A_MN, bool B_MN>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  using Cfg = GemmCfg<BN, STAGES, MODE, A_MN, B_MN>;
  auto kern = gemm_tcgen05_kernel<BN, STAGES, MODE, A_MN, B_MN>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM) != cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  return qb_launch_ex(kern, dim3(grid), dim3(THREADS), Cfg::SMEM, st, 1, true, ta, tb, p);
}

template <int MODE, bool A_MN, bool B_MN, int PBN>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  auto kern = gemm_pair_kernel<MODE, A_MN, B_MN, PBN>;
  constexpr int SMEM = PairShape<PBN>::SMEM;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  constexpr int TN = MODE == 4 ? PBN / 2 : PBN;
  const int tiles = ((p.M + 255) / 256) * ((p.N + TN - 1) / TN) * (MODE == 2 && p.ksplit > 1 ? p.ksplit : 1);
  const int pairs = tiles < sm_count() / 2 ? tiles : sm_count() / 2;
  return qb_launch_ex(kern, dim3((unsigned)(2 * pairs)), dim3(THREADS), SMEM, st, 2, true, ta, tb, p);
}

template <int S, int MODE, bool A_MN, bool B_MN>
int launch_split(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  auto kern = gemm_split_kernel<S, MODE, A_MN, B_MN>;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SplitCfg<S>::SMEM) != cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  return qb_launch_ex(kern, dim3((unsigned)(p.tiles_m * p.tiles_n * S)), dim3(THREADS), SplitCfg<S>::SMEM, st, S, true, ta,
                   tb, p);
}

template <int S, bool A_MN, bool B_MN>
int launch_split_mode(int mode, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  if (mode == 0) return launch_split<S, 0, A_MN, B_MN>(ta, tb, p, st);
  if (mode == 1) return launch_split<S, 1, A_MN, B_MN>(ta, tb, p, st);
  return launch_split<S, 2, A_MN, B_MN>(ta, tb, p, st);
}

template <bool A_MN, bool B_MN>
int launch_split_s(int S, int mode, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  return S == 2 ? launch_split_mode<2, A_MN, B_MN>(mode, ta, tb, p, st)
                : launch_split_mode<4, A_MN, B_MN>(mode, ta, tb, p, st);
}

// How many S-CTA clusters of the split kernel are resident at once (0 if none fit): a split
// launch with more tiles than this would run in waves, which the split layout is not meant for.
int split_clusters(int S) {
  static int cached[5] = {-1, -1, -1, -1, -1};
  if (cached[S] >= 0) return cached[S];
  auto kern = S == 2 ? gemm_split_kernel<2, 0, false, false> : gemm_split_kernel<4, 0, false, false>;
  const int smem = S == 2 ? SplitCfg<2>::SMEM : SplitCfg<4>::SMEM;
  int n = 0;
  bool ok = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess;
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(S * 64));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attrs[1];
    attrs[0].id = cudaLaunchAttributeClusterDimension;
    attrs[0].val.clusterDim.x = S;
    attrs[0].val.clusterDim.y = 1;
    attrs[0].val.clusterDim.z = 1;
    cfg.attrs = attrs;
    cfg.numAttrs = 1;
    ok = cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess;
  }
  if (!ok) {
    n = 0;
    (void)cudaGetLastError();  // the failed query's own error: the split layout is just not used
  }
  cached[S] = n;
  return n;
}

template <bool A_MN, bool B_MN, int PBN>
int launch_pair_mode(int mode, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  if (mode == 0) return launch_pair<0, A_MN, B_MN, PBN>(ta, tb, p, st);
  if (mode == 1) return launch_pair<1, A_MN, B_MN, PBN>(ta, tb, p, st);
  return launch_pair<2, A_MN, B_MN, PBN>(ta, tb, p, st);
}

template <bool A_MN, bool B_MN>
int launch_pair_pbn(int pbn, int mode, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p,
                    cudaStream_t st) {
  (void)pbn;  // plan_gemm only picks 256-wide pair tiles
  return launch_pair_mode<A_MN, B_MN, 256>(mode, ta, tb, p, st);
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
int launch_mode(int mode, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  if (mode == 0) return launch<BN, STAGES, 0, A_MN, B_MN>(ta, tb, p, st);
  if (mode == 1) return launch<BN, STAGES, 1, A_MN, B_MN>(ta, tb, p, st);
  return launch<BN, STAGES, 2, A_MN, B_MN>(ta, tb, p, st);
}

template <bool A_MN, bool B_MN>
int launch_layout(int bn, int mode, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams p, cudaStream_t st) {
  if (bn == 256) return launch_mode<256, 4, A_MN, B_MN>(mode, ta, tb, p, st);
  if (bn == 192) return launch_mode<192, 5, A_MN, B_MN>(mode, ta, tb, p, st);
  return launch_mode<128, 6, A_MN, B_MN>(mode, ta, tb, p, st);
}

inline bool al16(const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; }

// The layout of one product.  256x256 tiles on CTA pairs when they fill every SM pair at least
// once; 128 x 256 single-CTA tiles when they cover every SM at least once.  Otherwise every
// candidate is costed by the operand bytes its busiest SM pulls: 128 x {128, 192} single-CTA
// tiles in waves over the SMs, 256 x 256 pair tiles in waves over the SM pairs, or 128 x 128
// tiles split along K over a cluster of 2 or 4 CTAs (one wave, plus the partials' exchange,
// costed as two K blocks).
struct GemmPlan {
  bool pair;
  int bn;     // tile width (N): of the pair's 256-row tile, or of the single CTA's 128-row tile
  int split;  // K split: over the CTAs of a 128 x 128 tile's cluster (single), or over pairs (MODE 2)
};

// pair_split: the K range of a pair tile may be split over several pairs whose partials are added
// to C atomically (MODE 2, C += A.B^T): weight gradients whose tiles leave pairs idle.
GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, bool b_mn, bool pair_split) {
  const int sms = sm_count(), P = sms / 2;
  const int64_t tm = (M + BM - 1) / BM, kblocks = (K + BK - 1) / BK;
  const int64_t pairs = ((M + 255) / 256) * ((N + 255) / 256);
  // 256 x 256 pair tiles, K split S ways: waves of units over the pairs x K blocks per unit
  // (a split must save 10%: its atomic adds to C are not in the cost)
  auto pair_plan = [&](int64_t& cost) {
    int S = 1;
    cost = (pairs + P - 1) / P * kblocks * (int64_t)(128 + 128) * BK * 2;
    const int64_t cost1 = cost;
    for (int s = 2; pair_split && s <= 4; ++s) {
      if (kblocks / s < 32) break;
      const int64_t c = (pairs * s + P - 1) / P * ((kblocks + s - 1) / s) * (int64_t)(128 + 128) * BK * 2;
      if (c < cost && 10 * c < 9 * cost1) { cost = c; S = s; }
    }
    return S;
  };
  if (N >= 256 && M >= 256 && pairs >= P) {
    int64_t c;
    const int S = pair_plan(c);
    return {true, 256, S};
  }
  if (N >= 256 && tm * ((N + 255) / 256) >= sms) return {false, 256, 1};
  const int64_t t128 = tm * ((N + 127) / 128), t192 = tm * ((N + 191) / 192);
  GemmPlan best_plan{false, 128, 1};
  const int64_t kb_bytes = (int64_t)(BM + 128) * BK * 2;
  int64_t best = (t128 + sms - 1) / sms * kblocks * kb_bytes;
  const int64_t c192 = (t192 + sms - 1) / sms * kblocks * (int64_t)(BM + 192) * BK * 2;
  if (N > 128 && c192 < best) { best = c192; best_plan = {false, 192, 1}; }
  (void)b_mn;
  // 256 x 256 tiles on CTA pairs that do not fill every SM pair: each SM pulls (128 + 128) rows per K
  // block for twice a 128 x 128 tile's MMA work, which long-K products need (a 128 x 128 tile's
  // operands alone would ask ~35 TB/s of L2 at the MMA rate).  Long K only (64+ K blocks), ties to
  // single-CTA tiles: the decode step's M = 512, K = 1024 products measured slower on pairs.
  if (M > 128 && N > 128 && kblocks >= 64) {
    int64_t c;
    const int S = pair_plan(c);
    if (c < best) { best = c; best_plan = {true, 256, S}; }
  }
  for (int S = 2; S <= 4; S *= 2) {
    if (kblocks < 2 * S || t128 > split_clusters(S)) continue;
    const int64_t c = (kblocks + S - 1) / S * kb_bytes + 2 * kb_bytes;
    if (c < best) { best = c; best_plan = {false, 128, S}; }
  }
  return best_plan;
}


int gemm_dispatch(const void* A, int64_t lda, bool a_mn, const void* B, int64_t ldb, bool b_mn, void* C,
                  int64_t ldc, int64_t M, int64_t N, int64_t K, int mode, int* err, cudaStream_t st) {
  const int b_static = (mode & QB_GEMM_B_STATIC) ? 1 : 0;
  mode &= ~QB_GEMM_B_STATIC;
  QB_CHECK_ARG(M >= 0 && N >= 0 && K >= 0 && mode >= 0 && mode <= 2);
  if (M == 0 || N == 0) return QB_OK;
  if (K == 0) return QB_ERR_UNSUPPORTED;
  // A and B feed TMA: 16-byte aligned bases and row pitches (a multiple of 8 bf16).
  QB_CHECK_ARG(A && B && C && al16(A) && al16(B) && lda % 8 == 0 && ldb % 8 == 0 && ldc >= N);
  QB_CHECK_ARG(lda >= (a_mn ? M : K) && ldb >= (b_mn ? N : K));
  QB_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31));
  const int64_t elem = mode == 0 ? 2 : 4;
  const int vec_ok = al16(C) && (ldc * elem) % 16 == 0;
  const GemmPlan pl = plan_gemm(M, N, K, b_mn, mode == 2);
  const int64_t tm = (M + BM - 1) / BM;
  const int pbn = pl.pair ? pl.bn : 0, bn = pl.bn, split = pl.pair ? 1 : pl.split;
  CUtensorMap ta, tb;
  if (pbn) {
    if (!operand_tmap(&ta, A, a_mn, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM)) return QB_ERR_INVALID;
    if (!operand_tmap(&tb, B, b_mn, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, (uint32_t)(pbn / 2)))
      return QB_ERR_INVALID;
    GemmParams pp{C, ldc, (int)M, (int)N, (int)K, 0, 0, vec_ok, err};
    pp.ksplit = pl.split;  // > 1 only in MODE 2
    if (!a_mn && !b_mn) return launch_pair_pbn<false, false>(pbn, mode, ta, tb, pp, st);
    if (!a_mn && b_mn) return launch_pair_pbn<false, true>(pbn, mode, ta, tb, pp, st);
    if (a_mn && !b_mn) return launch_pair_pbn<true, false>(pbn, mode, ta, tb, pp, st);
    return launch_pair_pbn<true, true>(pbn, mode, ta, tb, pp, st);
  }
  if (!operand_tmap(&ta, A, a_mn, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM)) return QB_ERR_INVALID;
  if (!operand_tmap(&tb, B, b_mn, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, (uint32_t)bn)) return QB_ERR_INVALID;
  GemmParams p{C, ldc, (int)M, (int)N, (int)K, (int)tm, (int)((N + bn - 1) / bn), vec_ok, err};
  p.b_static = b_static;
  if (split > 1) {
    if (!a_mn && !b_mn) return launch_split_s<false, false>(split, mode, ta, tb, p, st);
    if (!a_mn && b_mn) return launch_split_s<false, true>(split, mode, ta, tb, p, st);
    if (a_mn && !b_mn) return launch_split_s<true, false>(split, mode, ta, tb, p, st);
    return launch_split_s<true, true>(split, mode, ta, tb, p, st);
  }
  if (!a_mn && !b_mn) return launch_layout<false, false>(bn, mode, ta, tb, p, st);
  if (!a_mn && b_mn) return launch_layout<false, true>(bn, mode, ta, tb, p, st);
  if (a_mn && !b_mn) return launch_layout<true, false>(bn, mode, ta, tb, p, st);
  return launch_layout<true, true>(bn, mode, ta, tb, p, st);
}

// ---------------------------------------------------------------- gate_up projection -> SwiGLU
// H[M, I] = silu(A W_gate^T) * (A W_up^T) with W = [W_gate; W_up] the [2I, K] gate_up weight, in one
// GEMM whose N tiles pair each gate column block with the same up block (MODE 4); GU (nullable)
// also receives the bf16 gate_up product for a backward.  256-row tiles on CTA pairs (128 gate +
// 128 up columns) when they fill every SM pair, else single-CTA tiles of 96 + 96 or 128 + 128
// columns by the busiest SM's operand bytes.
int gemm_swiglu(const void* A, int64_t lda, const void* W, int64_t ldw, void* H, int64_t ldh, void* GU, int64_t ldgu,
                int64_t M, int64_t I, int64_t K, int flags, int* err, cudaStream_t st) {
  QB_CHECK_ARG(M >= 0 && I > 0 && K > 0 && (flags & ~QB_GEMM_B_STATIC) == 0);
  if (M == 0) return QB_OK;
  QB_CHECK_ARG(A && W && H && al16(A) && al16(W) && lda % 8 == 0 && ldw % 8 == 0 && lda >= K && ldw >= K);
  QB_CHECK_ARG(ldh >= I && (GU == nullptr || ldgu >= 2 * I));
  QB_CHECK_ARG(M < (1ll << 31) && I < (1ll << 30) && K < (1ll << 31));
  const int vec_ok = al16(H) && ldh % 8 == 0 && (GU == nullptr || (al16(GU) && ldgu % 8 == 0 && I % 8 == 0));
  const int sms = sm_count();
  const int64_t tm = (M + BM - 1) / BM, kblocks = (K + BK - 1) / BK;
  const bool pair = M >= 256 && ((M + 255) / 256) * ((I + 127) / 128) >= sms / 2;
  int bn = 256;
  if (!pair) {
    int64_t best = -1;
    for (int cand = 192; cand <= 256; cand += 64) {
      const int64_t tiles = tm * ((I + cand / 2 - 1) / (cand / 2));
      const int64_t c = (tiles + sms - 1) / sms * kblocks * (int64_t)(BM + cand) * BK * 2;
      if (best < 0 || c < best) { best = c; bn = cand; }
    }
  }
  CUtensorMap ta, tb;
  if (!operand_tmap(&ta, A, false, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM)) return QB_ERR_INVALID;
  if (!operand_tmap(&tb, W, false, (uint64_t)(2 * I), (uint64_t)K, (uint64_t)ldw, (uint32_t)(pair ? 128 : bn / 2)))
    return QB_ERR_INVALID;
  GemmParams p{H, ldh, (int)M, (int)I, (int)K, (int)tm, (int)((I + bn / 2 - 1) / (bn / 2)), vec_ok, err};
  p.b_static = (flags & QB_GEMM_B_STATIC) ? 1 : 0;
  p.C2 = GU;
  p.ld2 = ldgu;
  p.half = (int)I;
  if (pair) return launch_pair<4, false, false, 256>(ta, tb, p, st);
  return bn == 256 ? launch<256, 4, 4, false, false>(ta, tb, p, st) : launch<192, 5, 4, false, false>(ta, tb, p, st);
}

// ---------------------------------------------------------------- qkv projection -> QK-norm + RoPE
// The qkv projection (N = (hq + 2 hkv) * 128) with QK-norm, RoPE and the paged K/V store in its
// epilogue (MODE 5): whole heads per tile, 256-row tiles on CTA pairs when they fill every SM pair,
// else single-CTA tiles of one or two heads by the busiest SM's operand bytes.
int gemm_qk_norm_rope(const void* A, int64_t lda, const void* W, int64_t ldw, int64_t M, int hq, int hkv, int64_t K,
                      const GemmParams::QkEpilogue& qk, void* out, int64_t ld_out, void* raw, int64_t ld_raw,
                      int flags, int* err, cudaStream_t st) {
  QB_CHECK_ARG(M >= 0 && hq > 0 && hkv > 0 && K > 0 && (flags & ~QB_GEMM_B_STATIC) == 0);
  if (M == 0) return QB_OK;
  const int64_t N = (int64_t)(hq + 2 * hkv) * 128;
  QB_CHECK_ARG(A && W && al16(A) && al16(W) && lda % 8 == 0 && ldw % 8 == 0 && lda >= K && ldw >= K);
  QB_CHECK_ARG(qk.positions && qk.cos_sin && qk.max_pos > 0 && qk.qw && qk.kw);
  QB_CHECK_ARG((reinterpret_cast<uintptr_t>(qk.cos_sin) & 15) == 0 && (reinterpret_cast<uintptr_t>(qk.qw) & 7) == 0 &&
               (reinterpret_cast<uintptr_t>(qk.kw) & 7) == 0);
  QB_CHECK_ARG(out == nullptr || (al16(out) && ld_out >= N && ld_out % 8 == 0));
  QB_CHECK_ARG(raw == nullptr || (al16(raw) && ld_raw >= N && ld_raw % 8 == 0));
  QB_CHECK_ARG(qk.q_out == nullptr || al16(qk.q_out));
  QB_CHECK_ARG((qk.k_cache == nullptr) == (qk.v_cache == nullptr));
  QB_CHECK_ARG(qk.k_cache == nullptr || (al16(qk.k_cache) && al16(qk.v_cache) && qk.slots && qk.num_slots > 0));
  QB_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31));
  const int sms = sm_count();
  const int64_t tm = (M + BM - 1) / BM, kblocks = (K + BK - 1) / BK;
  const bool pair = M >= 256 && ((M + 255) / 256) * ((N + 255) / 256) >= sms / 2;
  int bn = 256;
  if (!pair) {
    int64_t best = -1;
    for (int cand = 128; cand <= 256; cand += 128) {
      const int64_t tiles = tm * ((N + cand - 1) / cand);
      const int64_t c = (tiles + sms - 1) / sms * kblocks * (int64_t)(BM + cand) * BK * 2;
      if (best < 0 || c < best) { best = c; bn = cand; }
    }
  }
  CUtensorMap ta, tb;
  if (!operand_tmap(&ta, A, false, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BM)) return QB_ERR_INVALID;
  if (!operand_tmap(&tb, W, false, (uint64_t)N, (uint64_t)K, (uint64_t)ldw, (uint32_t)(pair ? 128 : bn)))
    return QB_ERR_INVALID;
  GemmParams p{out, ld_out, (int)M, (int)N, (int)K, (int)tm, (int)((N + bn - 1) / bn), 1, err};
  p.b_static = (flags & QB_GEMM_B_STATIC) ? 1 : 0;
  p.C2 = raw;
  p.ld2 = ld_raw;
  p.qk = qk;
  p.qk.hq = hq;
  p.qk.hkv = hkv;
  if (pair) return launch_pair<5, false, false, 256>(ta, tb, p, st);
  return bn == 256 ? launch<256, 4, 5, false, false>(ta, tb, p, st) : launch<128, 6, 5, false, false>(ta, tb, p, st);
}

// ---------------------------------------------------------------- lm_head -> log-softmax -> gather
// The per-tile (max, sum of exp) pairs of a row are merged into the row's log-sum-exp, and the
// target's log-prob is its fp32 logit minus that.  One warp per row.
__global__ void __launch_bounds__(128)
lse_combine_kernel(const float2* __restrict__ part, int n_part, const float* __restrict__ tgt_logit,
                   const int64_t* __restrict__ targets, const int64_t* __restrict__ dest, int64_t n, int64_t V,
                   float* __restrict__ logp, float* __restrict__ lse, int* err) {
  qb_pdl_trigger();
  qb_pdl_wait();
  constexpr float LN2 = 0.6931471805599453f;
  const int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n) return;
  const float2* pr = part + row * n_part;
  float m = -INFINITY;
  for (int i = lane; i < n_part; i += 32) m = fmaxf(m, pr[i].x);
  m = warp_max(m);
  float s = 0.f;
  for (int i = lane; i < n_part; i += 32) {
    const float2 v = pr[i];
    s += v.y * exp2f(v.x - m);
  }
  s = warp_sum(s);
  if (lane == 0) {
    const float l = (m + log2f(s)) * LN2;
    if (lse) lse[row] = l;
    const int64_t d = dest ? dest[row] : row;
    if (d >= 0) {
      const int64_t t = targets[row];
      if (t < 0 || t >= V) {
        qb_set_err(err, QB_DEVERR_TOKEN);
        logp[d] = 0.f;
      } else {
        logp[d] = tgt_logit[row] - l;
      }
    }
  }
}

inline int64_t lse_parts_bound(int64_t V) { return (V + 127) / 128; }

int lm_head_logprob(const void* h, int64_t ldh, const void* W, int64_t ldw, int64_t n, int64_t V, int64_t K,
                    const int64_t* targets, const int64_t* dest, float* logp, float* lse, void* logits,
                    int64_t ld_logits, void* workspace, int* err, cudaStream_t st) {
  QB_CHECK_ARG(n >= 0 && V > 0 && K > 0);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(h && W && targets && logp && workspace && al16(h) && al16(W) && ldh % 8 == 0 && ldw % 8 == 0);
  QB_CHECK_ARG(ldh >= K && ldw >= K && (!logits || ld_logits >= V));
  QB_CHECK_ARG(n < (1ll << 31) && V < (1ll << 31) && K < (1ll << 31));
  QB_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 15) == 0);
  const int sms = sm_count();
  const int64_t tm = (n + BM - 1) / BM;
  const bool pair = V >= 256 && n >= 256 && ((n + 255) / 256) * ((V + 255) / 256) >= sms / 2;
  const int bn = pair || V >= 256 ? 256 : 128;
  const int n_part = (int)((V + bn - 1) / bn);
  float2* part = reinterpret_cast<float2*>(workspace);
  float* tgt = reinterpret_cast<float*>(part + n * lse_parts_bound(V));
  const int vec_ok = logits && al16(logits) && (ld_logits * 2) % 16 == 0;
  GemmParams p{logits, ld_logits, (int)n, (int)V, (int)K, (int)tm, n_part, vec_ok, err, targets, part, tgt, n_part};
  CUtensorMap ta, tb;
  if (!operand_tmap(&ta, h, false, (uint64_t)n, (uint64_t)K, (uint64_t)ldh, BM)) return QB_ERR_INVALID;
  if (!operand_tmap(&tb, W, false, (uint64_t)V, (uint64_t)K, (uint64_t)ldw, pair ? 128 : (uint32_t)bn))
    return QB_ERR_INVALID;
  int status = pair ? launch_pair<3, false, false, 256>(ta, tb, p, st)
                    : (bn == 256 ? launch<256, 4, 3, false, false>(ta, tb, p, st)
                                 : launch<128, 6, 3, false, false>(ta, tb, p, st));
  if (status != QB_OK) return status;
  return qb_launch(lse_combine_kernel, dim3((unsigned)((n + 3) / 4)), dim3(128), 0, st, 1, part, n_part, tgt, targets,
                   dest, n, V, logp, lse, err);
}

}  // namespace

extern "C" int qb_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                            int64_t M, int64_t N, int64_t K, int mode, int* err, qb_stream_t stream) {
  return gemm_dispatch(A, lda, false, B, ldb, false, C, ldc, M, N, K, mode, err, (cudaStream_t)stream);
}

extern "C" int qb_gemm_bf16_ex(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb,
                               int b_mn_major, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int mode,
                               int* err, qb_stream_t stream) {
  return gemm_dispatch(A, lda, a_mn_major != 0, B, ldb, b_mn_major != 0, C, ldc, M, N, K, mode, err,
                       (cudaStream_t)stream);
}

extern "C" int qb_lm_head_logprob(const void* h, int64_t ldh, const void* W, int64_t ldw, int64_t n, int64_t V,
                                  int64_t K, const int64_t* targets, const int64_t* dest, float* logp, float* lse,
                                  void* logits, int64_t ld_logits, void* workspace, int* err, qb_stream_t stream) {
  return lm_head_logprob(h, ldh, W, ldw, n, V, K, targets, dest, logp, lse, logits, ld_logits, workspace, err,
                         (cudaStream_t)stream);
}

extern "C" int qb_gemm_swiglu(const void* A, int64_t lda, const void* W, int64_t ldw, void* H, int64_t ldh, void* GU,
                              int64_t ldgu, int64_t M, int64_t I, int64_t K, int flags, int* err,
                              qb_stream_t stream) {
  return gemm_swiglu(A, lda, W, ldw, H, ldh, GU, ldgu, M, I, K, flags, err, (cudaStream_t)stream);
}

extern "C" int qb_gemm_qk_norm_rope(const void* A, int64_t lda, const void* W, int64_t ldw, int64_t M, int hq, int hkv,
                                    int64_t K, const int64_t* positions, const float* cos_sin, int64_t max_pos,
                                    const void* q_norm_w, const void* k_norm_w, float eps, void* out, int64_t ld_out,
                                    void* raw, int64_t ld_raw, void* q_out, void* k_cache, void* v_cache,
                                    const int32_t* slot_mapping, int64_t num_slots, float* q_rstd, float* k_rstd,
                                    int flags, int* err, qb_stream_t stream) {
  GemmParams::QkEpilogue qk{positions, cos_sin, max_pos, (const bf16*)q_norm_w, (const bf16*)k_norm_w, eps, hq, hkv,
                            (bf16*)q_out, (bf16*)k_cache, (bf16*)v_cache, slot_mapping, num_slots, q_rstd, k_rstd};
  return gemm_qk_norm_rope(A, lda, W, ldw, M, hq, hkv, K, qk, out, ld_out, raw, ld_raw, flags, err,
                           (cudaStream_t)stream);
}

extern "C" int qb_gemm_plan(int64_t M, int64_t N, int64_t K, int b_mn_major, int mode, int* pair, int* tile_n,
                            int* split) {
  QB_CHECK_ARG(M > 0 && N > 0 && K > 0 && mode >= 0 && mode <= 2 && pair && tile_n && split);
  const GemmPlan pl = plan_gemm(M, N, K, b_mn_major != 0, mode == 2);
  *pair = pl.pair ? 1 : 0;
  *tile_n = pl.bn;
  *split = pl.split;
  return QB_OK;
}

extern "C" size_t qb_lm_head_logprob_workspace_bytes(int64_t n, int64_t V) {
  if (n <= 0 || V <= 0) return 16;
  const size_t bytes = (size_t)n * (size_t)lse_parts_bound(V) * sizeof(float2) + (size_t)n * sizeof(float);
  return (bytes + 255) / 256 * 256;
}
