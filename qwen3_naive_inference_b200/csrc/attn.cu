// Causal GQA attention for the GRPO step: paged decode (one query token per
// sequence), paged/dense varlen prefill, and the dense varlen backward used by
// the log-prob recompute.
//
// Tensor-core work runs on warp-level mma.sync m16n8k16 (bf16 in, fp32
// accumulate); K/V tiles are staged in shared memory with cp.async 16-byte
// copies in an XOR-swizzled 256-byte-row layout (swz128), double or triple
// buffered.  Page ids come from block_tables and are bounds-checked: a bad id
// zero-fills the tile and raises QB_DEVERR_PAGE instead of reading out of range.
//
// Layout of the paged KV cache (qwen3_naive.py:1059-1066): per layer
// [num_blocks, 256, hkv, 128] bf16, so token j of a page for kv head h is the
// 256-byte row at ((page*256 + j)*hkv + h)*128.
#include <algorithm>

#include "common.cuh"

namespace {

constexpr int D = 128;           // head dim
constexpr int ROWB = D * 2;      // bytes per K/V row
constexpr int PAGE = 256;        // tokens per page
constexpr float LOG2E = 1.4426950408889634f;
constexpr float NEG_INF = -INFINITY;

// ============================================================================
// Paged decode attention
// ============================================================================
// CTA = (split, kv head, sequence).  Four warps; a stage holds 64 tokens of K
// and V for one kv head (16 KB each).  Each warp computes S^T = K Q^T for its
// 16 tokens with the tokens in the M dimension (the two query heads of the kv
// group fill 2 of the 8 N columns), then O^T += V^T P^T, so K and V are read
// exactly once per kv head.
constexpr int DEC_TOK = 64;
constexpr int DEC_STAGES = 3;
constexpr int DEC_WARPS = 4;
constexpr int DEC_STAGE_BYTES = 2 * DEC_TOK * ROWB;  // K + V
constexpr int DEC_SMEM = DEC_STAGES * DEC_STAGE_BYTES;
// Partial-result row in the split-K workspace: 128 fp32 outputs, the log2-domain
// LSE at [128], padded to 132 floats so every row starts on a 16-byte boundary.
constexpr int WS_ROW = D + 4;

struct DecodeParams {
  const bf16* q;
  const bf16* kc;
  const bf16* vc;
  int64_t num_blocks;
  const int32_t* bt;
  int64_t bt_stride;
  const int32_t* seqlens;
  int seqlen_add;
  int hq, hkv;
  float scale_log2;
  int split_tokens, max_splits;
  float* ws;
  bf16* out;
  int* err;
  // Split-K partial layout: sequence b, slot s, head h at ws[((b*n_slots + s)*hq + h)*WS_ROW].
  // This kernel's split i goes to slot slot_off + i.  kv_start (nullable): the first key
  // read for each sequence (a multiple of 64; the keys before it belong to a shared
  // prefix handled elsewhere).
  int n_slots, slot_off;
  const int32_t* kv_start;
};

// Marks the partial of (b, slot, h) empty (log2-domain LSE = -inf) so the merge ignores it.
QB_DEVICE void write_empty_partial(const DecodeParams& p, int b, int slot, int h) {
  p.ws[(((int64_t)b * p.n_slots + slot) * p.hq + h) * WS_ROW + D] = NEG_INF;
}

// Loads one 64-token stage of K and V for kv head kvh of sequence b (keys [tok0, tok0 + 64), rows
// at or past tok_end zero-filled) into a stage buffer with 16-byte cp.async; a bad page id reads
// nothing and raises QB_DEVERR_PAGE.
QB_DEVICE void own_load_stage(const DecodeParams& p, uint32_t kbase, int b, int kvh, int tok0, int tok_end, int tid) {
  const uint32_t vbase = kbase + DEC_TOK * ROWB;
  const int32_t* btrow = p.bt + (int64_t)b * p.bt_stride;
  const bool col_ok = tok0 / PAGE < p.bt_stride;  // page-table row is bt_stride entries wide
  int page = col_ok ? btrow[tok0 / PAGE] : -1;
  const bool page_ok = page >= 0 && page < p.num_blocks;
  if (!page_ok) {
    if (tid == 0) qb_set_err(p.err, QB_DEVERR_PAGE);
    page = 0;
  }
  const int64_t row0 = ((int64_t)page * PAGE + (tok0 % PAGE)) * p.hkv + kvh;
  // 64 rows x 16 chunks for K and for V: 2048 copies / 128 threads = 16 each.
#pragma unroll
  for (int i = 0; i < (DEC_TOK * 16) / (DEC_WARPS * 32); ++i) {
    const int idx = tid + i * DEC_WARPS * 32;
    const int r = idx >> 4, c = idx & 15;
    const bool ok = page_ok && (tok0 + r < tok_end);
    const int64_t goff = (row0 + (int64_t)r * p.hkv) * D + c * 8;
    cp_async_16(kbase + swz128(r, c), ok ? (const void*)(p.kc + goff) : (const void*)p.kc, ok ? 16 : 0);
    cp_async_16(vbase + swz128(r, c), ok ? (const void*)(p.vc + goff) : (const void*)p.vc, ok ? 16 : 0);
  }
}

// One warp's share of a 64-token stage of an own-key tile: its 16 tokens (rows wrow.. of the
// stage, keys tok_base + wrow + ...) against the kv head's two query heads.  S^T = K Q^T with the
// tokens in the M dimension (the two heads fill 2 of the 8 N columns), online softmax, then
// O^T += V^T P^T.
QB_DEVICE void own_stage(const DecodeParams& p, uint32_t kbase, int wrow, int tok_base, int tok_end,
                         const uint32_t (&qb)[8][2], float (&m_run)[2], float (&l_run)[2], float (&o)[8][4],
                         int lane) {
  const int g = lane >> 2, t4 = lane & 3;
  const uint32_t vbase = kbase + DEC_TOK * ROWB;
  // S^T[16 tok x 8] = K[16 x 128] * Q^T[128 x 8]
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    uint32_t a[4];
    ldmatrix_x4(kbase + swz128(wrow + (lane & 15), kk * 2 + (lane >> 4)), a[0], a[1], a[2], a[3]);
    mma_bf16_16816(sc, a, qb[kk][0], qb[kk][1]);
  }
  const int tokA = tok_base + wrow + g;  // rows g and g+8
  float x[4];
  x[0] = (t4 == 0 && tokA < tok_end) ? sc[0] * p.scale_log2 : NEG_INF;
  x[1] = (t4 == 0 && tokA < tok_end) ? sc[1] * p.scale_log2 : NEG_INF;
  x[2] = (t4 == 0 && tokA + 8 < tok_end) ? sc[2] * p.scale_log2 : NEG_INF;
  x[3] = (t4 == 0 && tokA + 8 < tok_end) ? sc[3] * p.scale_log2 : NEG_INF;
  float mloc[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) mloc[h] = fmaxf(mloc[h], __shfl_xor_sync(0xffffffffu, mloc[h], off));
    mloc[h] = __shfl_sync(0xffffffffu, mloc[h], 0);
  }
  float alpha[2], mnew[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    mnew[h] = fmaxf(m_run[h], mloc[h]);
    alpha[h] = (mnew[h] == NEG_INF) ? 1.f : exp2f(m_run[h] - mnew[h]);
  }
  float pv[4];
  pv[0] = (mnew[0] == NEG_INF) ? 0.f : exp2f(x[0] - mnew[0]);
  pv[1] = (mnew[1] == NEG_INF) ? 0.f : exp2f(x[1] - mnew[1]);
  pv[2] = (mnew[0] == NEG_INF) ? 0.f : exp2f(x[2] - mnew[0]);
  pv[3] = (mnew[1] == NEG_INF) ? 0.f : exp2f(x[3] - mnew[1]);
  float lsum[2] = {pv[0] + pv[2], pv[1] + pv[3]};
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) lsum[h] += __shfl_xor_sync(0xffffffffu, lsum[h], off);
    lsum[h] = __shfl_sync(0xffffffffu, lsum[h], 0);
    l_run[h] = l_run[h] * alpha[h] + lsum[h];
    m_run[h] = mnew[h];
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    o[mt][0] *= alpha[0];
    o[mt][1] *= alpha[1];
    o[mt][2] *= alpha[0];
    o[mt][3] *= alpha[1];
  }
  // P^T as the B operand: lane (g, t4) needs P[tok 2t4, 2t4+1, 2t4+8, 2t4+9][head g].
  const int srcA = 8 * t4, srcB = 8 * t4 + 4;
  float a0 = __shfl_sync(0xffffffffu, pv[0], srcA), a1 = __shfl_sync(0xffffffffu, pv[1], srcA);
  float a2 = __shfl_sync(0xffffffffu, pv[2], srcA), a3 = __shfl_sync(0xffffffffu, pv[3], srcA);
  float c0 = __shfl_sync(0xffffffffu, pv[0], srcB), c1 = __shfl_sync(0xffffffffu, pv[1], srcB);
  float c2 = __shfl_sync(0xffffffffu, pv[2], srcB), c3 = __shfl_sync(0xffffffffu, pv[3], srcB);
  uint32_t pb0 = 0u, pb1 = 0u;
  if (g == 0) {
    pb0 = pack_bf16x2(a0, c0);
    pb1 = pack_bf16x2(a2, c2);
  } else if (g == 1) {
    pb0 = pack_bf16x2(a1, c1);
    pb1 = pack_bf16x2(a3, c3);
  }
  // O^T[128 x 8] += V^T[128 x 16 tok] * P^T[16 tok x 8]
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    uint32_t a[4];
    ldmatrix_x4_trans(vbase + swz128(wrow + (lane & 7) + ((lane >> 4) << 3), mt * 2 + ((lane >> 3) & 1)), a[0],
                      a[1], a[2], a[3]);
    mma_bf16_16816(o[mt], a, pb0, pb1);
  }
}

// Merges the four warps' (m, l, O) of an own-key tile through `scratch` (DEC_WARPS * 2 * (D + 2)
// floats) and writes the result of sequence b, heads 2*kvh and 2*kvh + 1: the output itself when
// max_splits == 1, else the split-K partial of slot slot_off + split.  Contains __syncthreads.
QB_DEVICE void own_merge(const DecodeParams& p, float* scratch, int b, int kvh, int split, const float (&m_run)[2],
                         const float (&l_run)[2], const float (&o)[8][4], int tid) {
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
  float* so = scratch;
  float* sm = so + DEC_WARPS * 2 * D;
  float* sl = sm + DEC_WARPS * 2;
  if (t4 == 0) {
#pragma unroll
    for (int mt = 0; mt < 8; ++mt) {
      so[(warp * 2 + 0) * D + mt * 16 + g] = o[mt][0];
      so[(warp * 2 + 1) * D + mt * 16 + g] = o[mt][1];
      so[(warp * 2 + 0) * D + mt * 16 + g + 8] = o[mt][2];
      so[(warp * 2 + 1) * D + mt * 16 + g + 8] = o[mt][3];
    }
  }
  if (lane == 0) {
    sm[warp * 2 + 0] = m_run[0];
    sm[warp * 2 + 1] = m_run[1];
    sl[warp * 2 + 0] = l_run[0];
    sl[warp * 2 + 1] = l_run[1];
  }
  __syncthreads();
  const int h = tid >> 6;         // 0..1
  const int d0 = (tid & 63) * 2;  // 2 dims per thread
  float M = NEG_INF;
#pragma unroll
  for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, sm[w * 2 + h]);
  float L = 0.f, acc0 = 0.f, acc1 = 0.f;
#pragma unroll
  for (int w = 0; w < DEC_WARPS; ++w) {
    const float mw = sm[w * 2 + h];
    const float f = (mw == NEG_INF) ? 0.f : exp2f(mw - M);
    L += sl[w * 2 + h] * f;
    acc0 += so[(w * 2 + h) * D + d0] * f;
    acc1 += so[(w * 2 + h) * D + d0 + 1] * f;
  }
  const float inv = (L > 0.f) ? 1.f / L : 0.f;
  if (p.max_splits == 1) {
    bf16* orow = p.out + ((int64_t)b * p.hq + kvh * 2 + h) * D + d0;
    *reinterpret_cast<uint32_t*>(orow) = pack_bf16x2(acc0 * inv, acc1 * inv);
  } else {
    float* wrow = p.ws + (((int64_t)b * p.n_slots + p.slot_off + split) * p.hq + kvh * 2 + h) * WS_ROW;
    wrow[d0] = acc0 * inv;
    wrow[d0 + 1] = acc1 * inv;
    if (d0 == 0) wrow[D] = (L > 0.f) ? M + log2f(L) : NEG_INF;  // log2-domain LSE
  }
}

// Key range of own-key item (split, sequence b): [kv_start[b] + split*split_tokens, +split_tokens)
// clipped to the sequence length; false (and nothing to read) when it is empty or misaligned (a
// 64-token stage must not straddle a page: the first key of a split is 64-aligned; SHAPE raised).
QB_DEVICE bool own_range(const DecodeParams& p, int split, int b, int& tok_begin, int& tok_end, int tid) {
  const int len = p.seqlens[b] + p.seqlen_add;
  tok_begin = (p.kv_start ? p.kv_start[b] : 0) + split * p.split_tokens;
  const bool misaligned = (tok_begin & (DEC_TOK - 1)) != 0 || tok_begin < 0;
  if (misaligned && tid == 0) qb_set_err(p.err, QB_DEVERR_SHAPE);
  tok_end = min(len, tok_begin + p.split_tokens);
  return !misaligned && tok_begin < len;
}

// Result of an item with no keys: the empty partial (log2-domain LSE = -inf) of both heads, or
// zero output rows when there are no split-K slots.
QB_DEVICE void own_empty(const DecodeParams& p, int b, int kvh, int split, int tid) {
  if (p.max_splits > 1) {
    if (tid < 2) write_empty_partial(p, b, p.slot_off + split, kvh * 2 + tid);
  } else {
    for (int i = tid; i < D; i += DEC_WARPS * 32)
      reinterpret_cast<uint32_t*>(p.out + ((int64_t)b * p.hq + kvh * 2) * D)[i] = 0u;
  }
}

// One (split, kv head, sequence) work item of the per-sequence decode: keys
// [kv_start[b] + split*split_tokens, +split_tokens) of sequence b, through STAGES stage buffers.
template <int STAGES>
QB_DEVICE void decode_own_tile(const DecodeParams& p, uint8_t* smem, int split, int kvh, int b) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  int tok_begin, tok_end;
  if (!own_range(p, split, b, tok_begin, tok_end, tid)) {
    own_empty(p, b, kvh, split, tid);
    return;
  }
  const int n_stages = (tok_end - tok_begin + DEC_TOK - 1) / DEC_TOK;
  const int h0 = kvh * 2;

  // Q^T fragments: b0 = Q[h0+g][kk*16 + 2t4, +1], b1 = Q[h0+g][kk*16 + 2t4 + 8, +9].
  uint32_t qb[8][2];
  {
    const bool valid = g < 2;
    const bf16* qrow = p.q + ((int64_t)b * p.hq + h0 + (valid ? g : 0)) * D;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qb[kk][0] = valid ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4) : 0u;
      qb[kk][1] = valid ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * t4 + 8) : 0u;
    }
  }
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < n_stages)
      own_load_stage(p, smem_u32(smem + s * DEC_STAGE_BYTES), b, kvh, tok_begin + s * DEC_TOK, tok_end, tid);
    cp_async_commit();
  }
  float m_run[2] = {NEG_INF, NEG_INF}, l_run[2] = {0.f, 0.f};
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int s = 0; s < n_stages; ++s) {
    const int sn = s + STAGES - 1;
    if (sn < n_stages)
      own_load_stage(p, smem_u32(smem + (sn % STAGES) * DEC_STAGE_BYTES), b, kvh, tok_begin + sn * DEC_TOK,
                     tok_end, tid);
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncthreads();
    own_stage(p, smem_u32(smem + (s % STAGES) * DEC_STAGE_BYTES), warp * 16, tok_begin + s * DEC_TOK, tok_end,
              qb, m_run, l_run, o, lane);
    __syncthreads();
  }
  cp_async_wait<0>();
  __syncthreads();
  own_merge(p, reinterpret_cast<float*>(smem), b, kvh, split, m_run, l_run, o, tid);
}

__global__ void __launch_bounds__(DEC_WARPS * 32)
paged_decode_kernel(DecodeParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  decode_own_tile<DEC_STAGES>(p, smem, blockIdx.x, blockIdx.y, blockIdx.z);
}

// One warp per (sequence, q head): weights w_s = 2^(lse_s - max lse).  Every lane reads the LSE of
// slots lane, lane + 32, ... at once (one round trip instead of one per slot), then the slots'
// outputs are accumulated four slots per step so their loads overlap.  Empty slots (LSE = -inf)
// were never written: their outputs are not read.
__global__ void paged_decode_combine_kernel(DecodeParams p, int batch) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= batch * p.hq) return;
  const int lane = threadIdx.x & 31;
  const int b = item / p.hq, h = item % p.hq;
  const int ns = p.n_slots;
  const float* base = p.ws + ((int64_t)b * p.n_slots * p.hq + h) * WS_ROW;
  const int64_t sstride = (int64_t)p.hq * WS_ROW;
  float M = NEG_INF;
  for (int s = lane; s < ns; s += 32) M = fmaxf(M, base[s * sstride + D]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, W = 0.f;
#pragma unroll 4
  for (int s = 0; s < ns; ++s) {
    const float ls = base[s * sstride + D];
    const bool live = ls != NEG_INF;
    const float w = live ? exp2f(ls - M) : 0.f;
    const float4 v = live ? *reinterpret_cast<const float4*>(base + s * sstride + lane * 4)
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    W += w;
    acc[0] += w * v.x; acc[1] += w * v.y; acc[2] += w * v.z; acc[3] += w * v.w;
  }
  const float inv = (W > 0.f) ? 1.f / W : 0.f;
  bf16* orow = p.out + ((int64_t)b * p.hq + h) * D + lane * 4;
  uint2 r;
  r.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  r.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  *reinterpret_cast<uint2*>(orow) = r;
}

// ============================================================================
// Shared-prefix decode attention (GRPO groups)
// ============================================================================
// The G <= 8 completions of one prompt share the K/V pages of that prompt (the reference keeps
// a copy per completion).  The grouped decode runs two kinds of CTA in one launch, then the
// split-K combine:
//   shared CTA (split, kv head, group): keys [split*S, min(shared_len, (split+1)*S)) in the
//     pages of the group's first member, read once for the 2*G query heads of the kv head,
//     which form the 16 rows of one M=16 MMA tile (row r: member r/2, head h0 + r%2);
//   own CTA (split, kv head, sequence): decode_own_tile over keys [kv_start + split*S, ...).
// Both stage 64 tokens of K and V per step with cp.async (two buffers), warp w on tokens
// [16w, 16w+16), and write one split-K partial per (sequence, head): shared splits to slots
// [0, shared_splits), own splits after them.  paged_decode_combine_kernel merges the slots.
constexpr int GMAX = 8;  // members per group at most (2 * GMAX = 16 query rows, one MMA M tile)

struct GroupParams {
  const int32_t* members;     // [n_groups, GMAX] sequence indices, -1 padded
  const int32_t* shared_len;  // [n_groups] keys shared by the group
  int batch;
  int shared_splits, own_splits;
  int n_shared_ctas;          // shared_splits * hkv * n_groups; the own CTAs follow
};

template <int STAGES>
QB_DEVICE void decode_shared_tile(const DecodeParams& p, const GroupParams& gp, uint8_t* smem, int split, int kvh,
                                  int grp) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int h0 = kvh * 2;
  int mem = -1;  // lanes 0..GMAX-1: member `lane` of the group (-1 when absent)
  if (lane < GMAX) {
    mem = gp.members[grp * GMAX + lane];
    if (mem >= gp.batch) {
      qb_set_err(p.err, QB_DEVERR_SHAPE);
      mem = -1;
    }
    if (mem < 0) mem = -1;
  }
  const int leader = __shfl_sync(0xffffffffu, mem, 0);
  const int tok_begin = split * p.split_tokens;
  const int tok_end = leader < 0 ? 0 : min(gp.shared_len[grp], tok_begin + p.split_tokens);
  if (tok_begin >= tok_end) {  // no shared keys in this split: empty partials
    const int m = __shfl_sync(0xffffffffu, mem, (lane >> 1) & (GMAX - 1));
    if (tid < 2 * GMAX && m >= 0) write_empty_partial(p, m, split, h0 + (tid & 1));
    return;
  }
  const int n_stages = (tok_end - tok_begin + DEC_TOK - 1) / DEC_TOK;

  // Q as the A operand, rows g (member g/2) and g + 8 (member 4 + g/2), head h0 + g%2
  uint32_t qa[8][4];
  {
    const int m0 = __shfl_sync(0xffffffffu, mem, g >> 1), m1 = __shfl_sync(0xffffffffu, mem, 4 + (g >> 1));
    const bf16* q0 = p.q + ((int64_t)(m0 < 0 ? 0 : m0) * p.hq + h0 + (g & 1)) * D;
    const bf16* q1 = p.q + ((int64_t)(m1 < 0 ? 0 : m1) * p.hq + h0 + (g & 1)) * D;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int c = kk * 16 + 2 * t4;
      qa[kk][0] = m0 >= 0 ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
      qa[kk][1] = m1 >= 0 ? *reinterpret_cast<const uint32_t*>(q1 + c) : 0u;
      qa[kk][2] = m0 >= 0 ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
      qa[kk][3] = m1 >= 0 ? *reinterpret_cast<const uint32_t*>(q1 + c + 8) : 0u;
    }
  }

  const int32_t* btrow = p.bt + (int64_t)leader * p.bt_stride;
  auto load_stage = [&](int s) {
    const int buf = s % STAGES;
    const uint32_t kbase = smem_u32(smem + buf * DEC_STAGE_BYTES);
    const uint32_t vbase = kbase + DEC_TOK * ROWB;
    const int tok0 = tok_begin + s * DEC_TOK;
    const bool col_ok = tok0 / PAGE < p.bt_stride;
    int page = col_ok ? btrow[tok0 / PAGE] : -1;
    const bool page_ok = page >= 0 && page < p.num_blocks;
    if (!page_ok) {
      if (tid == 0) qb_set_err(p.err, QB_DEVERR_PAGE);
      page = 0;
    }
    const int64_t row0 = ((int64_t)page * PAGE + (tok0 % PAGE)) * p.hkv + kvh;
#pragma unroll
    for (int i = 0; i < (DEC_TOK * 16) / (DEC_WARPS * 32); ++i) {
      const int idx = tid + i * DEC_WARPS * 32;
      const int r = idx >> 4, c = idx & 15;
      const bool ok = page_ok && (tok0 + r < tok_end);  // rows past the keys are zero-filled
      const int64_t goff = (row0 + (int64_t)r * p.hkv) * D + c * 8;
      cp_async_16(kbase + swz128(r, c), ok ? (const void*)(p.kc + goff) : (const void*)p.kc, ok ? 16 : 0);
      cp_async_16(vbase + swz128(r, c), ok ? (const void*)(p.vc + goff) : (const void*)p.vc, ok ? 16 : 0);
    }
  };
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < n_stages) load_stage(s);
    cp_async_commit();
  }

  float m_run[2] = {NEG_INF, NEG_INF}, l_run[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int wrow = warp * 16;
  for (int s = 0; s < n_stages; ++s) {
    if (s + STAGES - 1 < n_stages) load_stage(s + STAGES - 1);
    cp_async_commit();
    cp_async_wait<STAGES - 1>();
    __syncthreads();
    const int buf = s % STAGES;
    const uint32_t kbase = smem_u32(smem + buf * DEC_STAGE_BYTES);
    const uint32_t vbase = kbase + DEC_TOK * ROWB;
    const int key0 = tok_begin + s * DEC_TOK + wrow;
    if (key0 < tok_end) {  // this warp's 16 tokens hold at least one key
      // S[16 q x 16 tok] = Q K^T (two n-tiles of 8 tokens)
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(kbase + swz128(wrow + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), r0, r1, r2,
                    r3);
        mma_bf16_16816(sc[0], qa[kk], r0, r1);
        mma_bf16_16816(sc[1], qa[kk], r2, r3);
      }
      float mt[2] = {NEG_INF, NEG_INF};
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int kc = key0 + nt * 8 + 2 * t4;
        sc[nt][0] = kc < tok_end ? sc[nt][0] * p.scale_log2 : NEG_INF;
        sc[nt][1] = kc + 1 < tok_end ? sc[nt][1] * p.scale_log2 : NEG_INF;
        sc[nt][2] = kc < tok_end ? sc[nt][2] * p.scale_log2 : NEG_INF;
        sc[nt][3] = kc + 1 < tok_end ? sc[nt][3] * p.scale_log2 : NEG_INF;
        mt[0] = fmaxf(mt[0], fmaxf(sc[nt][0], sc[nt][1]));
        mt[1] = fmaxf(mt[1], fmaxf(sc[nt][2], sc[nt][3]));
      }
      float alpha[2], mnew[2], rs[2] = {0.f, 0.f};
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 1));
        mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 2));
        mnew[r] = fmaxf(m_run[r], mt[r]);
        alpha[r] = (mnew[r] == NEG_INF) ? 1.f : exp2f(m_run[r] - mnew[r]);
        m_run[r] = mnew[r];
      }
      uint32_t pa[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const float p0 = (mnew[0] == NEG_INF) ? 0.f : exp2f(sc[nt][0] - mnew[0]);
        const float p1 = (mnew[0] == NEG_INF) ? 0.f : exp2f(sc[nt][1] - mnew[0]);
        const float p2 = (mnew[1] == NEG_INF) ? 0.f : exp2f(sc[nt][2] - mnew[1]);
        const float p3 = (mnew[1] == NEG_INF) ? 0.f : exp2f(sc[nt][3] - mnew[1]);
        rs[0] += p0 + p1;
        rs[1] += p2 + p3;
        pa[2 * nt] = pack_bf16x2(p0, p1);
        pa[2 * nt + 1] = pack_bf16x2(p2, p3);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
        l_run[r] = l_run[r] * alpha[r] + rs[r];
      }
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][0] *= alpha[0];
        o[dt][1] *= alpha[0];
        o[dt][2] *= alpha[1];
        o[dt][3] *= alpha[1];
      }
      // O[16 x 128] += P[16 x 16 tok] V[16 tok x 128]
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4_trans(vbase + swz128(wrow + (lane & 7) + (((lane >> 3) & 1) << 3), dp * 2 + (lane >> 4)), r0, r1,
                          r2, r3);
        mma_bf16_16816(o[2 * dp], pa, r0, r1);
        mma_bf16_16816(o[2 * dp + 1], pa, r2, r3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Merge the four warps: smem [warp][16 rows][128] floats + m, l per (warp, row).
  float* so = reinterpret_cast<float*>(smem);
  float* sm = so + DEC_WARPS * 16 * D;
  float* sl = sm + DEC_WARPS * 16;
  __syncthreads();
#pragma unroll
  for (int dt = 0; dt < 16; ++dt) {
    *reinterpret_cast<float2*>(so + (wrow + g) * D + dt * 8 + 2 * t4) = make_float2(o[dt][0], o[dt][1]);
    *reinterpret_cast<float2*>(so + (wrow + g + 8) * D + dt * 8 + 2 * t4) = make_float2(o[dt][2], o[dt][3]);
  }
  if (t4 == 0) {
    sm[wrow + g] = m_run[0];
    sm[wrow + g + 8] = m_run[1];
    sl[wrow + g] = l_run[0];
    sl[wrow + g + 8] = l_run[1];
  }
  __syncthreads();
  {
    const int r = tid >> 3, d0 = (tid & 7) * 16;  // row r: member r/2, head h0 + r%2
    const int b = __shfl_sync(0xffffffffu, mem, r >> 1);
    float M = NEG_INF;
#pragma unroll
    for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, sm[w * 16 + r]);
    float L = 0.f, acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
    for (int w = 0; w < DEC_WARPS; ++w) {
      const float mw = sm[w * 16 + r];
      const float f = (mw == NEG_INF) ? 0.f : exp2f(mw - M);
      L += sl[w * 16 + r] * f;
#pragma unroll
      for (int i = 0; i < 16; i += 4) {
        const float4 v = *reinterpret_cast<const float4*>(so + (w * 16 + r) * D + d0 + i);
        acc[i] += v.x * f;
        acc[i + 1] += v.y * f;
        acc[i + 2] += v.z * f;
        acc[i + 3] += v.w * f;
      }
    }
    if (b >= 0) {
      const float inv = (L > 0.f) ? 1.f / L : 0.f;
      float* wr = p.ws + (((int64_t)b * p.n_slots + split) * p.hq + h0 + (r & 1)) * WS_ROW;
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<float4*>(wr + d0 + i) = make_float4(acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv,
                                                              acc[i + 3] * inv);
      if ((tid & 7) == 0) wr[D] = (L > 0.f) ? M + log2f(L) : NEG_INF;
    }
  }
}

// Two stage buffers (64 KB): three CTAs per SM overlap one another's start-up latency, which
// dominates the short own-key items of a decode step.
constexpr int GRP_STAGES = 2;
constexpr int GRP_SMEM = GRP_STAGES * DEC_STAGE_BYTES;

__global__ void __launch_bounds__(DEC_WARPS * 32)
paged_decode_grouped_kernel(DecodeParams p, GroupParams gp) {
  qb_pdl_trigger();
  qb_pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  int i = blockIdx.x;
  if (i < gp.n_shared_ctas) {
    const int split = i % gp.shared_splits;
    i /= gp.shared_splits;
    decode_shared_tile<GRP_STAGES>(p, gp, smem, split, i % p.hkv, i / p.hkv);
  } else {
    i -= gp.n_shared_ctas;
    const int split = i % gp.own_splits;
    i /= gp.own_splits;
    decode_own_tile<GRP_STAGES>(p, smem, split, i % p.hkv, i / p.hkv);
  }
}

// ============================================================================
// Varlen causal forward (paged or dense K/V), FlashAttention-2 schedule
// ============================================================================
// CTA = (64-row query tile, q head).  4 warps x 16 query rows.  K/V tiles of 64
// keys, double buffered.  Smem: Q 16 KB + 2 x (K 16 KB + V 16 KB) = 80 KB.
constexpr int FA_BM = 64, FA_BN = 64, FA_WARPS = 4;
constexpr int FA_TILE_BYTES = FA_BN * ROWB;
constexpr int FA_SMEM = FA_BM * ROWB + 2 * 2 * FA_TILE_BYTES;

struct FwdParams {
  const bf16* q;
  int64_t q_stride;
  const bf16* k;
  const bf16* v;
  int64_t kv_stride;
  const int32_t* bt;
  int64_t bt_stride, num_blocks;
  const int32_t* cu_q;
  const int32_t* cu_k;
  const int32_t* tiles;
  int tiles_per_seq;
  int hq, hkv;
  float scale_log2;
  bf16* out;
  int64_t o_stride;
  float* lse;
  int64_t total_q;
  int* err;
};

template <bool PAGED>
__global__ void __launch_bounds__(FA_WARPS * 32)
attn_fwd_kernel(FwdParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const int tile = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int b = p.tiles ? p.tiles[2 * tile] : tile / p.tiles_per_seq;
  const int q_start = p.tiles ? p.tiles[2 * tile + 1] : (tile % p.tiles_per_seq) * FA_BM;
  const int qb0 = p.cu_q[b], Lq = p.cu_q[b + 1] - qb0;
  const int kb0 = p.cu_k[b], Lk = p.cu_k[b + 1] - kb0;
  if (q_start >= Lq || Lk < Lq) {
    if (Lk < Lq && tid == 0) qb_set_err(p.err, QB_DEVERR_SHAPE);
    return;
  }
  const int kvh = h / (p.hq / p.hkv);
  const int shift = Lk - Lq;  // query row i sits at key position shift + i
  const int n_kv = min(Lk, q_start + FA_BM + shift);
  const int n_tiles = (n_kv + FA_BN - 1) / FA_BN;

  const uint32_t sQ = smem_u32(smem);
  const uint32_t sKV = sQ + FA_BM * ROWB;  // buf i: K at sKV + i*2*TILE, V after it

  // Q tile load (zero-fill rows >= Lq).
#pragma unroll
  for (int i = 0; i < (FA_BM * 16) / (FA_WARPS * 32); ++i) {
    const int idx = tid + i * FA_WARPS * 32;
    const int r = idx >> 4, c = idx & 15;
    const bool ok = q_start + r < Lq;
    const bf16* src = p.q + (int64_t)(qb0 + q_start + (ok ? r : 0)) * p.q_stride + h * D + c * 8;
    cp_async_16(sQ + swz128(r, c), src, ok ? 16 : 0);
  }
  const int32_t* btrow = PAGED ? p.bt + (int64_t)b * p.bt_stride : nullptr;
  auto load_kv = [&](int j, int buf) {
    const uint32_t kb = sKV + buf * 2 * FA_TILE_BYTES, vb = kb + FA_TILE_BYTES;
    const int key0 = j * FA_BN;
#pragma unroll
    for (int i = 0; i < (FA_BN * 16) / (FA_WARPS * 32); ++i) {
      const int idx = tid + i * FA_WARPS * 32;
      const int r = idx >> 4, c = idx & 15;
      const int key = key0 + r;
      bool ok = key < n_kv;
      int64_t off = 0;
      if (ok) {
        if (PAGED) {
          const int page = (key / PAGE < p.bt_stride) ? btrow[key / PAGE] : -1;
          if (page < 0 || page >= p.num_blocks) {
            qb_set_err(p.err, QB_DEVERR_PAGE);
            ok = false;
          } else {
            off = (((int64_t)page * PAGE + key % PAGE) * p.hkv + kvh) * D + c * 8;
          }
        } else {
          off = (int64_t)(kb0 + key) * p.kv_stride + kvh * D + c * 8;
        }
      }
      cp_async_16(kb + swz128(r, c), ok ? (const void*)(p.k + off) : (const void*)p.k, ok ? 16 : 0);
      cp_async_16(vb + swz128(r, c), ok ? (const void*)(p.v + off) : (const void*)p.v, ok ? 16 : 0);
    }
  };
  load_kv(0, 0);
  cp_async_commit();  // group 0: Q + KV tile 0

  float m_run[2] = {NEG_INF, NEG_INF}, l_run[2] = {0.f, 0.f};
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  uint32_t qa[8][4];
  const int row_g = q_start + warp * 16 + g;  // query row index (within seq) of c0/c1
  const int lim0 = shift + row_g, lim1 = shift + row_g + 8;  // inclusive key limits

  for (int j = 0; j < n_tiles; ++j) {
    if (j + 1 < n_tiles) load_kv(j + 1, (j + 1) & 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        ldmatrix_x4(sQ + swz128(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), qa[kk][0], qa[kk][1],
                    qa[kk][2], qa[kk][3]);
    }
    const uint32_t kb = sKV + (j & 1) * 2 * FA_TILE_BYTES, vb = kb + FA_TILE_BYTES;
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(kb + swz128(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), r0,
                    r1, r2, r3);
        mma_bf16_16816(s[2 * np], qa[kk], r0, r1);
        mma_bf16_16816(s[2 * np + 1], qa[kk], r2, r3);
      }
    }
    // scale, mask, online softmax (two rows per lane: g and g+8)
    const int key0 = j * FA_BN;
    float mt[2] = {NEG_INF, NEG_INF};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int kc = key0 + nt * 8 + 2 * t4;
      s[nt][0] = (kc <= lim0 && kc < n_kv) ? s[nt][0] * p.scale_log2 : NEG_INF;
      s[nt][1] = (kc + 1 <= lim0 && kc + 1 < n_kv) ? s[nt][1] * p.scale_log2 : NEG_INF;
      s[nt][2] = (kc <= lim1 && kc < n_kv) ? s[nt][2] * p.scale_log2 : NEG_INF;
      s[nt][3] = (kc + 1 <= lim1 && kc + 1 < n_kv) ? s[nt][3] * p.scale_log2 : NEG_INF;
      mt[0] = fmaxf(mt[0], fmaxf(s[nt][0], s[nt][1]));
      mt[1] = fmaxf(mt[1], fmaxf(s[nt][2], s[nt][3]));
    }
    float alpha[2], mnew[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 1));
      mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], 2));
      mnew[r] = fmaxf(m_run[r], mt[r]);
      alpha[r] = (mnew[r] == NEG_INF) ? 1.f : exp2f(m_run[r] - mnew[r]);
      m_run[r] = mnew[r];
    }
    float rs[2] = {0.f, 0.f};
    uint32_t pa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = (mnew[0] == NEG_INF) ? 0.f : exp2f(s[nt][0] - mnew[0]);
      const float p1 = (mnew[0] == NEG_INF) ? 0.f : exp2f(s[nt][1] - mnew[0]);
      const float p2 = (mnew[1] == NEG_INF) ? 0.f : exp2f(s[nt][2] - mnew[1]);
      const float p3 = (mnew[1] == NEG_INF) ? 0.f : exp2f(s[nt][3] - mnew[1]);
      rs[0] += p0 + p1;
      rs[1] += p2 + p3;
      const int ks = nt >> 1;
      if ((nt & 1) == 0) {
        pa[ks][0] = pack_bf16x2(p0, p1);
        pa[ks][1] = pack_bf16x2(p2, p3);
      } else {
        pa[ks][2] = pack_bf16x2(p0, p1);
        pa[ks][3] = pack_bf16x2(p2, p3);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      o[dt][0] *= alpha[0];
      o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1];
      o[dt][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4_trans(vb + swz128(ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), dp * 2 + (lane >> 4)),
                          r0, r1, r2, r3);
        mma_bf16_16816(o[2 * dp], pa[ks], r0, r1);
        mma_bf16_16816(o[2 * dp + 1], pa[ks], r2, r3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // Epilogue: normalise and store rows < Lq.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = row_g + r * 8;
    if (qi >= Lq) continue;
    const float inv = (l_run[r] > 0.f) ? 1.f / l_run[r] : 0.f;
    bf16* orow = p.out + (int64_t)(qb0 + qi) * p.o_stride + h * D;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
      *reinterpret_cast<uint32_t*>(orow + dt * 8 + 2 * t4) =
          pack_bf16x2(o[dt][2 * r] * inv, o[dt][2 * r + 1] * inv);
    if (p.lse && t4 == 0)
      p.lse[(int64_t)h * p.total_q + qb0 + qi] =
          (l_run[r] > 0.f) ? (m_run[r] + log2f(l_run[r])) / LOG2E : NEG_INF;
  }
}

// ============================================================================
// Dense varlen backward (Lq == Lk), FlashAttention-2 style, deterministic:
//   delta = rowsum(dO * O);
//   dK, dV per key tile (both query heads of the kv group summed in registers);
//   dQ per query tile in a second kernel (no atomics).
// ============================================================================
struct BwdParams {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  int64_t stride;
  const bf16* o;
  const bf16* dout;
  int64_t o_stride;
  const float* lse;
  const int32_t* cu;
  const int32_t* tiles;
  int hq, hkv;
  float scale, scale_log2;
  int64_t total;
  float* delta;
  bf16* dq;
  bf16* dk;
  bf16* dv;
  int* err;
};

// delta[h, row] = sum_d dO[row,h,d] * O[row,h,d]; one warp per (row, head).
__global__ void attn_bwd_delta_kernel(BwdParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= p.total * p.hq) return;
  const int lane = threadIdx.x & 31;
  const int64_t row = item / p.hq;
  const int h = (int)(item % p.hq);
  const bf16* orow = p.o + row * p.o_stride + h * D + lane * 4;
  const bf16* drow = p.dout + row * p.o_stride + h * D + lane * 4;
  uint2 ou = *reinterpret_cast<const uint2*>(orow), du = *reinterpret_cast<const uint2*>(drow);
  float2 o0 = unpack_bf16x2(ou.x), o1 = unpack_bf16x2(ou.y);
  float2 d0 = unpack_bf16x2(du.x), d1 = unpack_bf16x2(du.y);
  float acc = o0.x * d0.x + o0.y * d0.y + o1.x * d1.x + o1.y * d1.y;
  acc = warp_sum(acc);
  if (lane == 0) p.delta[(int64_t)h * p.total + row] = acc;
}

// Loads a [64 x 128] bf16 tile (rows row0.., valid while < nvalid) into swizzled smem.
QB_DEVICE void load_tile64(uint32_t dst, const bf16* base, int64_t stride, int row0, int nvalid,
                           int col_off, int tid, int nthreads) {
  for (int idx = tid; idx < 64 * 16; idx += nthreads) {
    const int r = idx >> 4, c = idx & 15;
    const bool ok = r < nvalid;
    const bf16* src = base + (int64_t)(row0 + (ok ? r : 0)) * stride + col_off + c * 8;
    cp_async_16(dst + swz128(r, c), src, ok ? 16 : 0);
  }
}

// CTA = (64-key tile, kv head), 4 warps x 16 keys.  Loops over the query tiles at
// or after the key tile and over the hq/hkv query heads of the group, as one flat sequence
// whose next (Q, dO, lse, delta) tile is copied in while the current one is used.
// Smem: K 16K, V 16K, 2 x (Q 16K, dO 16K, lse 256 B, delta 256 B) = 97 KB.
constexpr int DKDV_SMEM = 6 * 64 * ROWB + 2 * 2 * 64 * 4;
// dQ: Q 16K, dO 16K, 2 x (K 16K, V 16K) = 96 KB; the next key tile is copied in while the
// current one is used.
constexpr int DQ_SMEM = 6 * 64 * ROWB;

__global__ void __launch_bounds__(128)
attn_bwd_dkdv_kernel(BwdParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const int tile = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int b = p.tiles[2 * tile], k_start = p.tiles[2 * tile + 1];
  const int base = p.cu[b], L = p.cu[b + 1] - base;
  if (k_start >= L) return;
  const int group = p.hq / p.hkv;
  const uint32_t sK = smem_u32(smem), sV = sK + 64 * ROWB;
  // buffer b: Q at sQb(b), dO 16 KB after it; lse and delta (64 fp32 each) at sLb(b)
  auto sQb = [&](int buf) { return sV + 64 * ROWB + buf * 2 * 64 * ROWB; };
  auto sLb = [&](int buf) { return sK + 6 * 64 * ROWB + buf * 2 * 64 * 4; };
  const float* sLf = reinterpret_cast<const float*>(smem + 6 * 64 * ROWB);
  const int nk = min(64, L - k_start);
  const int q0 = (k_start / 64) * 64;
  const int nqt = (L - q0 + 63) / 64;  // query tiles per head
  const int n_it = group * nqt;
  auto load_it = [&](int it, int buf) {
    const int h = kvh * group + it / nqt, q_start = q0 + (it % nqt) * 64;
    const int nq = min(64, L - q_start);
    load_tile64(sQb(buf), p.q, p.stride, base + q_start, nq, h * D, tid, 128);
    load_tile64(sQb(buf) + 64 * ROWB, p.dout, p.o_stride, base + q_start, nq, h * D, tid, 128);
    {  // lse (idx < 64) and delta (idx >= 64) of the tile's queries, zero past the sequence
      const int which = tid >> 6, j = tid & 63;
      const bool ok = j < nq;
      const float* src = (which ? p.delta : p.lse) + (int64_t)h * p.total + base + q_start + (ok ? j : 0);
      cp_async_4(sLb(buf) + which * 256 + j * 4, src, ok ? 4 : 0);
    }
  };
  load_tile64(sK, p.k, p.stride, base + k_start, nk, kvh * D, tid, 128);
  load_tile64(sV, p.v, p.stride, base + k_start, nk, kvh * D, tid, 128);
  load_it(0, 0);
  cp_async_commit();
  float dk[16][4], dv[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int key_g = k_start + warp * 16 + g;  // key index of rows g / g+8 in this warp
  for (int it = 0; it < n_it; ++it) {
    const int q_start = q0 + (it % nqt) * 64;
    const int buf = it & 1;
    if (it + 1 < n_it) load_it(it + 1, buf ^ 1);  // the buffer read in iteration it - 1
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const uint32_t sQ = sQb(buf), sD = sQ + 64 * ROWB;
    const float* sl = sLf + buf * 128;  // lse [0, 64), delta [64, 128)
    {
      // S^T[16 keys x 64 q] = K Q^T ; dP^T = V dO^T
      float st[8][4], dpt[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
        dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        // K and V fragments as A operands (rows = this warp's 16 keys), re-read from smem.
        uint32_t ka[4], va[4];
        ldmatrix_x4(sK + swz128(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), ka[0], ka[1], ka[2], ka[3]);
        ldmatrix_x4(sV + swz128(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), va[0], va[1], va[2], va[3]);
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t r0, r1, r2, r3;
          ldmatrix_x4(sQ + swz128(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), r0,
                      r1, r2, r3);
          mma_bf16_16816(st[2 * np], ka, r0, r1);
          mma_bf16_16816(st[2 * np + 1], ka, r2, r3);
          ldmatrix_x4(sD + swz128(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), r0,
                      r1, r2, r3);
          mma_bf16_16816(dpt[2 * np], va, r0, r1);
          mma_bf16_16816(dpt[2 * np + 1], va, r2, r3);
        }
      }
      // P^T = exp(S^T*scale - lse[q]) masked to key <= q ; dS^T = P^T * (dP^T - delta[q])
      uint32_t pt[4][4], dst[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int qc = q_start + nt * 8 + 2 * t4;  // query index of cols (c0,c2) ; +1 for (c1,c3)
        float pv[4], dsv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int qi = qc + (e & 1);
          const int ki = key_g + ((e >> 1) << 3);
          const bool ok = qi < L && ki <= qi && ki < L;
          const float l = sl[qi - q_start];
          const float dl = sl[64 + qi - q_start];
          const float pe = ok ? exp2f(st[nt][e] * p.scale_log2 - l * LOG2E) : 0.f;
          pv[e] = pe;
          dsv[e] = pe * (dpt[nt][e] - dl);
        }
        const int ks = nt >> 1;
        if ((nt & 1) == 0) {
          pt[ks][0] = pack_bf16x2(pv[0], pv[1]);
          pt[ks][1] = pack_bf16x2(pv[2], pv[3]);
          dst[ks][0] = pack_bf16x2(dsv[0], dsv[1]);
          dst[ks][1] = pack_bf16x2(dsv[2], dsv[3]);
        } else {
          pt[ks][2] = pack_bf16x2(pv[0], pv[1]);
          pt[ks][3] = pack_bf16x2(pv[2], pv[3]);
          dst[ks][2] = pack_bf16x2(dsv[0], dsv[1]);
          dst[ks][3] = pack_bf16x2(dsv[2], dsv[3]);
        }
      }
      // dV += P^T dO ; dK += dS^T Q   (B operands: [q][d] tiles -> ldmatrix.trans)
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int dp = 0; dp < 8; ++dp) {
          uint32_t r0, r1, r2, r3;
          const uint32_t off = swz128(ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), dp * 2 + (lane >> 4));
          ldmatrix_x4_trans(sD + off, r0, r1, r2, r3);
          mma_bf16_16816(dv[2 * dp], pt[ks], r0, r1);
          mma_bf16_16816(dv[2 * dp + 1], pt[ks], r2, r3);
          ldmatrix_x4_trans(sQ + off, r0, r1, r2, r3);
          mma_bf16_16816(dk[2 * dp], dst[ks], r0, r1);
          mma_bf16_16816(dk[2 * dp + 1], dst[ks], r2, r3);
        }
      }
    }
    __syncthreads();  // this buffer is refilled by the copy issued in iteration it + 1
  }
  // Store dK (times scale) and dV for rows < L.
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int ki = key_g + r * 8;
    if (ki >= L) continue;
    bf16* dkrow = p.dk + (int64_t)(base + ki) * p.stride + kvh * D;
    bf16* dvrow = p.dv + (int64_t)(base + ki) * p.stride + kvh * D;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      *reinterpret_cast<uint32_t*>(dkrow + dt * 8 + 2 * t4) =
          pack_bf16x2(dk[dt][2 * r] * p.scale, dk[dt][2 * r + 1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvrow + dt * 8 + 2 * t4) = pack_bf16x2(dv[dt][2 * r], dv[dt][2 * r + 1]);
    }
  }
}

// CTA = (64-query tile, q head), 4 warps x 16 queries; loops over key tiles <= the query tile.
__global__ void __launch_bounds__(128)
attn_bwd_dq_kernel(BwdParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  extern __shared__ __align__(128) uint8_t smem[];
  const int tile = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int b = p.tiles[2 * tile], q_start = p.tiles[2 * tile + 1];
  const int base = p.cu[b], L = p.cu[b + 1] - base;
  if (q_start >= L) return;
  const int kvh = h / (p.hq / p.hkv);
  const uint32_t sQ = smem_u32(smem), sD = sQ + 64 * ROWB;
  // key tile buffer b: K at sKb(b), V 16 KB after it
  auto sKb = [&](int buf) { return sD + 64 * ROWB + buf * 2 * 64 * ROWB; };
  const int nq = min(64, L - q_start);
  const int kend = min(L, q_start + 64);
  const int n_kt = (kend + 63) / 64;
  auto load_kv = [&](int kt, int buf) {
    const int nk = min(64, L - kt * 64);
    load_tile64(sKb(buf), p.k, p.stride, base + kt * 64, nk, kvh * D, tid, 128);
    load_tile64(sKb(buf) + 64 * ROWB, p.v, p.stride, base + kt * 64, nk, kvh * D, tid, 128);
  };
  load_tile64(sQ, p.q, p.stride, base + q_start, nq, h * D, tid, 128);
  load_tile64(sD, p.dout, p.o_stride, base + q_start, nq, h * D, tid, 128);
  load_kv(0, 0);
  cp_async_commit();
  uint32_t qa[8][4], da[8][4];
  const int qg = q_start + warp * 16 + g;
  float lse_r[2], dl_r[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = min(qg + r * 8, L - 1);
    lse_r[r] = p.lse[(int64_t)h * p.total + base + qi] * LOG2E;
    dl_r[r] = p.delta[(int64_t)h * p.total + base + qi];
  }
  float dq[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  for (int kt = 0; kt < n_kt; ++kt) {
    const int k_start = kt * 64;
    if (kt + 1 < n_kt) load_kv(kt + 1, (kt + 1) & 1);  // the buffer read in iteration kt - 1
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kt == 0) {  // Q and dO fragments stay in registers for the whole key loop
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        ldmatrix_x4(sQ + swz128(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), qa[kk][0], qa[kk][1], qa[kk][2],
                    qa[kk][3]);
        ldmatrix_x4(sD + swz128(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)), da[kk][0], da[kk][1], da[kk][2],
                    da[kk][3]);
      }
    }
    const uint32_t sK = sKb(kt & 1), sV = sK + 64 * ROWB;
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
      dp[i][0] = dp[i][1] = dp[i][2] = dp[i][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(sK + swz128(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), r0, r1,
                    r2, r3);
        mma_bf16_16816(s[2 * np], qa[kk], r0, r1);
        mma_bf16_16816(s[2 * np + 1], qa[kk], r2, r3);
        ldmatrix_x4(sV + swz128(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 2 + ((lane >> 3) & 1)), r0, r1,
                    r2, r3);
        mma_bf16_16816(dp[2 * np], da[kk], r0, r1);
        mma_bf16_16816(dp[2 * np + 1], da[kk], r2, r3);
      }
    }
    uint32_t dsa[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int kc = k_start + nt * 8 + 2 * t4;
      float dsv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ki = kc + (e & 1);
        const int qi = qg + ((e >> 1) << 3);
        const bool ok = qi < L && ki <= qi;
        const float pe = ok ? exp2f(s[nt][e] * p.scale_log2 - lse_r[e >> 1]) : 0.f;
        dsv[e] = pe * (dp[nt][e] - dl_r[e >> 1]);
      }
      const int ks = nt >> 1;
      if ((nt & 1) == 0) {
        dsa[ks][0] = pack_bf16x2(dsv[0], dsv[1]);
        dsa[ks][1] = pack_bf16x2(dsv[2], dsv[3]);
      } else {
        dsa[ks][2] = pack_bf16x2(dsv[0], dsv[1]);
        dsa[ks][3] = pack_bf16x2(dsv[2], dsv[3]);
      }
    }
    // dQ += dS K   (B = K [key][d] -> ldmatrix.trans)
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int dpi = 0; dpi < 8; ++dpi) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4_trans(sK + swz128(ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), dpi * 2 + (lane >> 4)), r0,
                          r1, r2, r3);
        mma_bf16_16816(dq[2 * dpi], dsa[ks], r0, r1);
        mma_bf16_16816(dq[2 * dpi + 1], dsa[ks], r2, r3);
      }
    }
    __syncthreads();  // this buffer is refilled by the copy issued in iteration kt + 1
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qg + r * 8;
    if (qi >= L) continue;
    bf16* row = p.dq + (int64_t)(base + qi) * p.stride + h * D;
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
      *reinterpret_cast<uint32_t*>(row + dt * 8 + 2 * t4) =
          pack_bf16x2(dq[dt][2 * r] * p.scale, dq[dt][2 * r + 1] * p.scale);
  }
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// ================================================================ C ABI
// tcgen05 forward for packed sequences (attn_tc.cu)
int attn_fwd_tc_launch(const void* q, int64_t q_stride, const void* k, const void* v, int64_t kv_stride,
                       const int32_t* cu_seqlens, int batch, const int32_t* tile_info, int n_tiles, int tiles_per_seq,
                       int hq, int hkv, float scale, void* out, int64_t o_stride, float* lse, int64_t total_q, int* err,
                       cudaStream_t st);

int attn_bwd_dkdv_tc_launch(const void* q, const void* k, const void* v, int64_t stride, const void* dout,
                            int64_t o_stride, const float* lse, const float* delta, const int32_t* cu_seqlens,
                            const int32_t* tile_info, int n_tiles, int hq, int hkv, float scale, int64_t total,
                            void* dk, void* dv, int* err, cudaStream_t st);

int attn_bwd_dq_tc_launch(const void* q, const void* k, const void* v, int64_t stride, const void* dout,
                          int64_t o_stride, const float* lse, const float* delta, const int32_t* cu_seqlens,
                          const int32_t* tile_info, int n_tiles, int hq, int hkv, float scale, int64_t total, void* dq,
                          int* err, cudaStream_t st);

extern "C" size_t qb_paged_decode_workspace_bytes(int batch, int hq, int Dh, int max_splits) {
  if (max_splits <= 1) return 0;
  return (size_t)batch * max_splits * hq * (Dh + 4) * sizeof(float);
}

extern "C" int qb_paged_decode_attn(const void* q, const void* k_cache, const void* v_cache,
                                    int64_t num_blocks, int page_size, const int32_t* block_tables,
                                    int64_t bt_stride, const int32_t* seqlens, int seqlen_add,
                                    int batch, int hq, int hkv, int Dh, float scale,
                                    int split_tokens, int max_splits, float* workspace, void* out,
                                    int* err, qb_stream_t stream) {
  if (Dh != D || page_size != PAGE || hq != 2 * hkv) return QB_ERR_UNSUPPORTED;
  QB_CHECK_ARG(batch >= 0 && batch <= 65535 && hkv > 0 && num_blocks > 0 && max_splits >= 1 &&
               max_splits <= 65535);
  QB_CHECK_ARG(split_tokens >= DEC_TOK && split_tokens % DEC_TOK == 0);
  if (batch == 0) return QB_OK;
  QB_CHECK_ARG(q && k_cache && v_cache && block_tables && seqlens && out && al16(q) && al16(k_cache) &&
               al16(v_cache) && al16(out) && bt_stride > 0);
  QB_CHECK_ARG(max_splits == 1 || (workspace && al16(workspace)));
  DecodeParams p{(const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, num_blocks, block_tables,
                 bt_stride, seqlens, seqlen_add, hq, hkv, scale * LOG2E, split_tokens, max_splits,
                 workspace, (bf16*)out, err, max_splits, 0, nullptr};
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(paged_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DEC_SMEM);
    attr_set = true;
  }
  dim3 grid((unsigned)max_splits, (unsigned)hkv, (unsigned)batch);
  int st = qb_launch(paged_decode_kernel, dim3(grid), dim3(DEC_WARPS * 32), DEC_SMEM, (cudaStream_t)stream, 1, p);
  if (st != QB_OK || max_splits == 1) return st;
  const int wpb = 8;
  return qb_launch(paged_decode_combine_kernel, dim3((unsigned)((batch * hq + wpb - 1) / wpb)), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, p, batch);
}

extern "C" size_t qb_paged_decode_grouped_workspace_bytes(int batch, int hq, int Dh, int n_slots) {
  // split-K partials: n_slots per (sequence, head)
  return (size_t)batch * n_slots * hq * (Dh + 4) * sizeof(float);
}

extern "C" int qb_paged_decode_attn_grouped(const void* q, const void* k_cache, const void* v_cache,
                                            int64_t num_blocks, int page_size, const int32_t* block_tables,
                                            int64_t bt_stride, const int32_t* seqlens, int seqlen_add, int batch,
                                            int hq, int hkv, int Dh, float scale, const int32_t* group_members,
                                            const int32_t* shared_len, int n_groups, const int32_t* kv_start,
                                            int split_tokens, int shared_splits, int own_splits, float* workspace,
                                            void* out, int* err, qb_stream_t stream) {
  if (Dh != D || page_size != PAGE || hq != 2 * hkv) return QB_ERR_UNSUPPORTED;
  QB_CHECK_ARG(batch >= 0 && batch <= 65535 && n_groups >= 0 && n_groups <= 65535 && hkv > 0 && num_blocks > 0);
  QB_CHECK_ARG(split_tokens >= DEC_TOK && split_tokens % DEC_TOK == 0 && shared_splits >= 1 && own_splits >= 1 &&
               shared_splits + own_splits <= 65535);
  if (batch == 0) return QB_OK;
  QB_CHECK_ARG(q && k_cache && v_cache && block_tables && seqlens && out && workspace && group_members &&
               shared_len && kv_start && al16(q) && al16(k_cache) && al16(v_cache) && al16(workspace) &&
               al16(out) && bt_stride > 0);
  const int n_slots = shared_splits + own_splits;
  const int64_t n_shared = (int64_t)shared_splits * hkv * n_groups;
  const int64_t n_ctas = n_shared + (int64_t)own_splits * hkv * batch;
  QB_CHECK_ARG(n_ctas < (1ll << 31));
  // shared splits fill slots [0, shared_splits), own splits the rest; n_slots >= 2, so every CTA
  // writes a partial and the combine kernel produces the output
  DecodeParams d{(const bf16*)q, (const bf16*)k_cache, (const bf16*)v_cache, num_blocks, block_tables, bt_stride,
                 seqlens, seqlen_add, hq, hkv, scale * LOG2E, split_tokens, n_slots, workspace, (bf16*)out, err,
                 n_slots, shared_splits, kv_start};
  GroupParams gp{group_members, shared_len, batch, shared_splits, own_splits, (int)n_shared};
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(paged_decode_grouped_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GRP_SMEM);
    attr_set = true;
  }
  int st = qb_launch(paged_decode_grouped_kernel, dim3((unsigned)n_ctas), dim3(DEC_WARPS * 32), GRP_SMEM, (cudaStream_t)stream, 1, d, gp);
  if (st != QB_OK) return st;
  const int wpb = 8;
  // launched early: resident while the tile kernel finishes, it starts the moment that completes
  return qb_launch_ex(paged_decode_combine_kernel, dim3((unsigned)((batch * hq + wpb - 1) / wpb)), dim3(wpb * 32), 0,
                      (cudaStream_t)stream, 1, true, d, batch);
}

extern "C" int qb_attn_varlen_fwd(const void* q, int64_t q_stride, const void* k, const void* v,
                                  int64_t kv_stride, const int32_t* block_tables, int64_t bt_stride,
                                  int64_t num_blocks, int page_size, const int32_t* cu_seqlens_q,
                                  const int32_t* cu_seqlens_k, int batch, const int32_t* tile_info,
                                  int n_tiles, int tiles_per_seq, int hq, int hkv, int Dh,
                                  float scale, void* out, int64_t o_stride, float* lse,
                                  int64_t total_q, int* err, qb_stream_t stream) {
  if (Dh != D || hq % hkv != 0) return QB_ERR_UNSUPPORTED;
  const bool paged = block_tables != nullptr;
  if (paged && page_size != PAGE) return QB_ERR_UNSUPPORTED;
  QB_CHECK_ARG(batch >= 0 && n_tiles >= 0 && hkv > 0);
  if (!tile_info) {
    QB_CHECK_ARG(tiles_per_seq >= 0);
    n_tiles = batch * tiles_per_seq;
  }
  if (n_tiles == 0 || batch == 0) return QB_OK;
  QB_CHECK_ARG(q && k && v && out && cu_seqlens_q && cu_seqlens_k);
  QB_CHECK_ARG(al16(q) && al16(k) && al16(v) && al16(out) && q_stride % 8 == 0 && o_stride % 8 == 0);
  QB_CHECK_ARG(paged ? (num_blocks > 0 && bt_stride > 0) : (kv_stride % 8 == 0));
  QB_CHECK_ARG(lse == nullptr || total_q > 0);
  if (!paged && hq == 2 * hkv && cu_seqlens_q == cu_seqlens_k)  // training / recompute: tcgen05 kernel
    return attn_fwd_tc_launch(q, q_stride, k, v, kv_stride, cu_seqlens_q, batch, tile_info, n_tiles,
                              tile_info ? 0 : tiles_per_seq, hq, hkv, scale, out, o_stride, lse, total_q, err,
                              (cudaStream_t)stream);
  FwdParams p{(const bf16*)q, q_stride, (const bf16*)k, (const bf16*)v, kv_stride, block_tables, bt_stride,
              num_blocks, cu_seqlens_q, cu_seqlens_k, tile_info, tiles_per_seq, hq, hkv, scale * LOG2E,
              (bf16*)out, o_stride, lse, total_q, err};
  dim3 grid((unsigned)n_tiles, (unsigned)hq);
  if (paged) {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_fwd_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
      set = true;
    }
    return qb_launch(attn_fwd_kernel<true>, dim3(grid), dim3(FA_WARPS * 32), FA_SMEM, (cudaStream_t)stream, 1, p);
  } else {
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(attn_fwd_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, FA_SMEM);
      set = true;
    }
    return qb_launch(attn_fwd_kernel<false>, dim3(grid), dim3(FA_WARPS * 32), FA_SMEM, (cudaStream_t)stream, 1,
                     p);
  }
}

extern "C" int qb_attn_varlen_bwd(const void* q, const void* k, const void* v, int64_t stride,
                                  const void* o, const void* dout, int64_t o_stride, const float* lse,
                                  const int32_t* cu_seqlens, int batch, const int32_t* tile_info,
                                  int n_tiles, int hq, int hkv, int Dh, float scale, int64_t total,
                                  float* delta, void* dq, void* dk, void* dv, int* err,
                                  qb_stream_t stream) {
  if (Dh != D || hq % hkv != 0) return QB_ERR_UNSUPPORTED;
  QB_CHECK_ARG(batch >= 0 && n_tiles >= 0 && total >= 0 && hkv > 0);
  if (n_tiles == 0 || batch == 0 || total == 0) return QB_OK;
  QB_CHECK_ARG(q && k && v && o && dout && lse && cu_seqlens && tile_info && delta && dq && dk && dv);
  QB_CHECK_ARG(al16(q) && al16(k) && al16(v) && al16(o) && al16(dout) && al16(dq) && al16(dk) && al16(dv));
  QB_CHECK_ARG(stride % 8 == 0 && o_stride % 8 == 0);
  BwdParams p{(const bf16*)q, (const bf16*)k, (const bf16*)v, stride, (const bf16*)o, (const bf16*)dout,
              o_stride, lse, cu_seqlens, tile_info, hq, hkv, scale, scale * LOG2E, total, delta,
              (bf16*)dq, (bf16*)dk, (bf16*)dv, err};
  const int wpb = 8;
  int st = qb_launch(attn_bwd_delta_kernel, dim3((unsigned)((total * hq + wpb - 1) / wpb)), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, p);
  if (st != QB_OK) return st;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(attn_bwd_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DKDV_SMEM);
    cudaFuncSetAttribute(attn_bwd_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM);
    set = true;
  }
  if (hq == 2 * hkv) {  // dK, dV on tcgen05
    st = attn_bwd_dkdv_tc_launch(q, k, v, stride, dout, o_stride, lse, delta, cu_seqlens, tile_info, n_tiles, hq,
                                 hkv, scale, total, dk, dv, err, (cudaStream_t)stream);
  } else {
    st = qb_launch(attn_bwd_dkdv_kernel, dim3(dim3((unsigned)n_tiles, (unsigned)hkv)), dim3(128), DKDV_SMEM, (cudaStream_t)stream, 1, p);
  }
  if (st != QB_OK) return st;
  if (hq == 2 * hkv)  // dQ on tcgen05
    return attn_bwd_dq_tc_launch(q, k, v, stride, dout, o_stride, lse, delta, cu_seqlens, tile_info, n_tiles, hq, hkv,
                                 scale, total, dq, err, (cudaStream_t)stream);
  return qb_launch(attn_bwd_dq_kernel, dim3(dim3((unsigned)n_tiles, (unsigned)hq)), dim3(128), DQ_SMEM, (cudaStream_t)stream, 1, p);
}
