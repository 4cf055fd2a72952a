// Embedding, RMSNorm, fused add+RMSNorm, QK-Norm + RoPE (+ paged KV store),
// SwiGLU and residual adds, forward and backward.
//
// All of these are HBM-bound row kernels: one warp owns one row (or one head
// of one token) and moves it with 16-byte vector loads, so every byte is read
// and written once.  fp32 is used for every reduction, bf16 only at the store,
// following the reference's RMSNorm (qwen3_naive.py:156-169) and Triton RoPE
// (qwen3_naive.py:53-67) rounding points.
#include "common.cuh"

namespace {

// ---------------------------------------------------------------- vector helpers
struct alignas(16) bf16x8 {
  uint32_t u[4];
};

QB_DEVICE void load8(const bf16* p, float (&v)[8]) {
  bf16x8 r = *reinterpret_cast<const bf16x8*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = unpack_bf16x2(r.u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
QB_DEVICE void unpack8(const bf16x8& r, float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(r.u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
QB_DEVICE void store8(bf16* p, const float (&v)[8]) {
  bf16x8 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) r.u[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<bf16x8*>(p) = r;
}

// ---------------------------------------------------------------- embedding
__global__ void embedding_fwd_kernel(const int64_t* __restrict__ ids, int64_t n,
                                     const bf16* __restrict__ table, int64_t vocab,
                                     int64_t hidden, bf16* __restrict__ out, int* err) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t id = ids[row];
  bf16* o = out + row * hidden;
  if (id < 0 || id >= vocab) {
    if (lane == 0) qb_set_err(err, QB_DEVERR_TOKEN);
    for (int64_t c = lane * 8; c < hidden; c += 256) *reinterpret_cast<bf16x8*>(o + c) = bf16x8{};
    return;
  }
  const bf16* t = table + id * hidden;
  for (int64_t c = lane * 8; c < hidden; c += 256)
    *reinterpret_cast<bf16x8*>(o + c) = *reinterpret_cast<const bf16x8*>(t + c);
}

__global__ void embedding_bwd_kernel(const int64_t* __restrict__ ids, int64_t n,
                                     const bf16* __restrict__ dout, int64_t vocab, int64_t hidden,
                                     float* __restrict__ dtable, int* err) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  const int lane = threadIdx.x & 31;
  const int64_t id = ids[row];
  if (id < 0 || id >= vocab) {
    if (lane == 0) qb_set_err(err, QB_DEVERR_TOKEN);
    return;
  }
  const bf16* g = dout + row * hidden;
  float* d = dtable + id * hidden;
  for (int64_t c = lane * 8; c < hidden; c += 256) {
    float v[8];
    load8(g + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) atomicAdd(d + c + i, v[i]);
  }
}

// ---------------------------------------------------------------- RMSNorm
// One warp per row; NV = cols / 256 vectors of 8 elements per lane.
template <int NV>
__global__ void rmsnorm_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                   bf16* __restrict__ y, float* __restrict__ rstd_out,
                                   int64_t rows, float eps) {
  qb_pdl_trigger();
  qb_pdl_wait();
  constexpr int COLS = NV * 256;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    load8(x + row * COLS + j * 256 + lane * 8, v[j]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += v[j][i] * v[j][i];
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)COLS + eps);
  if (rstd_out && lane == 0) rstd_out[row] = rstd;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float wv[8], o[8];
    load8(w + j * 256 + lane * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[j][i] * rstd) * wv[i];
    store8(y + row * COLS + j * 256 + lane * 8, o);
  }
}

template <int NV>
__global__ void add_rmsnorm_fwd_kernel(const bf16* __restrict__ x, bf16* __restrict__ res,
                                       const bf16* __restrict__ w, bf16* __restrict__ y,
                                       int64_t rows, float eps) {
  qb_pdl_trigger();
  qb_pdl_wait();
  constexpr int COLS = NV * 256;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  float v[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float r[8];
    const int64_t off = row * COLS + j * 256 + lane * 8;
    load8(x + off, v[j]);
    load8(res + off, r);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[j][i] += r[i];
      ss += v[j][i] * v[j][i];
    }
    store8(res + off, v[j]);  // residual <- bf16(x + r)
  }
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)COLS + eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    float wv[8], o[8];
    load8(w + j * 256 + lane * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[j][i] * rstd) * wv[i];
    store8(y + row * COLS + j * 256 + lane * 8, o);
  }
}

// dx = rstd * (dy*w - xhat * mean(dy*w*xhat)),  dw += sum_rows(dy * xhat).
// Grid-strided over rows, one warp a row, 128-thread blocks, four blocks per SM: the weight row
// and each warp's dw partial sit in shared memory (a lane owns its columns, so no atomics there)
// and a row's x and dy stay packed bf16 until used.  The block folds its warps' partials and
// issues one 16-byte atomic add per four columns.
constexpr int RMSB_WARPS = 4;
template <int NV>
__global__ void __launch_bounds__(RMSB_WARPS * 32, 3)
rmsnorm_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x, const bf16* __restrict__ w,
                   const float* __restrict__ rstd, bf16* __restrict__ dx, float* __restrict__ dw, int64_t rows) {
  qb_pdl_trigger();
  qb_pdl_wait();
  constexpr int COLS = NV * 256;
  extern __shared__ float rms_smem[];  // w [COLS] then one dw partial [COLS] per warp
  float* w_s = rms_smem;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float* dw_w = rms_smem + COLS * (1 + wid);
  for (int c = threadIdx.x; c < COLS; c += blockDim.x) w_s[c] = bf2f(w[c]);
  for (int c = lane; c < COLS; c += 32) dw_w[c] = 0.f;
  __syncthreads();
  for (int64_t row = (int64_t)blockIdx.x * RMSB_WARPS + wid; row < rows; row += (int64_t)gridDim.x * RMSB_WARPS) {
    bf16x8 xr[NV], gr[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int64_t off = row * COLS + j * 256 + lane * 8;
      xr[j] = *reinterpret_cast<const bf16x8*>(x + off);
      gr[j] = *reinterpret_cast<const bf16x8*>(dy + off);
    }
    const float rs = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      float xv[8], g[8];
      unpack8(xr[j], xv);
      unpack8(gr[j], g);
      float4* dp = reinterpret_cast<float4*>(dw_w + j * 256 + lane * 8);
      const float4* wp = reinterpret_cast<const float4*>(w_s + j * 256 + lane * 8);
      float4 d0 = dp[0], d1 = dp[1];
      const float4 w0 = wp[0], w1 = wp[1];
      float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xh = xv[i] * rs;
        dv[i] += g[i] * xh;
        dot += (g[i] * wv[i]) * xh;
      }
      dp[0] = make_float4(dv[0], dv[1], dv[2], dv[3]);
      dp[1] = make_float4(dv[4], dv[5], dv[6], dv[7]);
    }
    dot = warp_sum(dot) / (float)COLS;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      float xv[8], g[8], o[8];
      unpack8(xr[j], xv);
      unpack8(gr[j], g);
      const float4* wp = reinterpret_cast<const float4*>(w_s + j * 256 + lane * 8);
      const float4 w0 = wp[0], w1 = wp[1];
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = rs * (g[i] * wv[i] - (xv[i] * rs) * dot);
      store8(dx + row * COLS + j * 256 + lane * 8, o);
    }
  }
  __syncthreads();
  for (int c = threadIdx.x * 4; c < COLS; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < RMSB_WARPS; ++k) {
      const float4 v = *reinterpret_cast<const float4*>(rms_smem + COLS * (1 + k) + c);
      acc.x += v.x;
      acc.y += v.y;
      acc.z += v.z;
      acc.w += v.w;
    }
    atomicAdd(reinterpret_cast<float4*>(dw + c), acc);
  }
}

// ---------------------------------------------------------------- QK-Norm + RoPE
// One warp per (token, head); lane l holds elements [4l, 4l+4) of the 128-wide
// head, so the RoPE partner (j <-> j+64) lives in lane l^16.
constexpr int HD = 128;

QB_DEVICE void load4(const bf16* p, float (&v)[4]) {
  uint2 r = *reinterpret_cast<const uint2*>(p);
  float2 a = unpack_bf16x2(r.x), b = unpack_bf16x2(r.y);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
QB_DEVICE void store4(bf16* p, const float (&v)[4]) {
  uint2 r;
  r.x = pack_bf16x2(v[0], v[1]);
  r.y = pack_bf16x2(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = r;
}

struct QkNormRopeParams {
  const bf16* qkv;
  int64_t T, ld_in;
  int hq, hkv;
  const int64_t* positions;
  const float* cos_sin;
  int64_t max_pos;
  const bf16* qw;
  const bf16* kw;
  float eps;
  bf16* out;
  int64_t ld_out;
  bf16* q_out;
  bf16* k_cache;
  bf16* v_cache;
  const int32_t* slots;
  int64_t num_slots;
  float* q_rstd;
  float* k_rstd;
  int* err;
};

// Grid: (T, ceil((hq + 2*hkv) / warps_per_block)).  Heads [0,hq) are q, [hq, hq+hkv)
// k, [hq+hkv, hq+2hkv) v.
__global__ void qk_norm_rope_fwd_kernel(QkNormRopeParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t t = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nheads = p.hq + 2 * p.hkv;
  if (head >= nheads) return;
  const bf16* src = p.qkv + t * p.ld_in + head * HD + lane * 4;
  float v[4];
  load4(src, v);

  int64_t slot = -1;
  if (p.k_cache != nullptr && head >= p.hq) {
    slot = p.slots[t];
    if (slot >= p.num_slots || slot < -1) {
      if (lane == 0) qb_set_err(p.err, QB_DEVERR_SLOT);
      slot = -1;
    }
  }

  if (head >= p.hq + p.hkv) {  // v: copy (and store into the cache)
    const int vh = head - p.hq - p.hkv;
    if (p.out) store4(p.out + t * p.ld_out + head * HD + lane * 4, v);
    if (slot >= 0) store4(p.v_cache + (slot * p.hkv + vh) * HD + lane * 4, v);
    return;
  }
  const bool is_q = head < p.hq;
  // RMSNorm over the 128-wide head, rounded to bf16 as the reference's q_norm/k_norm output.
  float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
  ss = warp_sum(ss);
  const float rstd = rsqrtf(ss / (float)HD + p.eps);
  if (lane == 0) {
    if (is_q && p.q_rstd) p.q_rstd[t * p.hq + head] = rstd;
    if (!is_q && p.k_rstd) p.k_rstd[t * p.hkv + (head - p.hq)] = rstd;
  }
  float wv[4];
  load4((is_q ? p.qw : p.kw) + lane * 4, wv);
  float xn[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) xn[i] = round_bf16((v[i] * rstd) * wv[i]);
  // RoPE, half-split pairing (j, j+64), fp32 internals.
  int64_t pos = p.positions[t];
  if (pos < 0 || pos >= p.max_pos) {
    if (lane == 0) qb_set_err(p.err, QB_DEVERR_SHAPE);
    pos = 0;
  }
  const int j0 = (lane & 15) * 4;
  const float* cs = p.cos_sin + pos * HD;
  float o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, xn[i], 16);
    const float c = cs[j0 + i], s = cs[HD / 2 + j0 + i];
    if (lane < 16) o[i] = xn[i] * c - partner * s;   // x1*c - x2*s
    else o[i] = xn[i] * c + partner * s;             // x2*c + x1*s
  }
  if (p.out) store4(p.out + t * p.ld_out + head * HD + lane * 4, o);
  if (is_q && p.q_out) store4(p.q_out + (t * p.hq + head) * HD + lane * 4, o);
  if (!is_q && slot >= 0) store4(p.k_cache + (slot * p.hkv + (head - p.hq)) * HD + lane * 4, o);
}

// One token per 128-thread block, up to eight blocks per SM: every half-warp (16 lanes x 8
// elements, 16-byte accesses) owns heads h, h+8, h+16, h+24 of the token.  The head rows are
// loaded as packed bf16 before anything that depends on the token's position, so a block has its
// whole row in flight at once and the position / slot loads overlap it; at 64 registers a thread
// eight blocks (eight rows) stay resident per SM.  RoPE partners (j, j+64) sit 8 lanes apart.
// Same rounding points as the warp kernel.
constexpr int QK8_MAXH = 4;  // heads per half-warp held in registers at once (32 heads per pass)

QB_DEVICE float half_warp_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
QB_DEVICE bf16x8 ld_row8(const bf16* p) { return *reinterpret_cast<const bf16x8*>(p); }
QB_DEVICE void st_row8(bf16* p, const bf16x8& r) { *reinterpret_cast<bf16x8*>(p) = r; }
// cos and sin of the eight rotation-table columns jj..jj+7 of one position
QB_DEVICE void load_rot8(const float* cos_sin, int64_t pos, int jj, float (&cv)[8], float (&sv)[8]) {
  const float4* cs4 = reinterpret_cast<const float4*>(cos_sin + pos * HD + jj);
  const float4* sn4 = reinterpret_cast<const float4*>(cos_sin + pos * HD + HD / 2 + jj);
  const float4 c0 = cs4[0], c1 = cs4[1], s0 = sn4[0], s1 = sn4[1];
  cv[0] = c0.x; cv[1] = c0.y; cv[2] = c0.z; cv[3] = c0.w; cv[4] = c1.x; cv[5] = c1.y; cv[6] = c1.z; cv[7] = c1.w;
  sv[0] = s0.x; sv[1] = s0.y; sv[2] = s0.z; sv[3] = s0.w; sv[4] = s1.x; sv[5] = s1.y; sv[6] = s1.z; sv[7] = s1.w;
}

__global__ void __launch_bounds__(128, 8)
qk_norm_rope_fwd8_kernel(QkNormRopeParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t t = blockIdx.x;
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int nheads = p.hq + 2 * p.hkv;
  const bf16* src = p.qkv + t * p.ld_in + l * 8;
  const int64_t pos_in = p.positions[t];
  const int64_t slot_in = p.k_cache != nullptr ? (int64_t)p.slots[t] : -1;
  for (int hc = 0; hc < nheads; hc += 8 * QK8_MAXH) {
    bf16x8 raw[QK8_MAXH];
#pragma unroll
    for (int k = 0; k < QK8_MAXH; ++k) {
      const int h = hc + hw + 8 * k;
      raw[k] = h < nheads ? ld_row8(src + h * HD) : bf16x8{};
    }
    int64_t pos = pos_in;
    if (pos < 0 || pos >= p.max_pos) {
      if (threadIdx.x == 0 && hc == 0) qb_set_err(p.err, QB_DEVERR_SHAPE);
      pos = 0;
    }
    int64_t slot = slot_in;
    if (slot >= p.num_slots || slot < -1) {
      if (threadIdx.x == 0 && hc == 0) qb_set_err(p.err, QB_DEVERR_SLOT);
      slot = -1;
    }
    float cv[8], sv[8];
    load_rot8(p.cos_sin, pos, (l & 7) * 8, cv, sv);
    const bf16x8 qwr = ld_row8(p.qw + l * 8), kwr = ld_row8(p.kw + l * 8);
#pragma unroll
    for (int k = 0; k < QK8_MAXH; ++k) {
      const int h = hc + hw + 8 * k;
      const bool live = h < nheads;
      const bool is_q = h < p.hq, is_v = h >= p.hq + p.hkv;
      float v[8], w[8];
      unpack8(raw[k], v);
      unpack8(is_q ? qwr : kwr, w);
      // RMSNorm over the head (every lane of the warp takes part in the shuffles; dead rows are 0)
      const float ss = half_warp_sum(qk_sumsq8(v));
      const float rstd = qk_rstd(ss, p.eps);
      float xn[8], o[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) xn[i] = round_bf16((v[i] * rstd) * w[i]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, xn[i], 8);
        o[i] = l < 8 ? qk_rope_lo(xn[i], partner, cv[i], sv[i]) : qk_rope_hi(xn[i], partner, cv[i], sv[i]);
      }
      if (!live) continue;
      if (is_v) {  // v: copied bit for bit (and stored into the cache)
        if (p.out) st_row8(p.out + t * p.ld_out + h * HD + l * 8, raw[k]);
        if (slot >= 0) st_row8(p.v_cache + (slot * p.hkv + (h - p.hq - p.hkv)) * HD + l * 8, raw[k]);
        continue;
      }
      if (l == 0) {
        if (is_q && p.q_rstd) p.q_rstd[t * p.hq + h] = rstd;
        if (!is_q && p.k_rstd) p.k_rstd[t * p.hkv + (h - p.hq)] = rstd;
      }
      if (p.out) store8(p.out + t * p.ld_out + h * HD + l * 8, o);
      if (is_q && p.q_out) store8(p.q_out + (t * p.hq + h) * HD + l * 8, o);
      if (!is_q && slot >= 0) store8(p.k_cache + (slot * p.hkv + (h - p.hq)) * HD + l * 8, o);
    }
  }
}

struct QkNormRopeBwdParams {
  const bf16* dout;
  const bf16* qkv;
  int64_t T, ld;
  int hq, hkv;
  const int64_t* positions;
  const float* cos_sin;
  int64_t max_pos;
  const bf16* qw;
  const bf16* kw;
  const float* q_rstd;
  const float* k_rstd;
  int rope_grad;
  bf16* dqkv;
  float* dqw;
  float* dkw;
  int* err;
};

// Grid: (ceil(T / TOK_PER_BLOCK)), block = 32*(hq+2hkv) threads?  Too many for 32 heads,
// so each block handles TOK_PER_BLOCK tokens with 8 warps striding over (token, head)
// pairs; norm-weight grads are folded in shared memory, one atomic per column per block.
constexpr int QKB_TOK = 16;
__global__ void qk_norm_rope_bwd_kernel(QkNormRopeBwdParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ float dqw_s[HD], dkw_s[HD];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int c = threadIdx.x; c < HD; c += blockDim.x) { dqw_s[c] = 0.f; dkw_s[c] = 0.f; }
  __syncthreads();
  const int nheads = p.hq + 2 * p.hkv;
  float dq_acc[4] = {0, 0, 0, 0}, dk_acc[4] = {0, 0, 0, 0};
  const int64_t t0 = (int64_t)blockIdx.x * QKB_TOK;
  for (int item = wid; item < QKB_TOK * nheads; item += nw) {
    const int64_t t = t0 + item / nheads;
    const int head = item % nheads;
    if (t >= p.T) break;
    const int64_t off = t * p.ld + head * HD + lane * 4;
    float g[4];
    load4(p.dout + off, g);
    if (head >= p.hq + p.hkv) {  // v passes through
      store4(p.dqkv + off, g);
      continue;
    }
    if (!p.rope_grad) {
      float z[4] = {0, 0, 0, 0};
      store4(p.dqkv + off, z);
      continue;
    }
    const bool is_q = head < p.hq;
    int64_t pos = p.positions[t];
    if (pos < 0 || pos >= p.max_pos) {
      if (lane == 0) qb_set_err(p.err, QB_DEVERR_SHAPE);
      pos = 0;
    }
    const int j0 = (lane & 15) * 4;
    const float* cs = p.cos_sin + pos * HD;
    // Inverse rotation: dx1 = dy1*c + dy2*s, dx2 = dy2*c - dy1*s.
    float dxn[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, g[i], 16);
      const float c = cs[j0 + i], s = cs[HD / 2 + j0 + i];
      dxn[i] = (lane < 16) ? (g[i] * c + partner * s) : (g[i] * c - partner * s);
    }
    float x[4], wv[4];
    load4(p.qkv + off, x);
    load4((is_q ? p.qw : p.kw) + lane * 4, wv);
    const float rs = is_q ? p.q_rstd[t * p.hq + head] : p.k_rstd[t * p.hkv + (head - p.hq)];
    float dot = 0.f, xh[4], gx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xh[i] = x[i] * rs;
      gx[i] = dxn[i] * wv[i];
      dot += gx[i] * xh[i];
      if (is_q) dq_acc[i] += dxn[i] * xh[i];
      else dk_acc[i] += dxn[i] * xh[i];
    }
    dot = warp_sum(dot) / (float)HD;
    float dx[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) dx[i] = rs * (gx[i] - xh[i] * dot);
    store4(p.dqkv + off, dx);
  }
  if (p.rope_grad) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      atomicAdd(&dqw_s[lane * 4 + i], dq_acc[i]);
      atomicAdd(&dkw_s[lane * 4 + i], dk_acc[i]);
    }
  }
  __syncthreads();
  if (p.rope_grad) {
    for (int c = threadIdx.x; c < HD; c += blockDim.x) {
      atomicAdd(p.dqw + c, dqw_s[c]);
      atomicAdd(p.dkw + c, dkw_s[c]);
    }
  }
}

// The backward with 16-byte accesses: a grid-stride loop over tokens, 128 threads a block and up
// to four blocks per SM, every half-warp owning heads h, h+8, h+16, h+24 of the current token.
// All of a token's loads (incoming gradients, raw q/k rows, their saved rstd) are issued before
// the rotation table that depends on its position, so each block keeps a whole token in flight.
// Norm-weight gradients are folded per lane across the block's tokens, then over the block in
// shared memory, then one global atomic per column.  When dqkv == dout the v columns, whose
// gradient passes through unchanged, are left in place.  Same arithmetic as
// qk_norm_rope_bwd_kernel.
constexpr int QKB8_BLOCKS_PER_SM = 4;
__global__ void __launch_bounds__(128, QKB8_BLOCKS_PER_SM)
qk_norm_rope_bwd8_kernel(QkNormRopeBwdParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ float dqw_s[HD], dkw_s[HD];
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  for (int c = threadIdx.x; c < HD; c += blockDim.x) {
    dqw_s[c] = 0.f;
    dkw_s[c] = 0.f;
  }
  __syncthreads();
  const int nheads = p.hq + 2 * p.hkv;
  const bool in_place = p.dqkv == p.dout;
  float dq_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0}, dk_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const bf16x8 qwr = ld_row8(p.qw + l * 8), kwr = ld_row8(p.kw + l * 8);
  for (int64_t t = blockIdx.x; t < p.T; t += gridDim.x) {
    const int64_t row = t * p.ld + l * 8;
    const int64_t pos_in = p.positions[t];
    for (int hc = 0; hc < nheads; hc += 8 * QK8_MAXH) {
      bf16x8 g[QK8_MAXH], x[QK8_MAXH];
      float rs[QK8_MAXH];
#pragma unroll
      for (int k = 0; k < QK8_MAXH; ++k) {
        const int h = hc + hw + 8 * k;
        const bool live = h < nheads, is_q = h < p.hq;
        const bool norm = live && h < p.hq + p.hkv && p.rope_grad;
        g[k] = live ? ld_row8(p.dout + row + h * HD) : bf16x8{};
        x[k] = norm ? ld_row8(p.qkv + row + h * HD) : bf16x8{};
        rs[k] = norm ? (is_q ? p.q_rstd[t * p.hq + h] : p.k_rstd[t * p.hkv + (h - p.hq)]) : 0.f;
      }
      int64_t pos = pos_in;
      if (pos < 0 || pos >= p.max_pos) {
        if (l == 0) qb_set_err(p.err, QB_DEVERR_SHAPE);
        pos = 0;
      }
      float cv[8], sv[8];
      load_rot8(p.cos_sin, pos, (l & 7) * 8, cv, sv);
#pragma unroll
      for (int k = 0; k < QK8_MAXH; ++k) {
        const int h = hc + hw + 8 * k;
        const bool live = h < nheads;
        const bool is_v = h >= p.hq + p.hkv, is_q = h < p.hq;
        float gv[8], xv[8], w[8];
        unpack8(g[k], gv);
        unpack8(x[k], xv);
        unpack8(is_q ? qwr : kwr, w);
        // inverse rotation: dx1 = dy1*c + dy2*s, dx2 = dy2*c - dy1*s
        float dxn[8], xh[8], gx[8];
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float partner = __shfl_xor_sync(0xffffffffu, gv[i], 8);
          dxn[i] = l < 8 ? gv[i] * cv[i] + partner * sv[i] : gv[i] * cv[i] - partner * sv[i];
          xh[i] = xv[i] * rs[k];
          gx[i] = dxn[i] * w[i];
          dot += gx[i] * xh[i];
        }
        dot = half_warp_sum(dot) / (float)HD;
        if (!live) continue;
        if (is_v) {  // v passes through
          if (!in_place) st_row8(p.dqkv + row + h * HD, g[k]);
          continue;
        }
        if (!p.rope_grad) {  // the reference's RoPE is invisible to autograd: q/k get no gradient
          st_row8(p.dqkv + row + h * HD, bf16x8{});
          continue;
        }
        float dx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (is_q) dq_acc[i] += dxn[i] * xh[i];
          else dk_acc[i] += dxn[i] * xh[i];
          dx[i] = rs[k] * (gx[i] - xh[i] * dot);
        }
        store8(p.dqkv + row + h * HD, dx);
      }
    }
  }
  if (p.rope_grad) {
    // lanes l and l + 16 of a warp hold the same columns
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dq_acc[i] += __shfl_xor_sync(0xffffffffu, dq_acc[i], 16);
      dk_acc[i] += __shfl_xor_sync(0xffffffffu, dk_acc[i], 16);
    }
    if ((threadIdx.x & 16) == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        atomicAdd(&dqw_s[l * 8 + i], dq_acc[i]);
        atomicAdd(&dkw_s[l * 8 + i], dk_acc[i]);
      }
    }
  }
  __syncthreads();
  if (p.rope_grad) {
    for (int c = threadIdx.x; c < HD; c += blockDim.x) {
      atomicAdd(p.dqw + c, dqw_s[c]);
      atomicAdd(p.dkw + c, dkw_s[c]);
    }
  }
}

// ---------------------------------------------------------------- SwiGLU / adds
QB_DEVICE float silu_f(float g) { return qb_silu(g); }

// One row per 128-thread block; a thread's (up to SILU_MAXV) 16-byte vectors of the row are all
// loaded before any is used.  Rows are the block index, so no per-element index division.
constexpr int SILU_MAXV = 3;
__global__ void __launch_bounds__(128, 8)
silu_mul_fwd_kernel(const bf16* __restrict__ gu, int64_t T, int64_t I, bf16* __restrict__ out) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t row = blockIdx.x;
  const bf16* g_row = gu + row * 2 * I;
  const bf16* u_row = g_row + I;
  for (int64_t c0 = threadIdx.x * 8; c0 < I; c0 += 128 * 8 * SILU_MAXV) {
    bf16x8 gr[SILU_MAXV], ur[SILU_MAXV];
#pragma unroll
    for (int k = 0; k < SILU_MAXV; ++k) {
      const int64_t c = c0 + k * 128 * 8;
      if (c < I) {
        gr[k] = *reinterpret_cast<const bf16x8*>(g_row + c);
        ur[k] = *reinterpret_cast<const bf16x8*>(u_row + c);
      }
    }
#pragma unroll
    for (int k = 0; k < SILU_MAXV; ++k) {
      const int64_t c = c0 + k * 128 * 8;
      if (c >= I) break;
      bf16x8 o;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 g = unpack_bf16x2(gr[k].u[i]), u = unpack_bf16x2(ur[k].u[i]);
        o.u[i] = pack_bf16x2(silu_f(g.x) * u.x, silu_f(g.y) * u.y);
      }
      *reinterpret_cast<bf16x8*>(out + row * I + c) = o;
    }
  }
}

__global__ void __launch_bounds__(128, 5)
silu_mul_bwd_kernel(const bf16* __restrict__ dout, const bf16* __restrict__ gu, int64_t T, int64_t I,
                    bf16* __restrict__ dgu) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t row = blockIdx.x;
  const bf16* g_row = gu + row * 2 * I;
  const bf16* u_row = g_row + I;
  for (int64_t c0 = threadIdx.x * 8; c0 < I; c0 += 128 * 8 * SILU_MAXV) {
    bf16x8 gr[SILU_MAXV], ur[SILU_MAXV], dr[SILU_MAXV];
#pragma unroll
    for (int k = 0; k < SILU_MAXV; ++k) {
      const int64_t c = c0 + k * 128 * 8;
      if (c < I) {
        gr[k] = *reinterpret_cast<const bf16x8*>(g_row + c);
        ur[k] = *reinterpret_cast<const bf16x8*>(u_row + c);
        dr[k] = *reinterpret_cast<const bf16x8*>(dout + row * I + c);
      }
    }
#pragma unroll
    for (int k = 0; k < SILU_MAXV; ++k) {
      const int64_t c = c0 + k * 128 * 8;
      if (c >= I) break;
      float g[8], u[8], d[8], dg[8], du[8];
      unpack8(gr[k], g);
      unpack8(ur[k], u);
      unpack8(dr[k], d);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float sg = 1.0f / (1.0f + expf(-g[j]));
        du[j] = d[j] * (g[j] * sg);
        dg[j] = d[j] * u[j] * sg * (1.0f + g[j] * (1.0f - sg));
      }
      store8(dgu + row * 2 * I + c, dg);
      store8(dgu + row * 2 * I + I + c, du);
    }
  }
}

__global__ void add_bf16_kernel(const bf16* __restrict__ a, const bf16* __restrict__ b,
                                bf16* __restrict__ out, int64_t n) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t nvec = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    float x[8], y[8];
    load8(a + i * 8, x);
    load8(b + i * 8, y);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] += y[k];
    store8(out + i * 8, x);
  }
  // scalar tail
  const int64_t tail0 = nvec * 8;
  for (int64_t i = tail0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f2bf(bf2f(a[i]) + bf2f(b[i]));
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, int64_t n) {
  qb_pdl_trigger();
  qb_pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = f2bf(src[i]);
}
__global__ void accumulate_bf16_kernel(const bf16* __restrict__ src, float* __restrict__ acc, int64_t n) {
  qb_pdl_trigger();
  qb_pdl_wait();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    acc[i] += bf2f(src[i]);
}

inline int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  const int64_t cap = 148 * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

// ================================================================ C ABI
extern "C" int qb_embedding_fwd(const int64_t* ids, int64_t n, const void* table, int64_t vocab,
                                int64_t hidden, void* out, int* err, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0 && vocab > 0 && hidden > 0 && hidden % 8 == 0);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(ids && table && out && aligned16(table) && aligned16(out));
  const int wpb = 8;
  return qb_launch(embedding_fwd_kernel, dim3((unsigned)((n + wpb - 1) / wpb)), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, ids, n, (const bf16*)table, vocab, hidden, (bf16*)out, err);
}

extern "C" int qb_embedding_bwd(const int64_t* ids, int64_t n, const void* dout, int64_t vocab,
                                int64_t hidden, float* dtable, int* err, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0 && vocab > 0 && hidden > 0 && hidden % 8 == 0);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(ids && dout && dtable && aligned16(dout));
  const int wpb = 8;
  return qb_launch(embedding_bwd_kernel, dim3((unsigned)((n + wpb - 1) / wpb)), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, ids, n, (const bf16*)dout, vocab, hidden, dtable, err);
}

#define QB_NV_DISPATCH(cols, KERNEL_CALL)  \
  switch ((cols) / 256) {                  \
    case 1: { constexpr int NV = 1; KERNEL_CALL; break; } \
    case 2: { constexpr int NV = 2; KERNEL_CALL; break; } \
    case 4: { constexpr int NV = 4; KERNEL_CALL; break; } \
    case 8: { constexpr int NV = 8; KERNEL_CALL; break; } \
    default: return QB_ERR_UNSUPPORTED;    \
  }

extern "C" int qb_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows,
                              int64_t cols, float eps, qb_stream_t stream) {
  QB_CHECK_ARG(rows >= 0 && cols > 0 && cols % 256 == 0);
  if (rows == 0) return QB_OK;
  QB_CHECK_ARG(x && w && y && aligned16(x) && aligned16(w) && aligned16(y));
  const int wpb = 8;
  const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
  int st = QB_OK;
  QB_NV_DISPATCH(cols, (st = qb_launch(rmsnorm_fwd_kernel<NV>, dim3(grid), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, (const bf16*)x, (const bf16*)w, (bf16*)y, rstd, rows, eps)));
  return st;
}

extern "C" int qb_add_rmsnorm_fwd(const void* x, void* residual, const void* w, void* y,
                                  int64_t rows, int64_t cols, float eps, qb_stream_t stream) {
  QB_CHECK_ARG(rows >= 0 && cols > 0 && cols % 256 == 0);
  if (rows == 0) return QB_OK;
  QB_CHECK_ARG(x && residual && w && y && aligned16(x) && aligned16(residual) && aligned16(w) &&
               aligned16(y));
  const int wpb = 8;
  const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
  int st = QB_OK;
  QB_NV_DISPATCH(cols, (st = qb_launch(add_rmsnorm_fwd_kernel<NV>, dim3(grid), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, (const bf16*)x, (bf16*)residual, (const bf16*)w, (bf16*)y, rows, eps)));
  return st;
}

extern "C" int qb_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd,
                              void* dx, float* dw, int64_t rows, int64_t cols, qb_stream_t stream) {
  QB_CHECK_ARG(rows >= 0 && cols > 0 && cols % 256 == 0);
  if (rows == 0) return QB_OK;
  QB_CHECK_ARG(dy && x && w && rstd && dx && dw && aligned16(dy) && aligned16(x) &&
               aligned16(w) && aligned16(dx));
  QB_CHECK_ARG((reinterpret_cast<uintptr_t>(dw) & 15) == 0);  // 16-byte atomic adds
  int64_t g = (rows + RMSB_WARPS - 1) / RMSB_WARPS;
  if (g > 148 * 3) g = 148 * 3;  // one wave of resident blocks; warps stride over the rows
  const size_t smem = (1 + RMSB_WARPS) * (size_t)cols * sizeof(float);
  int st = QB_OK;
  QB_NV_DISPATCH(cols, (st = qb_launch(rmsnorm_bwd_kernel<NV>, dim3((unsigned)g), dim3(RMSB_WARPS * 32), smem, (cudaStream_t)stream, 1, (const bf16*)dy, (const bf16*)x, (const bf16*)w, rstd, (bf16*)dx, dw,
                           rows)));
  return st;
}

extern "C" int qb_qk_norm_rope_fwd(const void* qkv, int64_t T, int64_t ld_in, int hq, int hkv,
                                   int D, const int64_t* positions, const float* cos_sin,
                                   int64_t max_pos, const void* q_norm_w, const void* k_norm_w,
                                   float eps, void* out, int64_t ld_out, void* q_out,
                                   void* k_cache, void* v_cache, const int32_t* slot_mapping,
                                   int64_t num_slots, float* q_rstd, float* k_rstd, int* err,
                                   qb_stream_t stream) {
  QB_CHECK_ARG(T >= 0 && hq > 0 && hkv > 0);
  if (D != HD) return QB_ERR_UNSUPPORTED;
  if (T == 0) return QB_OK;
  QB_CHECK_ARG(qkv && positions && cos_sin && q_norm_w && k_norm_w && max_pos > 0);
  QB_CHECK_ARG(ld_in >= (int64_t)(hq + 2 * hkv) * HD && ld_in % 4 == 0);
  QB_CHECK_ARG(out == nullptr || (ld_out >= (int64_t)(hq + 2 * hkv) * HD && ld_out % 4 == 0));
  QB_CHECK_ARG((k_cache == nullptr) == (v_cache == nullptr));
  QB_CHECK_ARG(k_cache == nullptr || (slot_mapping && num_slots > 0));
  QkNormRopeParams p{(const bf16*)qkv, T, ld_in, hq, hkv, positions, cos_sin, max_pos,
                     (const bf16*)q_norm_w, (const bf16*)k_norm_w, eps, (bf16*)out, ld_out,
                     (bf16*)q_out, (bf16*)k_cache, (bf16*)v_cache, slot_mapping, num_slots,
                     q_rstd, k_rstd, err};
  const bool vec16 = aligned16(qkv) && ld_in % 8 == 0 && (out == nullptr || (aligned16(out) && ld_out % 8 == 0)) &&
                     (q_out == nullptr || aligned16(q_out)) && (k_cache == nullptr || (aligned16(k_cache) &&
                     aligned16(v_cache))) && aligned16(q_norm_w) && aligned16(k_norm_w) && aligned16(cos_sin);
  if (vec16) {  // 16-byte accesses, one token per block
    return qb_launch(qk_norm_rope_fwd8_kernel, dim3((unsigned)T), dim3(128), 0, (cudaStream_t)stream, 1, p);
  }
  const int wpb = 8;
  dim3 grid((unsigned)T, (unsigned)((hq + 2 * hkv + wpb - 1) / wpb));
  return qb_launch(qk_norm_rope_fwd_kernel, dim3(grid), dim3(wpb * 32), 0, (cudaStream_t)stream, 1, p);
}

extern "C" int qb_qk_norm_rope_bwd(const void* dout, const void* qkv, int64_t T, int64_t ld,
                                   int hq, int hkv, int D, const int64_t* positions,
                                   const float* cos_sin, int64_t max_pos, const void* q_norm_w,
                                   const void* k_norm_w, const float* q_rstd, const float* k_rstd,
                                   int rope_grad, void* dqkv, float* dq_norm_w, float* dk_norm_w,
                                   int* err, qb_stream_t stream) {
  QB_CHECK_ARG(T >= 0 && hq > 0 && hkv > 0);
  if (D != HD) return QB_ERR_UNSUPPORTED;
  if (T == 0) return QB_OK;
  QB_CHECK_ARG(dout && qkv && dqkv && positions && cos_sin && ld % 4 == 0 &&
               ld >= (int64_t)(hq + 2 * hkv) * HD);
  QB_CHECK_ARG(!rope_grad || (q_norm_w && k_norm_w && q_rstd && k_rstd && dq_norm_w && dk_norm_w));
  QkNormRopeBwdParams p{(const bf16*)dout, (const bf16*)qkv, T, ld, hq, hkv, positions, cos_sin,
                        max_pos, (const bf16*)q_norm_w, (const bf16*)k_norm_w, q_rstd, k_rstd,
                        rope_grad, (bf16*)dqkv, dq_norm_w, dk_norm_w, err};
  const unsigned grid = (unsigned)((T + QKB_TOK - 1) / QKB_TOK);
  const bool vec16 = aligned16(dout) && aligned16(qkv) && aligned16(dqkv) && ld % 8 == 0 && aligned16(cos_sin) &&
                     (!rope_grad || (aligned16(q_norm_w) && aligned16(k_norm_w)));
  if (vec16 && q_norm_w && k_norm_w) {
    const int64_t cap = 148 * QKB8_BLOCKS_PER_SM;  // one wave of resident blocks; the kernel strides over tokens
    const int64_t g8 = T < cap ? T : cap;
    return qb_launch(qk_norm_rope_bwd8_kernel, dim3((unsigned)g8), dim3(128), 0, (cudaStream_t)stream, 1, p);
  }
  QB_CHECK_ARG(dout != dqkv);  // the warp kernel does not handle aliasing
  return qb_launch(qk_norm_rope_bwd_kernel, dim3(grid), dim3(256), 0, (cudaStream_t)stream, 1, p);
}

extern "C" int qb_silu_mul_fwd(const void* gate_up, int64_t T, int64_t I, void* out,
                               qb_stream_t stream) {
  QB_CHECK_ARG(T >= 0 && T < (int64_t)1 << 31 && I > 0 && I % 8 == 0);
  if (T == 0) return QB_OK;
  QB_CHECK_ARG(gate_up && out && aligned16(gate_up) && aligned16(out));
  return qb_launch(silu_mul_fwd_kernel, dim3((unsigned)T), dim3(128), 0, (cudaStream_t)stream, 1, (const bf16*)gate_up, T, I, (bf16*)out);
}

extern "C" int qb_silu_mul_bwd(const void* dout, const void* gate_up, int64_t T, int64_t I,
                               void* dgate_up, qb_stream_t stream) {
  QB_CHECK_ARG(T >= 0 && T < (int64_t)1 << 31 && I > 0 && I % 8 == 0);
  if (T == 0) return QB_OK;
  QB_CHECK_ARG(dout && gate_up && dgate_up && aligned16(dout) && aligned16(gate_up) &&
               aligned16(dgate_up));
  return qb_launch(silu_mul_bwd_kernel, dim3((unsigned)T), dim3(128), 0, (cudaStream_t)stream, 1, (const bf16*)dout, (const bf16*)gate_up, T, I, (bf16*)dgate_up);
}

extern "C" int qb_add_bf16(const void* a, const void* b, void* out, int64_t n, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(a && b && out && aligned16(a) && aligned16(b) && aligned16(out));
  return qb_launch(add_bf16_kernel, dim3(grid_for(n / 8 + 1, 256)), dim3(256), 0, (cudaStream_t)stream, 1, (const bf16*)a, (const bf16*)b, (bf16*)out, n);
}

extern "C" int qb_f32_to_bf16(const float* src, void* dst, int64_t n, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(src && dst);
  return qb_launch(f32_to_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, (cudaStream_t)stream, 1, src, (bf16*)dst, n);
}

extern "C" int qb_accumulate_bf16(const void* src, float* acc, int64_t n, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(src && acc);
  return qb_launch(accumulate_bf16_kernel, dim3(grid_for(n, 256)), dim3(256), 0, (cudaStream_t)stream, 1, (const bf16*)src, acc, n);
}
