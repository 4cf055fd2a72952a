// Sampling, token log-probabilities and the fused GRPO loss.
//
//   qb_sample        temperature / top-k sampling (inverse CDF over the full row,
//                    Gumbel-max over a top-k set) with the sampled token's log-prob
//                    (qwen3_naive.py:1632-1650)
//   qb_logprob_fwd   log_softmax + gather from bf16 logits (qwen3_grpo_train.py:48-52)
//   qb_logprob_bwd   its gradient w.r.t. the logits, in place
//   qb_grpo_*        advantages, clipped surrogate, k3 KL, masked token mean and
//                    the gradient w.r.t. the new log-probs (qwen3_grpo_train.py:162-199)
//
// Row kernels use one CTA per row and 16-byte loads.  Reductions that span CTAs
// write per-CTA partials to a caller workspace; the last CTA to finish (ticket
// counter, no spinning) folds them in a fixed order, so results are
// deterministic run to run.
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace {

struct alignas(16) bf16x8 {
  uint32_t u[4];
};

QB_DEVICE void unpack8(const bf16x8& r, float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = unpack_bf16x2(r.u[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Order-preserving 16-bit key of a bf16 value (larger value -> larger key).
QB_DEVICE uint32_t bf16_key(uint32_t bits16) {
  return (bits16 & 0x8000u) ? (~bits16 & 0xFFFFu) : (bits16 | 0x8000u);
}

// ---------------------------------------------------------------- Philox4x32-10
// Counter-based generator of Salmon, Moraes, Dror & Shaw, "Parallel random
// numbers: as easy as 1, 2, 3" (SC'11): ten rounds of two 32x32->64 multiplies
// with the published multipliers and Weyl key increments.
struct U4 {
  uint32_t x, y, z, w;
};
QB_DEVICE U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = M0 * c.x, hi0 = __umulhi(M0, c.x);
    const uint32_t lo1 = M1 * c.z, hi1 = __umulhi(M1, c.z);
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return c;
}
// Uniform in the open interval (0, 1) from the top 24 bits.
QB_DEVICE float u01(uint32_t v) { return ((float)(v >> 8) + 0.5f) * (1.0f / 16777216.0f); }
QB_DEVICE float gumbel(uint32_t v) { return -logf(-logf(u01(v))); }

// Gumbel noise for columns [c8, c8+8) of one row.
QB_DEVICE void gumbel8(uint64_t seed, uint64_t offset, int64_t row, int64_t c8, float (&g)[8]) {
  const uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint64_t q = (uint64_t)(c8 / 4 + h);
    U4 r = philox4x32_10(U4{(uint32_t)q, (uint32_t)row, (uint32_t)offset, (uint32_t)(offset >> 32)}, k0, k1);
    g[4 * h + 0] = gumbel(r.x);
    g[4 * h + 1] = gumbel(r.y);
    g[4 * h + 2] = gumbel(r.z);
    g[4 * h + 3] = gumbel(r.w);
  }
}

// ---------------------------------------------------------------- block reductions
struct MS {  // online log-sum-exp state
  float m, s;
};
QB_DEVICE MS ms_merge(MS a, MS b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return MS{m, 0.f};
  return MS{m, a.s * expf(a.m - m) + b.s * expf(b.m - m)};
}
QB_DEVICE void ms_add(MS& a, float x) {
  if (x > a.m) {
    a.s = (a.m == -INFINITY) ? 1.f : a.s * expf(a.m - x) + 1.f;
    a.m = x;
  } else if (x != -INFINITY) {
    a.s += expf(x - a.m);
  }
}
struct AM {  // argmax with lowest-index tie break
  float v;
  int64_t i;
};
QB_DEVICE AM am_merge(AM a, AM b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

template <int NT>
QB_DEVICE MS block_ms(MS v, MS* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)};
    v = ms_merge(v, other);
  }
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  if (wid == 0) {
    v = (lane < NT / 32) ? sh[lane] : MS{-INFINITY, 0.f};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      MS other{__shfl_xor_sync(0xffffffffu, v.m, o), __shfl_xor_sync(0xffffffffu, v.s, o)};
      v = ms_merge(v, other);
    }
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  MS r = sh[0];
  __syncthreads();
  return r;
}

template <int NT>
QB_DEVICE AM block_am(AM v, AM* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    AM other{__shfl_xor_sync(0xffffffffu, v.v, o), (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v.i, o)};
    v = am_merge(v, other);
  }
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  if (wid == 0) {
    v = (lane < NT / 32) ? sh[lane] : AM{-INFINITY, INT64_MAX};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      AM other{__shfl_xor_sync(0xffffffffu, v.v, o), (int64_t)__shfl_xor_sync(0xffffffffu, (long long)v.i, o)};
      v = am_merge(v, other);
    }
    if (lane == 0) sh[0] = v;
  }
  __syncthreads();
  AM r = sh[0];
  __syncthreads();
  return r;
}

// Exclusive prefix sum over the block (NT threads) of a small int; returns the block total in *total.
template <int NT>
QB_DEVICE int block_excl_scan(int v, int* sh, int* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) sh[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int w = (lane < NT / 32) ? sh[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < NT / 32) sh[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const int before = (wid == 0) ? 0 : sh[wid - 1];
  *total = sh[NT / 32 - 1];
  __syncthreads();
  return before + x - v;
}

// Exclusive prefix sum over the block of a float; the block total goes to *total.
template <int NT>
QB_DEVICE float block_excl_scan_f(float v, float* sh, float* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) sh[wid] = x;
  __syncthreads();
  if (wid == 0) {
    float w = (lane < NT / 32) ? sh[lane] : 0.f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < NT / 32) sh[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const float before = (wid == 0) ? 0.f : sh[wid - 1];
  *total = sh[NT / 32 - 1];
  __syncthreads();
  return before + x - v;
}

template <int NT>
QB_DEVICE float block_max_f(float v, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  float r = sh[0];
#pragma unroll 1
  for (int w = 1; w < NT / 32; ++w) r = fmaxf(r, sh[w]);
  __syncthreads();
  return r;
}

// Uniform in the open interval (0, 1) with 53 random bits, one per (row, stream position).
QB_DEVICE double row_uniform(uint64_t seed, uint64_t offset, int64_t row) {
  const U4 r = philox4x32_10(U4{0xFFFFFFFFu, (uint32_t)row, (uint32_t)offset, (uint32_t)(offset >> 32)},
                             (uint32_t)seed, (uint32_t)(seed >> 32));
  const uint64_t a = r.x >> 5, b = r.y >> 6;  // 27 + 26 bits
  return ((double)(a * 67108864ull + b) + 0.5) * (1.0 / 9007199254740992.0);
}

// ---------------------------------------------------------------- sampling
constexpr int SNT = 512;

struct SampleParams {
  const bf16* logits;
  int64_t V, ld;
  float temperature;
  int top_k;
  uint64_t seed;
  const uint64_t* offset;
  int64_t* tokens;
  float* logp;
  int* err;
};

__global__ void __launch_bounds__(SNT, 4) sample_kernel(SampleParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ MS sh_ms[32];
  __shared__ AM sh_am[32];
  __shared__ int hist[256];
  __shared__ int sh_scan[32];
  __shared__ int sh_sel[4];
  const int64_t row = blockIdx.x;
  const bf16* lrow = p.logits + row * p.ld;
  const int64_t nvec = p.V / 8;
  // rng_state = {counter, seed mix}, read at run time so graph replays draw fresh noise.
  const uint64_t off = p.offset ? p.offset[0] : 0ull;
  const uint64_t seed = p.seed ^ (p.offset ? p.offset[1] : 0ull);
  const int k = p.top_k;

  // --------------------------------------------------------- greedy (top_k == 1)
  if (k == 1) {
    AM best{-INFINITY, INT64_MAX};
    for (int64_t v = threadIdx.x; v < nvec; v += SNT) {
      bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
      float x[8];
      unpack8(r, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) best = am_merge(best, AM{x[i], v * 8 + i});
    }
    best = block_am<SNT>(best, sh_am);
    if (threadIdx.x == 0) {
      const bool ok = best.i >= 0 && best.i < p.V;  // false only for an all-NaN row
      if (!ok) qb_set_err(p.err, QB_DEVERR_TOKEN);
      p.tokens[row] = ok ? best.i : 0;
      p.logp[row] = 0.f;
    }
    return;
  }

  const bool use_topk = k > 1 && k < p.V;
  // --------------------------------------------------------- all V entries kept: inverse-CDF sampling
  // The row is visited in a fixed order (thread t, then its vectors t, t + SNT, ... in turn, then
  // the 8 entries of a vector).  One pass accumulates each thread's share of the softmax mass in
  // the log2 domain (running max, one exp2 per entry); a block scan of the shares places the row's
  // uniform draw u * S in one thread's range, and that thread walks its entries again to find the
  // token whose cumulative mass first exceeds it.  One uniform per row; no per-entry noise.
  if (!use_topk) {
    __shared__ float sh_f[32];
    __shared__ int sh_pick[2];
    const float k2 = 1.4426950408889634f / p.temperature;  // x / T in log2 units = x * k2
    float m = -INFINITY, sacc = 0.f;
    for (int64_t v = threadIdx.x; v < nvec; v += SNT) {
      const bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
      float x[8];
      unpack8(r, x);
      float mx = x[0];
#pragma unroll
      for (int i = 1; i < 8; ++i) mx = fmaxf(mx, x[i]);
      const float mn = fmaxf(m, mx * k2);
      if (mn == -INFINITY) continue;
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc += exp2f(fmaf(x[i], k2, -mn));
      sacc = sacc * exp2f(m - mn) + acc;
      m = mn;
    }
    const float M = block_max_f<SNT>(m, sh_f);
    const float w = (m == -INFINITY || M == -INFINITY) ? 0.f : sacc * exp2f(m - M);
    float S = 0.f;
    const float before = block_excl_scan_f<SNT>(w, sh_f, &S);
    const float target = (float)(row_uniform(seed, off, row) * (double)S);
    if (threadIdx.x == 0) {
      sh_pick[0] = SNT;  // lowest thread whose range holds the target
      sh_pick[1] = -1;   // highest thread with mass (rounding fallback)
    }
    __syncthreads();
    if (w > 0.f) {
      if (target >= before && target < before + w) atomicMin(&sh_pick[0], (int)threadIdx.x);
      atomicMax(&sh_pick[1], (int)threadIdx.x);
    }
    __syncthreads();
    const int t_pick = sh_pick[0] < SNT ? sh_pick[0] : sh_pick[1];
    if ((int)threadIdx.x == t_pick) {
      const float rem = target - before;
      float acc = 0.f;
      int64_t tok = -1, last = -1;
      for (int64_t v = threadIdx.x; v < nvec && tok < 0; v += SNT) {
        const bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
        float x[8];
        unpack8(r, x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float e = exp2f(fmaf(x[i], k2, -M));
          if (e > 0.f) last = v * 8 + i;
          acc += e;
          if (tok < 0 && e > 0.f && acc > rem) tok = v * 8 + i;
        }
      }
      if (tok < 0) tok = last;  // the target fell past this thread's re-summed mass by rounding
      p.tokens[row] = tok;
      p.logp[row] = (fmaf(bf2f(lrow[tok]), k2, -M) - log2f(S)) * 0.6931471805599453f;
    }
    if (t_pick < 0 && threadIdx.x == 0) {  // no finite logit in the row
      qb_set_err(p.err, QB_DEVERR_TOKEN);
      p.tokens[row] = 0;
      p.logp[row] = 0.f;
    }
    return;
  }

  // --------------------------------------------------------- top-k threshold (radix select on bf16 keys)
  uint32_t thr_key = 0;  // keep keys > thr_key, plus the first need_eq keys == thr_key
  int need_eq = 0;
  {
    for (int i = threadIdx.x; i < 256; i += SNT) hist[i] = 0;
    __syncthreads();
    // logits of similar size share a high byte: lanes with equal bins add once (warp aggregated)
    for (int64_t v = threadIdx.x; v < nvec; v += SNT) {
      bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
      const unsigned act = __activemask();
      const int lane = threadIdx.x & 31;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int bin = (int)(bf16_key((i & 1) ? (r.u[i >> 1] >> 16) : (r.u[i >> 1] & 0xFFFFu)) >> 8);
        const unsigned peers = __match_any_sync(act, bin);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int cum = 0, bin = 255;
      for (; bin > 0; --bin) {
        if (cum + hist[bin] >= k) break;
        cum += hist[bin];
      }
      sh_sel[0] = bin;
      sh_sel[1] = cum;  // count of keys with a larger high byte
    }
    __syncthreads();
    const int hb = sh_sel[0], above = sh_sel[1];
    for (int i = threadIdx.x; i < 256; i += SNT) hist[i] = 0;
    __syncthreads();
    for (int64_t v = threadIdx.x; v < nvec; v += SNT) {
      bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t key = bf16_key((i & 1) ? (r.u[i >> 1] >> 16) : (r.u[i >> 1] & 0xFFFFu));
        if ((int)(key >> 8) == hb) atomicAdd(&hist[key & 0xFF], 1);
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int cum = above, lb = 255;
      for (; lb > 0; --lb) {
        if (cum + hist[lb] >= k) break;
        cum += hist[lb];
      }
      sh_sel[2] = (hb << 8) | lb;
      sh_sel[3] = k - cum;  // how many keys equal to the threshold are kept
    }
    __syncthreads();
    thr_key = (uint32_t)sh_sel[2];
    need_eq = sh_sel[3];
  }

  // --------------------------------------------------------- LSE over kept entries + Gumbel argmax
  MS ms{-INFINITY, 0.f};
  AM best{-INFINITY, INT64_MAX};
  int eq_carry = 0;
  for (int64_t base = 0; base < nvec; base += SNT) {
    const int64_t v = base + threadIdx.x;
    bf16x8 r{};
    const bool live = v < nvec;
    if (live) r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
    float x[8];
    unpack8(r, x);
    uint32_t keys[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) keys[i] = bf16_key((i & 1) ? (r.u[i >> 1] >> 16) : (r.u[i >> 1] & 0xFFFFu));
    int my_eq = 0;
    if (use_topk && live) {
#pragma unroll
      for (int i = 0; i < 8; ++i) my_eq += (keys[i] == thr_key);
    }
    int rank = 0;
    if (use_topk) {
      int tot = 0;
      rank = eq_carry + block_excl_scan<SNT>(my_eq, sh_scan, &tot);
      eq_carry += tot;
    }
    if (!live) continue;
    bool any_kept = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) any_kept |= keys[i] >= thr_key;
    if (!any_kept) continue;  // noise is drawn only where an entry survives the top-k filter
    float gn[8];
    gumbel8(seed, off, row, v * 8, gn);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      bool keep = true;
      if (use_topk) {
        if (keys[i] > thr_key) keep = true;
        else if (keys[i] == thr_key) keep = (rank++ < need_eq);
        else keep = false;
      }
      if (!keep) continue;
      const float xs = __fdiv_rn(x[i], p.temperature);
      ms_add(ms, xs);
      best = am_merge(best, AM{xs + gn[i], v * 8 + i});
    }
  }
  ms = block_ms<SNT>(ms, sh_ms);
  best = block_am<SNT>(best, sh_am);
  if (threadIdx.x == 0) {
    const bool ok = best.i >= 0 && best.i < p.V;  // false only when no finite candidate exists
    if (!ok) qb_set_err(p.err, QB_DEVERR_TOKEN);
    const int64_t tok = ok ? best.i : 0;
    p.tokens[row] = tok;
    const float xt = __fdiv_rn(bf2f(lrow[tok]), p.temperature);
    p.logp[row] = (xt - ms.m) - logf(ms.s);
  }
}

// ---------------------------------------------------------------- log-prob fwd / bwd
constexpr int LNT = 256;

__global__ void __launch_bounds__(LNT)
logprob_fwd_kernel(const bf16* __restrict__ logits, int64_t V, int64_t ld, const int64_t* __restrict__ targets,
                   const int64_t* __restrict__ dest, float* __restrict__ logp, float* __restrict__ lse, int* err) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ MS sh[32];
  const int64_t row = blockIdx.x;
  const bf16* lrow = logits + row * ld;
  const int64_t nvec = V / 8;
  MS ms{-INFINITY, 0.f};
  for (int64_t v = threadIdx.x; v < nvec; v += LNT) {
    bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
    float x[8];
    unpack8(r, x);
    float mx = x[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) mx = fmaxf(mx, x[i]);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += expf(x[i] - mx);
    ms = ms_merge(ms, MS{mx, s});
  }
  ms = block_ms<LNT>(ms, sh);
  if (threadIdx.x == 0) {
    const float l = ms.m + logf(ms.s);
    lse[row] = l;
    const int64_t d = dest ? dest[row] : row;
    if (d >= 0) {
      int64_t t = targets[row];
      if (t < 0 || t >= V) {
        qb_set_err(err, QB_DEVERR_TOKEN);
        logp[d] = 0.f;
      } else {
        logp[d] = (bf2f(lrow[t]) - ms.m) - logf(ms.s);
      }
    }
  }
}

__global__ void __launch_bounds__(LNT)
logprob_bwd_kernel(bf16* __restrict__ logits, int64_t V, int64_t ld, const int64_t* __restrict__ targets,
                   const int64_t* __restrict__ dest, const float* __restrict__ lse, const float* __restrict__ gl) {
  qb_pdl_trigger();
  qb_pdl_wait();
  const int64_t row = blockIdx.x;
  bf16* lrow = logits + row * ld;
  const int64_t d = dest ? dest[row] : row;
  const float g = (d >= 0) ? gl[d] : 0.f;
  const float l = lse[row];
  const int64_t t = targets[row];
  const int64_t nvec = V / 8;
  for (int64_t v = threadIdx.x; v < nvec; v += LNT) {
    bf16x8 r = *reinterpret_cast<const bf16x8*>(lrow + v * 8);
    float x[8];
    unpack8(r, x);
    bf16x8 o;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t c = v * 8 + 2 * i;
      const float a = (c == t ? g : 0.f) - expf(x[2 * i] - l) * g;
      const float b = (c + 1 == t ? g : 0.f) - expf(x[2 * i + 1] - l) * g;
      o.u[i] = pack_bf16x2(a, b);
    }
    *reinterpret_cast<bf16x8*>(lrow + v * 8) = o;
  }
}

// ---------------------------------------------------------------- GRPO
// Workspace layout: [0] u32 mask ticket, [1] u32 loss ticket, [2] f32 denominator,
// [3] pad, then f32 partials.
constexpr int WS_HDR = 4;
constexpr int MS_BLOCKS = 256;

__global__ void mask_sum_kernel(const float* __restrict__ mask, int64_t n, float* __restrict__ out,
                                uint32_t* __restrict__ ws) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ float red[32];
  __shared__ bool last;
  float s = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    s += mask[i];
  s = block_sum(s, red);
  float* part = reinterpret_cast<float*>(ws + WS_HDR);
  if (threadIdx.x == 0) {
    part[blockIdx.x] = s;
    __threadfence();
    last = atomicAdd(&ws[0], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    float t = 0.f;
    for (unsigned b = 0; b < gridDim.x; ++b) t += reinterpret_cast<volatile float*>(part)[b];
    *out = t;
    ws[0] = 0u;
  }
}

// Group statistics of row r's group: mean and unbiased std over rows with equal id.
QB_DEVICE float group_advantage(const float* rewards, const int64_t* gids, int64_t n, int64_t r, float* red) {
  const int64_t gid = gids[r];
  float cnt = 0.f, sum = 0.f;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x)
    if (gids[j] == gid) {
      cnt += 1.f;
      sum += rewards[j];
    }
  cnt = block_sum(cnt, red);
  sum = block_sum(sum, red);
  const float mean = sum / cnt;
  float sq = 0.f;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x)
    if (gids[j] == gid) {
      const float d = rewards[j] - mean;
      sq += d * d;
    }
  sq = block_sum(sq, red);
  const float stdv = sqrtf(sq / (cnt - 1.f));
  return (rewards[r] - mean) / (stdv + 1e-8f);
}

__global__ void advantage_kernel(const float* __restrict__ rewards, const int64_t* __restrict__ gids, int64_t n,
                                 float* __restrict__ adv) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const float a = group_advantage(rewards, gids, n, r, red);
  if (threadIdx.x == 0) adv[r] = a;
}

// One token of the clipped surrogate + beta * k3 KL (ppo_clipped_loss, qwen3_grpo_train.py:193-199,
// and the GRPO paper's k3 estimator): its masked loss terms and d loss / d new_lp, where
// u = d loss / d sum(loss_token * mask) (1 / denominator, times the caller's grad scale).
struct TokenLoss {
  float surr_m, kl_m, gnew;
};

QB_DEVICE TokenLoss token_loss(float nw, float old, float ref, bool has_ref, float A, float m, float lo, float hi,
                               float beta, float u) {
  const float ratio = expf(nw - old);
  const float cr = fminf(fmaxf(ratio, lo), hi);
  const float s1 = ratio * A, s2 = cr * A;
  const float lt = -fminf(s1, s2);
  TokenLoss t{lt * m, 0.f, 0.f};
  float dkl = 0.f;
  if (has_ref) {
    const float d = ref - nw;
    const float e = expf(d);
    t.kl_m = (e - d - 1.f) * m;
    dkl = 1.f - e;
  }
  const float gl = u * m;     // grad of loss_token * mask w.r.t. loss_token
  const float gmin = -gl;     // loss_token = -min(s1, s2)
  const bool eq = s1 == s2;
  const float g1 = eq ? gmin * 0.5f : (s1 < s2 ? gmin : 0.f);
  const float g2 = eq ? gmin * 0.5f : (s2 < s1 ? gmin : 0.f);
  const float inr = (ratio >= lo && ratio <= hi) ? 1.f : 0.f;
  const float gratio = g1 * A + (g2 * A) * inr;
  t.gnew = gratio * ratio;
  if (has_ref) t.gnew += beta * gl * dkl;
  return t;
}

struct LossParams {
  const float* rewards;
  const int64_t* gids;
  const float* token_adv;  // [n_rows, S] per-token advantages (ppo_clipped_loss form)
  int64_t n_rows, S, row_begin;
  const float* new_lp;
  const float* old_lp;
  const float* ref_lp;
  const float* mask;
  const float* mask_total;  // resolved denominator (user's or the workspace slot)
  float lo, hi, beta;
  const float* grad_scale;
  float* grad_new;
  float* loss_out;
  float* adv_out;
  uint32_t* ws;
};

// FROM_REWARDS: A = group advantage of row r times mask (compute_grpo_advantage +
// token_advantages, qwen3_grpo_train.py:266-269); otherwise A = token_adv[i] as given
// to ppo_clipped_loss (:184-199).
template <bool FROM_REWARDS>
__global__ void grpo_loss_kernel(LossParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ float red[32];
  __shared__ bool last;
  const int64_t r = p.row_begin + blockIdx.x;
  float adv = 0.f;
  if (FROM_REWARDS) {
    adv = group_advantage(p.rewards, p.gids, p.n_rows, r, red);
    if (p.adv_out && threadIdx.x == 0) p.adv_out[r] = adv;
  }
  const float denom = *p.mask_total + 1e-8f;
  const float gs = p.grad_scale ? *p.grad_scale : 1.f;
  const float u = gs / denom;  // d loss / d sum(loss_token * mask)
  float surr = 0.f, klsum = 0.f;
  for (int64_t s = threadIdx.x; s < p.S; s += blockDim.x) {
    const int64_t i = r * p.S + s;
    const float m = p.mask[i];
    const float A = FROM_REWARDS ? adv * m : p.token_adv[i];
    const TokenLoss t = token_loss(p.new_lp[i], p.old_lp[i], p.ref_lp ? p.ref_lp[i] : 0.f, p.ref_lp != nullptr, A, m,
                                   p.lo, p.hi, p.beta, u);
    surr += t.surr_m;
    klsum += t.kl_m;
    if (p.grad_new) p.grad_new[i] = t.gnew;
  }
  surr = block_sum(surr, red);
  klsum = block_sum(klsum, red);
  float* part = reinterpret_cast<float*>(p.ws + WS_HDR);
  if (threadIdx.x == 0) {
    part[2 * blockIdx.x] = surr;
    part[2 * blockIdx.x + 1] = klsum;
    __threadfence();
    last = atomicAdd(&p.ws[1], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    volatile float* vp = part;
    float ts = 0.f, tk = 0.f;
    for (unsigned b = 0; b < gridDim.x; ++b) {
      ts += vp[2 * b];
      tk += vp[2 * b + 1];
    }
    if (p.loss_out) {
      const float ls = ts / denom, lk = tk / denom;
      p.loss_out[0] += ls + p.beta * lk;
      p.loss_out[1] += ls;
      p.loss_out[2] += lk;
    }
    p.ws[1] = 0u;
  }
}

// ---------------------------------------------------------------- single-pass log-prob + loss + logit gradient
// One row of bf16 logits (151,936 entries = 297 KB) is split over a cluster of LL_CTAS CTAs; each
// CTA brings its slice into shared memory with bulk copies (one read from HBM), folds it into a
// (max, sum of exp) pair, the cluster exchanges the pairs and the target's logit through
// distributed shared memory, every CTA forms the row's log-sum-exp, the token's log-prob, its
// GRPO loss terms and d loss / d logp identically, and writes d loss / d logits of its slice
// back over the logits from shared memory (one write).  The logits cross HBM once each way.
constexpr int LL_CTAS = 4;
constexpr int LL_THREADS = 256;
constexpr int LL_COPY = 32768;  // bytes per bulk copy

struct LogitLossParams {
  bf16* logits;
  int64_t ld, V, n_rows, S;
  const int64_t* targets;
  const float* adv;  // [n_rows / S] advantages of the sequences
  const float* old_lp;
  const float* ref_lp;
  const float* mask;
  const float* mask_total;
  float lo, hi, beta;
  float* new_lp;
  float* grad_new;
  float* row_part;  // [2 * n_rows]: masked surrogate and KL terms of each token
  int chunk;        // logits per CTA (multiple of 8)
  int* err;
};

QB_DEVICE void ll_merge(float& m2, float& s, float om2, float os) {
  const float nm = fmaxf(m2, om2);
  if (nm == -INFINITY) return;
  s = s * exp2f(m2 - nm) + os * exp2f(om2 - nm);
  m2 = nm;
}

__global__ void __launch_bounds__(LL_THREADS)
logit_loss_kernel(LogitLossParams p) {
  qb_pdl_trigger();
  qb_pdl_wait();
  constexpr float L2E = 1.4426950408889634f, LN2 = 0.6931471805599453f;
  extern __shared__ __align__(128) uint8_t ll_smem[];
  __shared__ float red[2][LL_THREADS / 32];
  __shared__ __align__(16) float4 slot;  // (max2, sum, target logit, 1 if this slice holds the target)
  __shared__ float bc[2];                // g, lse2
  __shared__ __align__(8) uint64_t bar;
  const uint32_t rank = cluster_rank();
  const int64_t row = blockIdx.x / LL_CTAS;
  const int64_t c0 = (int64_t)rank * p.chunk;
  const int64_t c1 = c0 + p.chunk < p.V ? c0 + p.chunk : p.V;
  const int nel = c1 > c0 ? (int)(c1 - c0) : 0;
  bf16* grow = p.logits + row * p.ld;
  const bf16* sx = reinterpret_cast<const bf16*>(ll_smem);
  const uint32_t mb = smem_u32(&bar);
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mb));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint32_t bytes = (uint32_t)nel * 2;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(bytes) : "memory");
    for (uint32_t o = 0; o < bytes; o += LL_COPY) {
      const uint32_t n = bytes - o < (uint32_t)LL_COPY ? bytes - o : (uint32_t)LL_COPY;
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(ll_smem) + o),
          "l"(reinterpret_cast<const uint8_t*>(grow + c0) + o), "r"(n), "r"(mb)
          : "memory");
    }
  }
  __syncthreads();
  // bounded wait for this CTA's slice (~2 s of SM clock)
  bool ready = false;
  const long long t0 = clock64();
  while (!ready) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.shared::cta.b64 q, [%1], 0;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(ok)
        : "r"(mb)
        : "memory");
    ready = ok != 0;
    if (!ready && clock64() - t0 > 4000000000ll) break;
  }
  if (!ready && threadIdx.x == 0) qb_set_err(p.err, QB_DEVERR_TIMEOUT);
  const int64_t tgt = p.targets[row];
  // this CTA's (max, sum of exp) in the log2 domain
  float m2 = -INFINITY, sm = 0.f;
  if (ready) {
    for (int v = threadIdx.x; v < nel / 8; v += LL_THREADS) {
      const uint4 u = reinterpret_cast<const uint4*>(sx)[v];
      float x[8];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        x[2 * j] = f.x;
        x[2 * j + 1] = f.y;
      }
      float mx = x[0];
#pragma unroll
      for (int j = 1; j < 8; ++j) mx = fmaxf(mx, x[j]);
      const float nm2 = fmaxf(m2, mx * L2E);
      float acc = sm * exp2f(m2 - nm2);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc += exp2f(fmaf(x[j], L2E, -nm2));
      sm = acc;
      m2 = nm2;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m2, o), os = __shfl_xor_sync(0xffffffffu, sm, o);
    ll_merge(m2, sm, om, os);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = m2;
    red[1][threadIdx.x >> 5] = sm;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = red[0][0], Sx = red[1][0];
    for (int w = 1; w < LL_THREADS / 32; ++w) ll_merge(M, Sx, red[0][w], red[1][w]);
    const bool has_t = ready && tgt >= c0 && tgt < c1;
    slot = make_float4(M, Sx, has_t ? bf2f(sx[tgt - c0]) : 0.f, has_t ? 1.f : 0.f);
  }
  cluster_sync();  // every CTA's slot is published
  if (threadIdx.x == 0) {
    float M = -INFINITY, Sx = 0.f, xt = 0.f;
    bool found = false;
    for (uint32_t r = 0; r < LL_CTAS; ++r) {
      float4 o;
      asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(o.x), "=f"(o.y), "=f"(o.z), "=f"(o.w)
                   : "r"(cluster_addr(smem_u32(&slot), r)));
      ll_merge(M, Sx, o.x, o.y);
      if (o.w != 0.f) {
        xt = o.z;
        found = true;
      }
    }
    const float lse2 = M + log2f(Sx);
    const int64_t seq = row / p.S;
    const float m = p.mask[row];
    const bool valid = found && tgt >= 0 && tgt < p.V;
    const float logp = valid ? xt - lse2 * LN2 : 0.f;
    const float u = 1.f / (*p.mask_total + 1e-8f);
    const TokenLoss t = token_loss(logp, p.old_lp[row], p.ref_lp ? p.ref_lp[row] : 0.f, p.ref_lp != nullptr,
                                   p.adv[seq] * m, m, p.lo, p.hi, p.beta, u);
    const float g = valid ? t.gnew : 0.f;
    bc[0] = g;
    bc[1] = lse2;
    if (rank == 0) {
      if (!valid) qb_set_err(p.err, QB_DEVERR_TOKEN);
      p.new_lp[row] = logp;
      if (p.grad_new) p.grad_new[row] = g;
      p.row_part[2 * row] = t.surr_m;
      p.row_part[2 * row + 1] = t.kl_m;
    }
  }
  // done with the other CTAs' slots; they may leave once everyone has read
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();
  const float g = bc[0], lse2 = bc[1];
  if (ready) {
    for (int v = threadIdx.x; v < nel / 8; v += LL_THREADS) {
      const uint4 u = reinterpret_cast<const uint4*>(sx)[v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      uint32_t o[4];
      const int64_t c = c0 + 8 * (int64_t)v;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        const float a = ((c + 2 * j == tgt) ? g : 0.f) - g * exp2f(fmaf(f.x, L2E, -lse2));
        const float b = ((c + 2 * j + 1 == tgt) ? g : 0.f) - g * exp2f(fmaf(f.y, L2E, -lse2));
        o[j] = pack_bf16x2(a, b);
      }
      reinterpret_cast<uint4*>(grow + c)[0] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// loss_out (+=) from the per-token terms, summed in a fixed order.
__global__ void logit_loss_reduce_kernel(const float* __restrict__ row_part, int64_t n_rows,
                                         const float* __restrict__ mask_total, float beta, float* loss_out) {
  qb_pdl_trigger();
  qb_pdl_wait();
  __shared__ float red[32];
  float su = 0.f, kl = 0.f;
  for (int64_t i = threadIdx.x; i < n_rows; i += blockDim.x) {
    su += row_part[2 * i];
    kl += row_part[2 * i + 1];
  }
  su = block_sum(su, red);
  kl = block_sum(kl, red);
  if (threadIdx.x == 0 && loss_out) {
    const float d = *mask_total + 1e-8f;
    loss_out[0] += su / d + beta * (kl / d);
    loss_out[1] += su / d;
    loss_out[2] += kl / d;
  }
}

inline bool al16(const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; }

}  // namespace

// ================================================================ C ABI
extern "C" int qb_sample(const void* logits, int64_t n, int64_t V, int64_t ld, float temperature, int top_k,
                         uint64_t seed, const uint64_t* offset, int64_t* tokens, float* logp, int* err,
                         qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0 && V > 0 && ld >= V && top_k >= 0 && temperature > 0.f);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(logits && tokens && logp && al16(logits) && ld % 8 == 0);
  if (V % 8 != 0) return QB_ERR_UNSUPPORTED;
  SampleParams p{(const bf16*)logits, V, ld, temperature, top_k, seed, offset, tokens, logp, err};
  return qb_launch(sample_kernel, dim3((unsigned)n), dim3(SNT), 0, (cudaStream_t)stream, 1, p);
}

extern "C" int qb_logprob_fwd(const void* logits, int64_t n, int64_t V, int64_t ld, const int64_t* targets,
                              const int64_t* dest, float* logp, float* lse, int* err, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0 && V > 0 && ld >= V);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(logits && targets && logp && lse && al16(logits) && ld % 8 == 0);
  if (V % 8 != 0) return QB_ERR_UNSUPPORTED;
  return qb_launch(logprob_fwd_kernel, dim3((unsigned)n), dim3(LNT), 0, (cudaStream_t)stream, 1, (const bf16*)logits, V, ld, targets, dest,
                                                                    logp, lse, err);
}

extern "C" int qb_logprob_bwd(void* logits, int64_t n, int64_t V, int64_t ld, const int64_t* targets,
                              const int64_t* dest, const float* lse, const float* grad_logp, int* err,
                              qb_stream_t stream) {
  (void)err;
  QB_CHECK_ARG(n >= 0 && V > 0 && ld >= V);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(logits && targets && lse && grad_logp && al16(logits) && ld % 8 == 0);
  if (V % 8 != 0) return QB_ERR_UNSUPPORTED;
  return qb_launch(logprob_bwd_kernel, dim3((unsigned)n), dim3(LNT), 0, (cudaStream_t)stream, 1, (bf16*)logits, V, ld, targets, dest, lse,
                                                                    grad_logp);
}

extern "C" int qb_grpo_advantage(const float* rewards, const int64_t* group_ids, int64_t n, float* adv,
                                 qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0 && n <= 65536);
  if (n == 0) return QB_OK;
  QB_CHECK_ARG(rewards && group_ids && adv);
  return qb_launch(advantage_kernel, dim3((unsigned)n), dim3(256), 0, (cudaStream_t)stream, 1, rewards, group_ids, n, adv);
}

extern "C" size_t qb_grpo_workspace_bytes(int64_t n_rows) {
  const int64_t parts = (2 * n_rows > MS_BLOCKS) ? 2 * n_rows : MS_BLOCKS;
  return (size_t)(WS_HDR + parts) * sizeof(float);
}

extern "C" int qb_mask_sum(const float* mask, int64_t n, float* mask_total, void* workspace, qb_stream_t stream) {
  QB_CHECK_ARG(n >= 0 && mask_total && workspace);
  QB_CHECK_ARG(n == 0 || mask);
  int64_t blocks = (n + 255) / 256;
  if (blocks > MS_BLOCKS) blocks = MS_BLOCKS;
  if (blocks < 1) blocks = 1;
  return qb_launch(mask_sum_kernel, dim3((unsigned)blocks), dim3(256), 0, (cudaStream_t)stream, 1, mask, n, mask_total, (uint32_t*)workspace);
}

extern "C" int qb_grpo_loss(const float* rewards, const int64_t* group_ids, int64_t n_rows, int64_t S,
                            int64_t row_begin, int64_t row_end, const float* new_lp, const float* old_lp,
                            const float* ref_lp, const float* mask, const float* mask_total, float clip_eps,
                            float beta, const float* grad_scale, float* grad_new, float* loss_out,
                            float* adv_out, void* workspace, qb_stream_t stream) {
  QB_CHECK_ARG(n_rows >= 0 && n_rows <= 65536 && S >= 0 && row_begin >= 0 && row_end <= n_rows &&
               row_begin <= row_end);
  if (row_end == row_begin) return QB_OK;
  QB_CHECK_ARG(rewards && group_ids && new_lp && old_lp && mask && workspace);
  uint32_t* ws = (uint32_t*)workspace;
  const float* denom = mask_total;
  if (!denom) {
    float* slot = reinterpret_cast<float*>(ws + 2);
    int st = qb_mask_sum(mask, n_rows * S, slot, workspace, stream);
    if (st != QB_OK) return st;
    denom = slot;
  }
  LossParams p{rewards, group_ids, nullptr, n_rows, S, row_begin, new_lp, old_lp, ref_lp, mask, denom,
               (float)(1.0 - (double)clip_eps), (float)(1.0 + (double)clip_eps), beta, grad_scale, grad_new,
               loss_out, adv_out, ws};
  return qb_launch(grpo_loss_kernel<true>, dim3((unsigned)(row_end - row_begin)), dim3(256), 0, (cudaStream_t)stream, 1, p);
}

extern "C" int qb_ppo_clipped_loss(const float* old_lp, const float* new_lp, const float* token_adv,
                                   const float* mask, const float* ref_lp, int64_t n_rows, int64_t S,
                                   const float* mask_total, float clip_eps, float beta, const float* grad_scale,
                                   float* grad_new, float* loss_out, void* workspace, qb_stream_t stream) {
  QB_CHECK_ARG(n_rows >= 0 && n_rows <= 65536 && S >= 0);
  if (n_rows == 0) return QB_OK;
  QB_CHECK_ARG(old_lp && new_lp && token_adv && mask && workspace);
  uint32_t* ws = (uint32_t*)workspace;
  const float* denom = mask_total;
  if (!denom) {
    float* slot = reinterpret_cast<float*>(ws + 2);
    int st = qb_mask_sum(mask, n_rows * S, slot, workspace, stream);
    if (st != QB_OK) return st;
    denom = slot;
  }
  LossParams p{nullptr, nullptr, token_adv, n_rows, S, 0, new_lp, old_lp, ref_lp, mask, denom,
               (float)(1.0 - (double)clip_eps), (float)(1.0 + (double)clip_eps), beta, grad_scale, grad_new,
               loss_out, nullptr, ws};
  return qb_launch(grpo_loss_kernel<false>, dim3((unsigned)n_rows), dim3(256), 0, (cudaStream_t)stream, 1, p);
}

// ================================================================ allocation-free GRPO loss
// Some callers cannot hand this library a workspace buffer or let it allocate one:
// a host whose device memory is owned by another allocator (a serving runtime or a
// framework caching allocator that has reserved the HBM pool up front), or a thin
// FFI binding that only forwards tensors it already owns.  For them the fused GRPO
// loss can run on a scratch area that lives in the library image itself: a fixed
// device array, set aside once per GPU that loads the library and held until the
// process exits.  Nothing here calls cudaMalloc or cudaFree.
namespace {
constexpr int64_t NOALLOC_MAX_ROWS = 16384;  // largest n_rows this variant accepts
// Header (tickets + denominator slot, 16 B) + two fp32 partials per row, rounded up to 256 B.
constexpr size_t NOALLOC_SCRATCH_BYTES = ((16 + 2 * NOALLOC_MAX_ROWS * 4) + 255) / 256 * 256;
static __device__ __align__(256) unsigned char g_grpo_scratch[NOALLOC_SCRATCH_BYTES];

// The symbol's device address.  Host code cannot use the array's name as a device pointer, so
// the address is looked up with cudaGetSymbolAddress, with the device current, the first time a
// device calls in, and cached per device together with the CUDA context it belongs to: a call
// under another context (after cudaDeviceReset, or on a context the caller made current) looks
// the address up again instead of writing through a stale one.  A mutex orders the cache for
// callers on several host threads.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  return fn;
}

void* noalloc_scratch_ptr(int* status) {
  constexpr int MAX_DEVICES = 64;
  static std::mutex mu;
  static CUcontext ctxs[MAX_DEVICES] = {};
  static void* ptrs[MAX_DEVICES] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
    *status = e != cudaSuccess ? QB_ERR_CUDA_BASE + (int)e : QB_ERR_UNSUPPORTED;
    return nullptr;
  }
  CtxGetCurrentFn get_ctx = ctx_get_current();
  CUcontext ctx = nullptr;
  if (get_ctx && get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ctx != nullptr && ctxs[dev] == ctx && ptrs[dev] != nullptr) {
    *status = QB_OK;
    return ptrs[dev];
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_grpo_scratch);  // initialises the device's context if needed
  if (e != cudaSuccess || p == nullptr) {
    *status = QB_ERR_CUDA_BASE + (int)(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    return nullptr;
  }
  if (get_ctx && get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  ctxs[dev] = ctx;  // a null context is never matched above: the address is then looked up per call
  ptrs[dev] = p;
  *status = QB_OK;
  return p;
}
}  // namespace

extern "C" int qb_grpo_loss_noalloc(const float* rewards, const int64_t* group_ids, int64_t n_rows, int64_t S,
                                    int64_t row_begin, int64_t row_end, const float* new_lp, const float* old_lp,
                                    const float* ref_lp, const float* mask, const float* mask_total,
                                    float clip_eps, float beta, const float* grad_scale, float* grad_new,
                                    float* loss_out, float* adv_out, qb_stream_t stream) {
  // The same argument checks as qb_grpo_loss, before the shared scratch or the stream is touched.
  QB_CHECK_ARG(n_rows >= 0 && S >= 0 && row_begin >= 0 && row_end <= n_rows && row_begin <= row_end);
  if (n_rows > NOALLOC_MAX_ROWS) return QB_ERR_INVALID;  // the fixed scratch holds at most this many rows
  if (row_end == row_begin) return QB_OK;
  QB_CHECK_ARG(rewards && group_ids && new_lp && old_lp && mask);
  int st = QB_OK;
  void* ws = noalloc_scratch_ptr(&st);
  if (!ws) return st;
  // The scratch keeps whatever the previous call left; the ticket counters and the
  // denominator slot must start at zero, so clear the 16-byte header on this stream.
  cudaError_t e = cudaMemsetAsync(ws, 0, 16, (cudaStream_t)stream);
  if (e != cudaSuccess) return QB_ERR_CUDA_BASE + (int)e;
  return qb_grpo_loss(rewards, group_ids, n_rows, S, row_begin, row_end, new_lp, old_lp, ref_lp, mask, mask_total,
                      clip_eps, beta, grad_scale, grad_new, loss_out, adv_out, ws, stream);
}

// ================================================================ single-pass config-1 path
namespace {
size_t ll_align(size_t x) { return (x + 255) / 256 * 256; }
}  // namespace

extern "C" size_t qb_grpo_logit_loss_workspace_bytes(int64_t n_seqs, int64_t S) {
  if (n_seqs <= 0 || S <= 0) return 256;
  // advantages [n_seqs] | per-token terms [2 n S] | mask-sum scratch (qb_grpo_workspace_bytes)
  return ll_align((size_t)n_seqs * 4) + ll_align((size_t)n_seqs * S * 8) + ll_align(qb_grpo_workspace_bytes(n_seqs * S));
}

extern "C" int qb_grpo_logit_loss(void* logits, int64_t ld, int64_t V, const int64_t* targets, const float* rewards,
                                  const int64_t* group_ids, int64_t n_seqs, int64_t S, const float* old_lp,
                                  const float* ref_lp, const float* mask, const float* mask_total, float clip_eps,
                                  float beta, float* new_lp, float* grad_new, float* loss_out, float* adv_out,
                                  void* workspace, int* err, qb_stream_t stream) {
  QB_CHECK_ARG(n_seqs >= 0 && n_seqs <= 65536 && S >= 0 && V > 0 && ld >= V);
  if (n_seqs == 0 || S == 0) return QB_OK;
  QB_CHECK_ARG(logits && targets && rewards && group_ids && old_lp && mask && new_lp && workspace);
  QB_CHECK_ARG(al16(logits) && ld % 8 == 0 && V % 8 == 0 && al16(workspace));
  const int64_t n_rows = n_seqs * S;
  QB_CHECK_ARG(n_rows <= (1ll << 29));  // grid = n_rows * LL_CTAS CTAs
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace;
  float* adv = reinterpret_cast<float*>(ws);
  float* part = reinterpret_cast<float*>(ws + ll_align((size_t)n_seqs * 4));
  void* ms_ws = ws + ll_align((size_t)n_seqs * 4) + ll_align((size_t)n_rows * 8);
  const float* denom = mask_total;
  if (!denom) {
    // the mask-sum scratch keeps its ticket at zero between calls; clear it once here
    if (cudaMemsetAsync(ms_ws, 0, 16, st) != cudaSuccess) return qb_launch_status();
    float* slot = reinterpret_cast<float*>(reinterpret_cast<uint32_t*>(ms_ws) + 2);
    int e = qb_mask_sum(mask, n_rows, slot, ms_ws, stream);
    if (e != QB_OK) return e;
    denom = slot;
  }
  const int st_adv = qb_launch(advantage_kernel, dim3((unsigned)n_seqs), dim3(256), 0, st, 1, rewards, group_ids,
                               n_seqs, adv);
  if (st_adv != QB_OK) return st_adv;
  if (adv_out && cudaMemcpyAsync(adv_out, adv, n_seqs * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return qb_launch_status();
  const int chunk = (int)(((V + LL_CTAS - 1) / LL_CTAS + 7) / 8 * 8);
  const int smem = chunk * 2;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(logit_loss_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return qb_launch_status();
    attr = true;
  }
  if (smem > 200 * 1024) return QB_ERR_UNSUPPORTED;
  LogitLossParams p{(bf16*)logits, ld, V, n_rows, S, targets, adv, old_lp, ref_lp, mask, denom,
                    (float)(1.0 - (double)clip_eps), (float)(1.0 + (double)clip_eps), beta, new_lp, grad_new, part,
                    chunk, err};
  const int st_ll = qb_launch(logit_loss_kernel, dim3((unsigned)(n_rows * LL_CTAS)), dim3(LL_THREADS), (size_t)smem,
                              st, LL_CTAS, p);
  if (st_ll != QB_OK) return st_ll;
  return qb_launch(logit_loss_reduce_kernel, dim3(1), dim3(1024), 0, st, 1, part, n_rows, denom, beta, loss_out);
}
