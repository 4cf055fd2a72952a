/*
 * qwen3b200.h — C ABI of the B200 (sm_100a) kernels behind the GRPO step of
 * qwen3-naive-inference.
 *
 * The reference has no C ABI of its own: its hot path is Python calling
 * Triton kernels, flash-attn and cuBLAS.  Each entry point below replaces one
 * of those call sites; the comment above it cites the reference line it
 * stands in for (paths are relative to the reference project root).
 *
 * Conventions shared by every entry point:
 *   - all pointers are device pointers unless documented otherwise;
 *   - `bf16` tensors are passed as void* and hold IEEE bfloat16;
 *   - row-major layouts, explicit element strides where a view may be strided;
 *   - `stream` is a cudaStream_t (passed as void*); nothing synchronises the
 *     host, nothing allocates, so every call can be captured in a CUDA graph;
 *   - `err` (nullable) is a device int that kernels OR error bits into when a
 *     data-dependent index is out of range; the access is skipped, never made;
 *   - the return value is QB_OK (0) or an error code; argument errors are
 *     detected on the host before any launch.
 */
#ifndef QWEN3B200_H
#define QWEN3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QB_OK 0
#define QB_ERR_INVALID 1       /* bad argument (null pointer, size, alignment) */
#define QB_ERR_UNSUPPORTED 2   /* shape outside what the kernels are built for */
#define QB_ERR_CUDA_BASE 1000  /* QB_ERR_CUDA_BASE + cudaError_t of a failed launch */

/* Device error bits written to *err. */
#define QB_DEVERR_PAGE 1
#define QB_DEVERR_SLOT 2
#define QB_DEVERR_TOKEN 4
#define QB_DEVERR_SHAPE 8
#define QB_DEVERR_TIMEOUT 16

typedef void* qb_stream_t;

/* Version of this ABI (bumped on any signature change). */
int qb_abi_version(void);
/* Static description of a status code. */
const char* qb_status_string(int status);
/* Programmatic dependent launch (library-wide, on by default): the tcgen05 GEMM and attention
 * kernels may be scheduled while the kernel before them in the stream is still running, so their
 * launch and prologue (barrier init, TMEM allocation) overlap it; they wait on the device for that
 * kernel's completion before touching memory.  Short kernels launch in plain stream order.  Works
 * inside CUDA graph capture.  qb_set_pdl(0) launches every kernel with plain stream ordering;
 * qb_get_pdl reports the setting. */
int qb_set_pdl(int on);
int qb_get_pdl(void);

/* ---------------------------------------------------------------- embedding
 * Replaces nn.Embedding forward used by Qwen3Model.forward / forward_prefill /
 * forward_decode (qwen3_naive.py:772, :788, :800).
 * out[i, :] = table[ids[i], :]                          (bf16, [n, hidden]) */
int qb_embedding_fwd(const int64_t* ids, int64_t n, const void* table, int64_t vocab,
                     int64_t hidden, void* out, int* err, qb_stream_t stream);
/* Backward of the lookup: dtable[ids[i], :] += dout[i, :] (fp32 accumulator). */
int qb_embedding_bwd(const int64_t* ids, int64_t n, const void* dout, int64_t vocab,
                     int64_t hidden, float* dtable, int* err, qb_stream_t stream);

/* ---------------------------------------------------------------- RMSNorm
 * Replaces RMSNorm._rms_norm (qwen3_naive.py:156-161):
 *   y = bf16( (x * rsqrt(mean(x^2) + eps)) * w )  in fp32.
 * rstd (nullable, [rows] fp32) receives rsqrt(mean(x^2)+eps) for the backward.
 * cols must be a multiple of 256 and at most 2048. */
int qb_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t rows,
                   int64_t cols, float eps, qb_stream_t stream);
/* Replaces RMSNorm._add_rms_norm (qwen3_naive.py:163-169):
 *   s = x + residual (fp32); residual <- bf16(s); y = bf16((s*rsqrt(mean(s^2)+eps))*w). */
int qb_add_rmsnorm_fwd(const void* x, void* residual, const void* w, void* y, int64_t rows,
                       int64_t cols, float eps, qb_stream_t stream);
/* Backward of qb_rmsnorm_fwd: dx (bf16) and dw += sum_rows(dy * x * rstd) (fp32). */
int qb_rmsnorm_bwd(const void* dy, const void* x, const void* w, const float* rstd, void* dx,
                   float* dw, int64_t rows, int64_t cols, qb_stream_t stream);

/* ---------------------------------------------------------------- QK-Norm + RoPE (+ KV store)
 * Replaces, for one token row of the fused qkv projection, the sequence
 *   q_norm/k_norm (qwen3_naive.py:610-611), RotaryEmbedding.forward with the
 *   Triton _apply_rope_kernel (:389-405, :44-80) and store_kvcache (:20-41, :626).
 * qkv:  [T, ld_in] bf16, q heads at column 0, k heads at hq*D, v heads at (hq+hkv)*D.
 * out:  [T, ld_out] bf16 in the same column layout: rotated q, rotated k, copied v
 *       (nullable when only the cache and q_out are wanted).
 * q_out: nullable [T, hq, D] contiguous rotated q (used by the paged paths).
 * k_cache/v_cache: nullable [num_slots, hkv, D]; row slot_mapping[t] receives the
 *       rotated k and raw v of token t; slot -1 skips the write (qwen3_naive.py:26).
 * cos_sin: [max_pos, D] fp32, first D/2 columns cos, last D/2 sin (qwen3_naive.py:383-387).
 * q_rstd/k_rstd: nullable [T, hq] / [T, hkv] fp32 saved for the backward.
 * D must be 128. */
int qb_qk_norm_rope_fwd(const void* qkv, int64_t T, int64_t ld_in, int hq, int hkv, int D,
                        const int64_t* positions, const float* cos_sin, int64_t max_pos,
                        const void* q_norm_w, const void* k_norm_w, float eps, void* out,
                        int64_t ld_out, void* q_out, void* k_cache, void* v_cache,
                        const int32_t* slot_mapping, int64_t num_slots, float* q_rstd,
                        float* k_rstd, int* err, qb_stream_t stream);
/* Backward of qb_qk_norm_rope_fwd (no cache).  dout: [T, ld] grads w.r.t. the
 * rotated q, rotated k and v; dqkv: [T, ld] grads w.r.t. the raw projection.
 * rope_grad = 0 reproduces the reference, whose Triton RoPE writes outside
 * autograd (qwen3_naive.py:74-80): q/k grads are zero and dq_norm_w/dk_norm_w
 * are left untouched.  dq_norm_w/dk_norm_w are fp32 [D] accumulators. */
int qb_qk_norm_rope_bwd(const void* dout, const void* qkv, int64_t T, int64_t ld, int hq,
                        int hkv, int D, const int64_t* positions, const float* cos_sin,
                        int64_t max_pos, const void* q_norm_w, const void* k_norm_w,
                        const float* q_rstd, const float* k_rstd, int rope_grad, void* dqkv,
                        float* dq_norm_w, float* dk_norm_w, int* err, qb_stream_t stream);

/* ---------------------------------------------------------------- SwiGLU, residual add
 * Replaces Qwen3MLP.forward's silu(gate)*up (qwen3_naive.py:695-701):
 *   gate_up [T, 2I] (gate = columns [0,I)), out [T, I] = bf16(silu(gate)*up). I % 8 == 0. */
int qb_silu_mul_fwd(const void* gate_up, int64_t T, int64_t I, void* out, qb_stream_t stream);
int qb_silu_mul_bwd(const void* dout, const void* gate_up, int64_t T, int64_t I,
                    void* dgate_up, qb_stream_t stream);
/* out = bf16(a + b), n elements (the bf16 residual adds of Qwen3DecoderLayer.forward, :715-719). */
int qb_add_bf16(const void* a, const void* b, void* out, int64_t n, qb_stream_t stream);

/* ---------------------------------------------------------------- attention
 * Causal GQA attention over variable-length sequences; replaces
 * flash_attn_varlen_func in Qwen3Attention.forward_prefill (qwen3_naive.py:631-637,
 * paged, block_table=) and in the varlen branch of Qwen3Attention.forward (:540-548,
 * dense).  Query row i of sequence b sits at absolute position Lk_b - Lq_b + i
 * and attends keys 0..Lk_b-Lq_b+i (flash-attn's bottom-right causal alignment).
 *   q:  row (cu_q[b] + i) at q + row*q_stride + h*D
 *   dense K/V (block_tables == NULL): row (cu_k[b] + j) at k/v + row*kv_stride + kvh*D
 *   paged K/V: k/v are caches [num_blocks, page_size, hkv, D]; token j of sequence b
 *       lives in page block_tables[b*bt_stride + j/page_size].
 * tile_info: [n_tiles, 2] int32 pairs (b, first query row of a 64-row tile); when
 *       NULL, tile t maps to b = t / tiles_per_seq, first row 64*(t % tiles_per_seq)
 *       (tiles past a sequence's end exit at once) and n_tiles = batch*tiles_per_seq.
 * out: row (cu_q[b]+i) at out + row*o_stride + h*D (bf16).
 * lse: nullable [hq, total_q] fp32 natural-log softmax normaliser (for the backward).
 * D = 128, page_size = 256, hq % hkv == 0. */
int qb_attn_varlen_fwd(const void* q, int64_t q_stride, const void* k, const void* v,
                       int64_t kv_stride, const int32_t* block_tables, int64_t bt_stride,
                       int64_t num_blocks, int page_size, const int32_t* cu_seqlens_q,
                       const int32_t* cu_seqlens_k, int batch, const int32_t* tile_info,
                       int n_tiles, int tiles_per_seq, int hq, int hkv, int D, float scale,
                       void* out, int64_t o_stride, float* lse, int64_t total_q, int* err,
                       qb_stream_t stream);
/* Backward of the dense form of qb_attn_varlen_fwd (Lq == Lk per sequence, i.e.
 * training on packed sequences).  q/k/v/dq/dk/dv share the row stride `stride`;
 * o/do share `o_stride`.  delta: scratch [hq, total] fp32.  dq/dk/dv are bf16 and
 * fully overwritten.  kv_tile_info: [n_tiles,2] (b, first key row of a 64-row tile);
 * q_tile_info: [n_tiles,2] as in the forward (the two lists are identical for
 * Lq == Lk and may alias). */
int qb_attn_varlen_bwd(const void* q, const void* k, const void* v, int64_t stride,
                       const void* o, const void* dout, int64_t o_stride, const float* lse,
                       const int32_t* cu_seqlens, int batch, const int32_t* tile_info,
                       int n_tiles, int hq, int hkv, int D, float scale, int64_t total,
                       float* delta, void* dq, void* dk, void* dv, int* err,
                       qb_stream_t stream);

/* Paged single-token decode attention; replaces flash_attn_with_kvcache in
 * Qwen3Attention.forward_decode (qwen3_naive.py:672-680).
 *   q: [batch, hq, D] bf16; caches [num_blocks, page_size, hkv, D];
 *   kv length of sequence b = seqlens[b] + seqlen_add (the reference passes
 *   cache_seqlens = context_lens + 1, i.e. seqlen_add = 1 on context_lens); a sequence
 *   with length <= 0 reads no keys and gets zero output (batch padding rows);
 *   the key range is split into chunks of split_tokens (multiple of 64) processed by
 *   separate CTAs; with max_splits > 1 partial results go to `workspace`
 *   (qb_paged_decode_workspace_bytes) and a second kernel merges them.
 *   out: [batch, hq, D] bf16.  D = 128, page_size = 256, hq == 2*hkv. */
int qb_paged_decode_attn(const void* q, const void* k_cache, const void* v_cache,
                         int64_t num_blocks, int page_size, const int32_t* block_tables,
                         int64_t bt_stride, const int32_t* seqlens, int seqlen_add, int batch,
                         int hq, int hkv, int D, float scale, int split_tokens, int max_splits,
                         float* workspace, void* out, int* err, qb_stream_t stream);
size_t qb_paged_decode_workspace_bytes(int batch, int hq, int D, int max_splits);
/* Decode attention for groups of sequences that share a prompt (GRPO's G completions of
 * one prompt; the reference keeps no such sharing, its siblings each hold and read their
 * own copy of the prompt K/V).  Same result as qb_paged_decode_attn.  Every sequence
 * belongs to exactly one group (singletons allowed): group g lists its members in
 * group_members[g*8 .. g*8+7] (-1 padded, at most 8) and shares its first shared_len[g]
 * keys, stored in the pages of its first member's block_tables row.  Sequence b attends to
 * those shared keys and to its own keys [kv_start[b], len_b) (positions in b's block_tables
 * row, len_b = seqlens[b] + seqlen_add); kv_start[b] >= shared_len of b's group and a
 * multiple of 64.  Keys in [shared_len, kv_start) are never read, so a member's own tokens
 * may start on a fresh page after a partially filled shared prompt page; with kv_start ==
 * shared_len the result equals qb_paged_decode_attn.  The shared keys are read once per group
 * for all members' query heads and each member's own keys separately (one launch), then a
 * second kernel merges the split-K partials (shared_splits + own_splits slots per sequence
 * and head).  workspace: qb_paged_decode_grouped_workspace_bytes(batch, hq, D,
 * shared_splits + own_splits) bytes, any contents (every call rewrites the partials it reads);
 * calls sharing one must not overlap. */
int qb_paged_decode_attn_grouped(const void* q, const void* k_cache, const void* v_cache,
                                 int64_t num_blocks, int page_size, const int32_t* block_tables,
                                 int64_t bt_stride, const int32_t* seqlens, int seqlen_add,
                                 int batch, int hq, int hkv, int D, float scale,
                                 const int32_t* group_members, const int32_t* shared_len,
                                 int n_groups, const int32_t* kv_start, int split_tokens,
                                 int shared_splits, int own_splits, float* workspace, void* out,
                                 int* err, qb_stream_t stream);
size_t qb_paged_decode_grouped_workspace_bytes(int batch, int hq, int D, int n_slots);

/* ---------------------------------------------------------------- lm_head log-prob / sampling
 * Token log-probability from bf16 logits rows; replaces the fp32
 * log_softmax + gather of forward_logprob (qwen3_grpo_train.py:48-52).
 *   logits: [n, ld] bf16 (first V columns used); targets [n] int64 (< V).
 *   logp[dest[i]] = logits[i, t_i] - lse_i, lse[i] = logsumexp(logits[i, :V]) (fp32).
 *   dest nullable (identity); dest[i] < 0 skips row i. */
int qb_logprob_fwd(const void* logits, int64_t n, int64_t V, int64_t ld, const int64_t* targets,
                   const int64_t* dest, float* logp, float* lse, int* err, qb_stream_t stream);
/* lm_head -> log-softmax -> gather in one pass over the tensor cores, without storing logits;
 * replaces `log_softmax(model(ids).float()).gather(ids)` of forward_logprob
 * (qwen3_grpo_train.py:46-53) together with the tied lm_head GEMM (qwen3_naive.py:826).
 *   h [n, K] bf16 (row pitch ldh), W [V, K] bf16 (the lm_head / embedding weight, pitch ldw).
 *   The tcgen05 GEMM's epilogue folds each fp32 logit tile into per-row (max, sum of exp)
 *   partials in `workspace` and keeps the target column's logit; a second kernel merges the
 *   partials:  lse[i] = logsumexp_v(h_i . W_v),  logp[dest[i]] = h_i . W_{t_i} - lse[i].
 *   The logits stay in fp32 (the reference rounds them to bf16 first; this is the more exact
 *   value of the same quantity).  dest nullable (identity), dest[i] < 0 skips row i; lse
 *   nullable; a target outside [0, V) sets QB_DEVERR_TOKEN and gives logp 0.
 *   logits (nullable): when given, the bf16 logits [n, V] (pitch ld_logits) are stored as well,
 *   for a backward pass that needs them.
 *   workspace: qb_lm_head_logprob_workspace_bytes(n, V) bytes, 16-byte aligned, any contents. */
int qb_lm_head_logprob(const void* h, int64_t ldh, const void* W, int64_t ldw, int64_t n, int64_t V,
                       int64_t K, const int64_t* targets, const int64_t* dest, float* logp, float* lse,
                       void* logits, int64_t ld_logits, void* workspace, int* err, qb_stream_t stream);
size_t qb_lm_head_logprob_workspace_bytes(int64_t n, int64_t V);
/* Backward: logits[i, v] <- bf16( g_i * (1[v == t_i] - exp(logits[i,v] - lse_i)) ), in place,
 * with g_i = grad_logp[dest[i]] (0 for skipped rows). */
int qb_logprob_bwd(void* logits, int64_t n, int64_t V, int64_t ld, const int64_t* targets,
                   const int64_t* dest, const float* lse, const float* grad_logp, int* err,
                   qb_stream_t stream);
/* Sampling with the sampled token's log-prob; replaces the temperature / top-k /
 * softmax / multinomial / log_softmax.gather block of
 * generate_continuous_with_logprobs (qwen3_naive.py:1632-1650).
 *   x = float(logits)/temperature; top_k = 0 keeps all V entries, otherwise the k
 *   largest (ties broken toward the lower index); token ~ softmax(x over kept) drawn from
 *   a counter-based Philox4x32-10 stream keyed by (seed ^ rng_state[1], rng_state[0], row):
 *   with every entry kept by inverse-CDF sampling on one 53-bit uniform per row, with top-k
 *   by the Gumbel-max rule over the kept entries (noise per column);
 *   logp = log_softmax(x over kept)[token].
 *   top_k = 1 is greedy argmax with logp = 0.  rng_state (nullable): device uint64[2]
 *   {counter, seed mix}, read at run time so a captured graph draws new noise per replay. */
int qb_sample(const void* logits, int64_t n, int64_t V, int64_t ld, float temperature,
              int top_k, uint64_t seed, const uint64_t* rng_state, int64_t* tokens, float* logp,
              int* err, qb_stream_t stream);

/* ---------------------------------------------------------------- GRPO
 * Group-relative advantages; replaces compute_grpo_advantage (qwen3_grpo_train.py:162-173):
 * adv[i] = (r[i] - mean_g) / (std_g + 1e-8), std unbiased over the members of i's group
 * (group = equal group_ids).  n <= 65536. */
int qb_grpo_advantage(const float* rewards, const int64_t* group_ids, int64_t n, float* adv,
                      qb_stream_t stream);
/* Fused GRPO loss and its gradient; replaces compute_grpo_advantage + token advantage +
 * ppo_clipped_loss (qwen3_grpo_train.py:266-269, :184-199) and adds the k3 KL term
 * kl = exp(ref - new) - (ref - new) - 1 weighted by beta.
 * Rows [row_begin, row_end) of the [n_rows, S] (row stride S) fp32 tensors are processed;
 * advantages use all n_rows rewards.  denom = mask_total ? *mask_total : sum(mask rows),
 * loss = sum(mask*(-min(r*A, clip(r)*A) + beta*kl)) / (denom + 1e-8), r = exp(new-old),
 * A = adv*mask.  grad_new (nullable) receives dloss/dnew times (*grad_scale or 1).
 * loss_out[3] (nullable): loss, surrogate part, kl part — accumulated (+=), so callers
 * zero it once and microbatches add up.  adv_out (nullable) [n_rows].
 * workspace: qb_grpo_workspace_bytes(); its first 16 bytes must be zero before the
 * first call and are left zero by every call. */
int qb_grpo_loss(const float* rewards, const int64_t* group_ids, int64_t n_rows, int64_t S,
                 int64_t row_begin, int64_t row_end, const float* new_lp, const float* old_lp,
                 const float* ref_lp, const float* mask, const float* mask_total, float clip_eps,
                 float beta, const float* grad_scale, float* grad_new, float* loss_out,
                 float* adv_out, void* workspace, qb_stream_t stream);
size_t qb_grpo_workspace_bytes(int64_t n_rows);
/* The same fused loss and gradient with caller-supplied per-token advantages
 * (token_adv [n_rows, S], already multiplied by the mask as in grpo_train_step);
 * replaces ppo_clipped_loss(old_log_probs, new_log_probs, advantages, response_mask)
 * (qwen3_grpo_train.py:184-199).  ref_lp nullable (beta ignored then). */
int qb_ppo_clipped_loss(const float* old_lp, const float* new_lp, const float* token_adv,
                        const float* mask, const float* ref_lp, int64_t n_rows, int64_t S,
                        const float* mask_total, float clip_eps, float beta,
                        const float* grad_scale, float* grad_new, float* loss_out,
                        void* workspace, qb_stream_t stream);
/* qb_grpo_loss without a workspace argument, for callers that cannot allocate device
 * memory or hand the library a scratch buffer: hosts whose GPU memory is owned by another
 * allocator (a serving runtime or a framework pool that reserved HBM up front, where a
 * surprise cudaMalloc fails or fragments the pool and cudaMalloc/cudaFree synchronise the
 * device) and thin FFI bindings that only forward tensors they already own.  It has no
 * counterpart in the reference.  Same arguments and results as qb_grpo_loss.
 *   - Scratch lives in a fixed device array inside this library (about 128 KiB, held by
 *     every GPU that loads the library until the process exits); n_rows above 16384 is
 *     rejected with QB_ERR_INVALID before anything runs.  Nothing is allocated.
 *   - The first call on a device looks up that array's device address with the device
 *     current, and again after the device's CUDA context changes (cudaDeviceReset);
 *     make that first call before any stream capture.
 *   - Arguments are checked as in qb_grpo_loss before the scratch or the stream is touched;
 *     an empty row range returns QB_OK at once.
 *   - Every call reuses the same array and clears its 16-byte counter header on `stream`
 *     first; calls that overlap on the GPU (different streams, or another thread) race
 *     on it and must be serialised by the caller. */
int qb_grpo_loss_noalloc(const float* rewards, const int64_t* group_ids, int64_t n_rows, int64_t S,
                         int64_t row_begin, int64_t row_end, const float* new_lp,
                         const float* old_lp, const float* ref_lp, const float* mask,
                         const float* mask_total, float clip_eps, float beta,
                         const float* grad_scale, float* grad_new, float* loss_out,
                         float* adv_out, qb_stream_t stream);
/* Config 1's whole pass in one read and one write of the logits: log-prob of each token from its
 * row of bf16 logits, group advantages, the clipped surrogate + beta * k3 KL loss and its
 * gradient, written back over the logits as d loss / d logits; replaces forward_logprob's
 * log_softmax + gather (qwen3_grpo_train.py:49-52), compute_grpo_advantage (:162-173),
 * ppo_clipped_loss (:184-199) and the autograd backward to the logits.
 *   logits [n_seqs * S, ld] bf16 (row = seq * S + position), overwritten with the gradient;
 *   targets [n_seqs * S]; rewards / group_ids [n_seqs]; old_lp, ref_lp (nullable), mask
 *   [n_seqs, S] fp32; mask_total as in qb_grpo_loss.  Outputs: new_lp [n_seqs, S] (0 and
 *   QB_DEVERR_TOKEN for a target outside [0, V)), grad_new (nullable) d loss / d new_lp,
 *   loss_out[3] += (loss, surrogate, kl), adv_out (nullable) [n_seqs].
 *   A row's slices are shared by a cluster of 4 CTAs through distributed shared memory.
 *   V % 8 == 0, V <= 409600; workspace: qb_grpo_logit_loss_workspace_bytes, 16-byte aligned,
 *   any contents. */
int qb_grpo_logit_loss(void* logits, int64_t ld, int64_t V, const int64_t* targets,
                       const float* rewards, const int64_t* group_ids, int64_t n_seqs, int64_t S,
                       const float* old_lp, const float* ref_lp, const float* mask,
                       const float* mask_total, float clip_eps, float beta, float* new_lp,
                       float* grad_new, float* loss_out, float* adv_out, void* workspace, int* err,
                       qb_stream_t stream);
size_t qb_grpo_logit_loss_workspace_bytes(int64_t n_seqs, int64_t S);
/* mask_total[0] = sum of the [n] fp32 mask (the reference's response_mask.sum(),
 * qwen3_grpo_train.py:198); workspace as above. */
int qb_mask_sum(const float* mask, int64_t n, float* mask_total, void* workspace,
                qb_stream_t stream);

/* ---------------------------------------------------------------- dense projections
 * bf16 GEMM on the sm_100a tensor cores (tcgen05.mma, TMEM accumulators, TMA loads);
 * replaces the cuBLAS nn.Linear calls of qkv_proj, o_proj, gate_up_proj, down_proj and the
 * tied lm_head (qwen3_naive.py:427-428, :692-693, :826):
 *   C[M, N] = A[M, K] . B[N, K]^T       A, B bf16 row-major with K contiguous (lda, ldb >= K)
 * mode 0: C bf16; mode 1: C fp32; mode 2: C fp32 += A.B^T.  Any K >= 1 (a K tail is
 * zero-filled); A and B 16-byte aligned with lda, ldb % 8 == 0 (TMA operands); any ldc >= N. */
int qb_gemm_bf16(const void* A, int64_t lda, const void* B, int64_t ldb, void* C, int64_t ldc,
                 int64_t M, int64_t N, int64_t K, int mode, int* err, qb_stream_t stream);
/* Flag ORed into the mode of qb_gemm_bf16 / qb_gemm_bf16_ex: B is written by no kernel that may
 * still be running on the stream when the GEMM is launched (weights during inference), so the
 * kernel may start fetching B before the kernel before it has finished. */
#define QB_GEMM_B_STATIC 0x100
/* The same product with either operand stored MN-major, for the backward of the projections
 * (the reference's autograd of nn.Linear / lm_head):
 *   a_mn_major = 0: A is [M, K] (K contiguous);  1: A is stored [K, M] (M contiguous, lda >= M)
 *   b_mn_major = 0: B is [N, K];                 1: B is stored [K, N] (N contiguous, ldb >= N)
 * dX = dY . W uses (0, 1); dW = dY^T . X uses (1, 1). */
int qb_gemm_bf16_ex(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb,
                    int b_mn_major, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int mode,
                    int* err, qb_stream_t stream);
/* gate_up projection fused with SwiGLU (Qwen3MLP.forward's gate_up_proj then silu(gate) * up,
 * qwen3_naive.py:692-701) in one GEMM:
 *   H[M, I] = bf16( silu(g) * u ),  g = bf16(A . W[0:I]^T), u = bf16(A . W[I:2I]^T)
 * with W the [2I, K] gate_up weight (gate rows first, ldw >= K) -- the same bits as qb_gemm_bf16
 * into [M, 2I] followed by qb_silu_mul_fwd.  GU (nullable, [M, ldgu >= 2I]) also receives the bf16
 * gate_up product (what the backward, qb_silu_mul_bwd, reads).  flags: 0 or QB_GEMM_B_STATIC.
 * A, W 16-byte aligned, lda, ldw % 8 == 0; any ldh >= I. */
int qb_gemm_swiglu(const void* A, int64_t lda, const void* W, int64_t ldw, void* H, int64_t ldh, void* GU,
                   int64_t ldgu, int64_t M, int64_t I, int64_t K, int flags, int* err, qb_stream_t stream);
/* qkv projection fused with QK-norm + RoPE and the paged K/V store (Qwen3Attention: qkv_proj,
 * q_norm / k_norm, the Triton RoPE and store_kvcache, qwen3_naive.py:608-627, :664-669) in one GEMM:
 * the projection A . W^T ([M, N = (hq + 2 hkv) * 128], W [N, K]) is rounded to bf16 per element and
 * each 128-wide head is then normed and rotated exactly as qb_qk_norm_rope_fwd does -- the same bits.
 * Outputs, each nullable: out [M, ld_out] (rotated q, k and the v columns), raw [M, ld_raw] (the
 * bf16 projection, for a backward), q_out [M, hq, 128], k_cache / v_cache [num_slots, hkv, 128]
 * (row slot_mapping[r] <- rotated k / v of row r; -1 skips), q_rstd [M, hq] / k_rstd [M, hkv].
 * cos_sin [max_pos, 128] fp32, 16-byte aligned; norm weights 8-byte aligned; every bf16 output
 * 16-byte aligned with a leading dimension % 8 == 0.  flags: 0 or QB_GEMM_B_STATIC. */
int qb_gemm_qk_norm_rope(const void* A, int64_t lda, const void* W, int64_t ldw, int64_t M, int hq, int hkv,
                         int64_t K, const int64_t* positions, const float* cos_sin, int64_t max_pos,
                         const void* q_norm_w, const void* k_norm_w, float eps, void* out, int64_t ld_out,
                         void* raw, int64_t ld_raw, void* q_out, void* k_cache, void* v_cache,
                         const int32_t* slot_mapping, int64_t num_slots, float* q_rstd, float* k_rstd, int flags,
                         int* err, qb_stream_t stream);
/* The tile layout qb_gemm_bf16 / qb_gemm_bf16_ex choose for an M x N x K product in `mode` (B
 * MN-major or not): *pair = 1 for 256-row tiles on a CTA pair, *tile_n = the tile's width (N),
 * *split = the number of CTAs a tile's K range is split over (1: none): the CTAs of a 128 x 128
 * tile's cluster, or in mode 2 (C +=) several pairs whose partials are added to C atomically, so
 * the sum's order varies from run to run.  Needs the current device (the split layouts are sized by
 * cluster occupancy).  For tests and tuning. */
int qb_gemm_plan(int64_t M, int64_t N, int64_t K, int b_mn_major, int mode, int* pair, int* tile_n,
                 int* split);

/* ---------------------------------------------------------------- optimizer helpers
 * dst (bf16) = bf16(src fp32); used to hand fp32-accumulated gradients to the
 * reference's torch AdamW (qwen3_grpo_train.py:327) as bf16 .grad tensors. */
int qb_f32_to_bf16(const float* src, void* dst, int64_t n, qb_stream_t stream);
/* acc (fp32) += bf16 src. */
int qb_accumulate_bf16(const void* src, float* acc, int64_t n, qb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN3B200_H */
