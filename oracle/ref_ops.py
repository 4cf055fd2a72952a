"""CPU restatements of the reference's ops on the GRPO path (test infrastructure only).

All functions take and return torch CPU tensors.  bf16 rounding points follow
the reference so that the CUDA kernels can be compared at bf16 resolution.
"""
from __future__ import annotations

import math

import torch

BF16 = torch.bfloat16


def rms_norm(x, w, eps):
    """qwen3_naive.py:156-161: bf16((x_f32 * rsqrt(mean(x^2)+eps)) * w_f32)."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * w.float()).to(x.dtype)


def add_rms_norm(x, residual, w, eps):
    """qwen3_naive.py:163-169: s = x + r (fp32); residual' = bf16(s); y from s (not from residual')."""
    s = x.float() + residual.float()
    r = s.to(x.dtype)
    y = s * torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (y * w.float()).to(x.dtype), r


def rope_cache(head_dim, max_position, theta):
    """qwen3_naive.py:380-387: [max_pos, head_dim] = [cos | sin] of pos * inv_freq."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    pos = torch.arange(0, max_position, dtype=torch.float)
    freqs = torch.outer(pos, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def apply_rope(x, positions, cos_sin, out_dtype=None):
    """The Triton _apply_rope_kernel (qwen3_naive.py:53-67): half-split pairs (j, j+D/2),
    fp32 internals: o1 = x1*c - x2*s, o2 = x2*c + x1*s.  x [N, H, D]."""
    D = x.shape[-1]
    half = D // 2
    cs = cos_sin[positions.long()]
    c, s = cs[:, None, :half], cs[:, None, half:]
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    out = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return out.to(out_dtype or x.dtype)


def qk_norm_rope(qkv, positions, cos_sin, qw, kw, eps, hq, hkv, D=128):
    """qkv_proj split -> q_norm/k_norm -> RoPE (qwen3_naive.py:603-613); returns q, k, v [T, H, D] bf16."""
    T = qkv.shape[0]
    q = qkv[:, :hq * D].reshape(T, hq, D)
    k = qkv[:, hq * D:(hq + hkv) * D].reshape(T, hkv, D)
    v = qkv[:, (hq + hkv) * D:].reshape(T, hkv, D)
    q = rms_norm(q, qw, eps)
    k = rms_norm(k, kw, eps)
    return apply_rope(q, positions, cos_sin), apply_rope(k, positions, cos_sin), v


def store_kvcache(k, v, k_cache, v_cache, slot_mapping):
    """qwen3_naive.py:20-41: cache row slot <- token row; slot -1 skipped.  Caches [slots, H, D]."""
    for i, s in enumerate(slot_mapping.tolist()):
        if s == -1:
            continue
        k_cache[s] = k[i]
        v_cache[s] = v[i]


def _attend(q, k, v, scale, shift):
    """Causal attention of q [Lq, Hq, D] on k/v [Lk, Hkv, D]; query i sees keys <= shift + i.
    Scores in fp32, softmax fp32, P rounded to bf16 before P@V (flash-attn keeps P in bf16 for
    the second matmul)."""
    Lq, Hq, D = q.shape
    Lk, Hkv, _ = k.shape
    g = Hq // Hkv
    kk = k.float().repeat_interleave(g, dim=1)
    vv = v.float().repeat_interleave(g, dim=1)
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
    qi = torch.arange(Lq)[:, None] + shift
    kj = torch.arange(Lk)[None, :]
    s = s.masked_fill((kj > qi)[None], float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("hqk,khd->qhd", p.to(BF16).float(), vv)
    return o.to(q.dtype)


def paged_attention(q, k_cache, v_cache, cu_q, cu_k, block_tables, scale, page=256):
    """flash_attn_varlen_func(..., causal=True, block_table=) as called at qwen3_naive.py:631-637:
    sequence b's keys are the first Lk_b cache rows reached through its page table;
    queries are the last Lq_b positions (bottom-right causal alignment)."""
    out = torch.empty_like(q)
    cu_q, cu_k = cu_q.tolist(), cu_k.tolist()
    for b in range(len(cu_q) - 1):
        q0, q1 = cu_q[b], cu_q[b + 1]
        Lk = cu_k[b + 1] - cu_k[b]
        idx = torch.arange(Lk)
        pages = block_tables[b, idx // page].long()
        rows = pages * page + idx % page
        k = k_cache.reshape(-1, *k_cache.shape[2:])[rows]
        v = v_cache.reshape(-1, *v_cache.shape[2:])[rows]
        out[q0:q1] = _attend(q[q0:q1], k, v, scale, Lk - (q1 - q0))
    return out


def paged_decode(q, k_cache, v_cache, block_tables, cache_seqlens, scale, page=256):
    """flash_attn_with_kvcache(q[:, None], ..., cache_seqlens, block_table, causal=True)
    (qwen3_naive.py:672-680): one query per sequence over its first cache_seqlens keys."""
    B = q.shape[0]
    cu_q = torch.arange(B + 1)
    cu_k = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(cache_seqlens.long(), 0)])
    return paged_attention(q, k_cache, v_cache, cu_q, cu_k, block_tables, scale, page)


def dense_attention(q, k, v, scale):
    """Qwen3Attention.forward's manual attention for one row (qwen3_naive.py:577-589):
    bf16 q@k^T * scale, causal -inf mask, softmax in fp32 rounded to bf16, @v in bf16."""
    Lq, Hq, D = q.shape
    g = Hq // k.shape[1]
    qh = q.transpose(0, 1)
    kh = k.repeat_interleave(g, dim=1).transpose(0, 1)
    vh = v.repeat_interleave(g, dim=1).transpose(0, 1)
    s = (qh @ kh.transpose(-2, -1)) * scale
    mask = torch.triu(torch.ones(Lq, Lq), diagonal=1).bool()
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s.float(), dim=-1).to(s.dtype)
    return (p @ vh).transpose(0, 1)


def silu_mul(gate_up):
    """Qwen3MLP.forward's silu(gate) * up with gate = first half (qwen3_naive.py:698-700), fp32 inside."""
    I = gate_up.shape[-1] // 2
    g, u = gate_up[..., :I].float(), gate_up[..., I:].float()
    return (torch.nn.functional.silu(g) * u).to(gate_up.dtype)


def log_probs(logits, targets):
    """forward_logprob's log_softmax(logits.float()).gather (qwen3_grpo_train.py:49-52)."""
    return torch.log_softmax(logits.float(), dim=-1).gather(-1, targets.long().unsqueeze(-1)).squeeze(-1)


def sample_distribution(logits, temperature, top_k):
    """The distribution generate_continuous_with_logprobs samples from (qwen3_naive.py:1632-1646):
    softmax of logits/T restricted to the top_k entries; returns (probs, log_probs).

    bf16 logits tie often; torch.topk keeps an unspecified member of a tie at the k-th
    value.  Here ties are broken toward the lower index (a stable descending sort), the
    rule the CUDA sampler uses; the kept *values*, hence every log-prob, are the same
    either way."""
    x = logits.float() / temperature
    if top_k is not None:
        order = torch.sort(x, dim=-1, descending=True, stable=True).indices[..., :top_k]
        x = torch.full_like(x, float("-inf")).scatter(-1, order, x.gather(-1, order))
    return torch.softmax(x, dim=-1), torch.log_softmax(x, dim=-1)


# ---------------------------------------------------------------- GRPO math
def grpo_advantage(rewards, prompt_ids):
    """compute_grpo_advantage (qwen3_grpo_train.py:162-173): per group (r - mean)/(std + 1e-8),
    std unbiased."""
    adv = torch.empty_like(rewards)
    for pid in prompt_ids.unique():
        m = prompt_ids == pid
        g = rewards[m]
        adv[m] = (g - g.mean()) / (g.std() + 1e-8)
    return adv


def ppo_loss(old, new, adv_tok, mask, clip_eps=0.2, ref=None, beta=0.0):
    """ppo_clipped_loss (qwen3_grpo_train.py:193-199) plus beta * k3 KL (GRPO paper's
    unbiased estimator exp(ref-new) - (ref-new) - 1, masked token mean with the same
    denominator).  Differentiable in ``new`` through torch autograd."""
    ratio = (new - old).exp()
    clipped = ratio.clamp(1.0 - clip_eps, 1.0 + clip_eps)
    lt = -torch.min(ratio * adv_tok, clipped * adv_tok)
    denom = mask.sum() + 1e-8
    loss = (lt * mask).sum() / denom
    if ref is not None and beta != 0.0:
        d = ref - new
        kl = d.exp() - d - 1.0
        loss = loss + beta * (kl * mask).sum() / denom
    return loss


def grpo_loss_and_grad(rewards, group_ids, new, old, mask, ref=None, beta=0.0, clip_eps=0.2):
    """advantages -> token advantages (x mask) -> loss; returns (loss, d loss / d new, adv)."""
    adv = grpo_advantage(rewards.float(), group_ids)
    tok = adv[:, None] * mask
    new = new.detach().clone().requires_grad_(True)
    loss = ppo_loss(old, new, tok, mask, clip_eps, ref, beta)
    loss.backward()
    return loss.detach(), new.grad, adv
