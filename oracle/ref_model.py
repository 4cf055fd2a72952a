"""CPU restatement of the reference's dense Qwen3 forward (test infrastructure only).

Follows Qwen3ForCausalLM.forward -> Qwen3Model.forward -> Qwen3DecoderLayer.forward ->
Qwen3Attention.forward (qwen3_naive.py:833-835, :770-776, :715-719, :553-593) with the
RoPE of the Triton kernel (:53-67), in torch on the CPU, differentiable, on a parameter
dict named like the product model's ``state_dict()``.
"""
from __future__ import annotations

import torch

from . import ref_ops as R


def init_params(cfg, seed=0, std=0.02, dtype=torch.bfloat16):
    """N(0, std) weights for every Linear and the embedding, RMSNorm weights 1 (seeded, CPU)."""
    g = torch.Generator().manual_seed(seed)
    H, I, V, D = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.head_dim
    hq, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    rnd = lambda *s: (torch.randn(*s, generator=g) * std).to(dtype)
    p = {"model.embed_tokens.weight": rnd(V, H)}
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}."
        p[pre + "input_layernorm.weight"] = torch.ones(H, dtype=dtype)
        p[pre + "self_attn.qkv_proj.weight"] = rnd((hq + 2 * hkv) * D, H)
        p[pre + "self_attn.o_proj.weight"] = rnd(H, hq * D)
        p[pre + "self_attn.q_norm.weight"] = torch.ones(D, dtype=dtype)
        p[pre + "self_attn.k_norm.weight"] = torch.ones(D, dtype=dtype)
        p[pre + "post_attention_layernorm.weight"] = torch.ones(H, dtype=dtype)
        p[pre + "mlp.gate_up_proj.weight"] = rnd(2 * I, H)
        p[pre + "mlp.down_proj.weight"] = rnd(H, I)
    p["model.norm.weight"] = torch.ones(H, dtype=dtype)
    p["lm_head.weight"] = p["model.embed_tokens.weight"]
    return p


def hidden(params, cfg, ids, cos_sin=None, rope_grad=True):
    """Final-norm hidden states [B, S, H] of the dense forward."""
    B, S = ids.shape
    D, hq, hkv, eps = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.rms_norm_eps
    if cos_sin is None:
        cos_sin = R.rope_cache(D, max(S, 1), cfg.rope_theta)
    pos = torch.arange(S)
    h = params["model.embed_tokens.weight"][ids]
    for i in range(cfg.num_hidden_layers):
        pre = f"model.layers.{i}."
        x = h
        n = R.rms_norm(x, params[pre + "input_layernorm.weight"], eps)
        qkv = n @ params[pre + "self_attn.qkv_proj.weight"].t()
        outs = []
        for b in range(B):
            q, k, v = R.qk_norm_rope(qkv[b], pos, cos_sin, params[pre + "self_attn.q_norm.weight"],
                                     params[pre + "self_attn.k_norm.weight"], eps, hq, hkv, D)
            if not rope_grad:  # the reference's Triton RoPE is invisible to autograd
                q, k = q.detach(), k.detach()
            outs.append(R.dense_attention(q, k, v, D ** -0.5).reshape(S, hq * D))
        o = torch.stack(outs)
        h = o @ params[pre + "self_attn.o_proj.weight"].t() + x
        n2 = R.rms_norm(h, params[pre + "post_attention_layernorm.weight"], eps)
        gu = n2 @ params[pre + "mlp.gate_up_proj.weight"].t()
        h = R.silu_mul(gu) @ params[pre + "mlp.down_proj.weight"].t() + h
    return R.rms_norm(h, params["model.norm.weight"], eps)


def logits(params, cfg, ids, **kw):
    """Dense logits [B, S, V] (bf16)."""
    return hidden(params, cfg, ids, **kw) @ params["lm_head.weight"].t()


def forward_logprob(params, cfg, ids, shift=False, **kw):
    """forward_logprob (qwen3_grpo_train.py:46-53); shift=True scores token t from position t-1."""
    lg = logits(params, cfg, ids, **kw)
    if not shift:
        return R.log_probs(lg, ids)
    lp = R.log_probs(lg[:, :-1], ids[:, 1:])
    return torch.cat([torch.zeros(ids.shape[0], 1), lp], dim=1)
