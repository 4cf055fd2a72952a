"""Pins the CPU oracle against golden vectors recorded from the reference (CPU only).

The RoPE and KV-store goldens come from the reference's own Triton kernels (run in
Triton's CPU interpreter); the GRPO and model goldens from the reference's PyTorch code.
"""
from pathlib import Path

import pytest
import torch

from oracle import ref_model
from oracle import ref_ops as R
from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config

GOLD = Path(__file__).parent / "golden"


def load(name):
    return torch.load(GOLD / name, weights_only=False)


def test_rope_matches_reference_kernel_exactly():
    g = load("kernels.pt")
    cs = R.rope_cache(128, 4096, 1e6)
    assert torch.equal(cs[4095], g["rope_cache_row_4095"])
    out = R.apply_rope(g["rope_x"], g["rope_pos"], cs, torch.float32)
    assert torch.equal(out, g["rope_out_fp32"])


def test_store_kvcache_matches_reference_kernel():
    g = load("kernels.pt")
    kc = torch.zeros_like(g["store_kc"])
    vc = torch.zeros_like(g["store_vc"])
    R.store_kvcache(g["store_k"], g["store_v"], kc, vc, g["store_slots"])
    assert torch.equal(kc, g["store_kc"]) and torch.equal(vc, g["store_vc"])


def test_grpo_math_matches_reference():
    g = load("grpo.pt")
    adv = R.grpo_advantage(g["rewards"], g["prompt_ids"])
    assert torch.allclose(adv, g["adv"], rtol=1e-6, atol=1e-7)
    loss, grad, adv2 = R.grpo_loss_and_grad(g["rewards"], g["prompt_ids"], g["new"], g["old"], g["mask"])
    assert torch.equal(adv2, adv)
    assert torch.allclose(loss, g["loss"], rtol=1e-6)
    assert torch.allclose(grad, g["grad_new"], rtol=1e-6, atol=1e-9)


@pytest.fixture(scope="module")
def tiny():
    g = load("model_tiny.pt")
    cfg = Qwen3Config(**g["config"])
    params = ref_model.init_params(cfg, seed=0)
    return g, cfg, params


def test_model_logits_match_reference(tiny):
    """The oracle's dense logits equal the reference's bit for bit (same bf16 rounding points)."""
    g, cfg, params = tiny
    with torch.no_grad():
        lg = ref_model.logits(params, cfg, g["ids"])
    assert torch.equal(lg, g["logits"])


def test_model_logprob_and_grads_match_reference(tiny):
    g, cfg, params = tiny
    p = {k: v.clone().requires_grad_(True) for k, v in params.items() if k != "lm_head.weight"}
    p["lm_head.weight"] = params["lm_head.weight"].clone().requires_grad_(True)  # separate Parameter, shared data
    lp = ref_model.forward_logprob(p, cfg, g["ids"], rope_grad=False)
    assert torch.equal(lp, g["logprob"])
    adv_tok = g["tok_adv"]
    loss = R.ppo_loss(g["old"], lp, adv_tok, g["mask"])
    assert torch.equal(loss.detach(), g["loss"])
    loss.backward()
    for name, gr in g["grads"].items():
        mine = p[name].grad
        if gr is None:  # the reference's RoPE quirk: q_norm / k_norm get no grad at all
            assert mine is None, name
            continue
        assert torch.equal(mine, gr), name


def test_reference_rope_quirk_blocks_qk_grads(tiny):
    """In the reference, q/k rows of qkv_proj get zero grad and q_norm/k_norm none."""
    g, cfg, _ = tiny
    qkv = g["grads"]["model.layers.0.self_attn.qkv_proj.weight"].float()
    hq, hkv, D = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    assert qkv[:(hq + hkv) * D].abs().max().item() == 0.0
    assert qkv[(hq + hkv) * D:].abs().max().item() > 0.0
    assert g["grads"]["model.layers.0.self_attn.q_norm.weight"] is None
