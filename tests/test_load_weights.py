"""load_weights (reference qwen3_naive.py:1682-1730) on a synthetic single-file safetensors
checkpoint with the Hugging Face Qwen3 tensor names, on the CPU: q/k/v rows are packed into
qkv_proj in that order and gate/up rows into gate_up_proj (the reference's packed_modules_mapping,
:814-820), every other tensor is copied by name (bf16, f16 and f32 entries), and lm_head.weight is
skipped, so the tied lm_head keeps the embedding's values."""
import json
import struct

import torch

from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config, build_model, load_weights

DTYPE_NAMES = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32"}


def write_safetensors(path, tensors):
    """8-byte little-endian header length, JSON header of {name: dtype, shape, data_offsets}, data."""
    header, blobs, off = {"__metadata__": {"format": "pt"}}, [], 0
    for name, t in tensors.items():
        raw = t.contiguous().view(torch.uint8).numpy().tobytes()
        header[name] = {"dtype": DTYPE_NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode("utf-8")
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        f.write(b"".join(blobs))


def test_load_weights_packs_fused_projections_and_copies_the_rest(tmp_path):
    d, hd, hq, hkv, inter, vocab, n_layers = 256, 128, 4, 2, 384, 512, 2
    cfg = Qwen3Config(hidden_size=d, num_attention_heads=hq, num_key_value_heads=hkv, head_dim=hd,
                      intermediate_size=inter, num_hidden_layers=n_layers, vocab_size=vocab,
                      max_position_embeddings=2048)
    model = build_model(cfg, device="cpu", seed=0)
    g = torch.Generator().manual_seed(3)

    def rnd(*shape, dtype=torch.bfloat16):
        return torch.randn(*shape, generator=g).to(dtype)

    ck = {"model.embed_tokens.weight": rnd(vocab, d), "model.norm.weight": rnd(d, dtype=torch.float32),
          "lm_head.weight": rnd(vocab, d)}
    for i in range(n_layers):
        p = f"model.layers.{i}."
        ck.update({p + "self_attn.q_proj.weight": rnd(hq * hd, d), p + "self_attn.k_proj.weight": rnd(hkv * hd, d),
                   p + "self_attn.v_proj.weight": rnd(hkv * hd, d), p + "self_attn.o_proj.weight": rnd(d, hq * hd),
                   p + "self_attn.q_norm.weight": rnd(hd, dtype=torch.float16),
                   p + "self_attn.k_norm.weight": rnd(hd, dtype=torch.float16),
                   p + "mlp.gate_proj.weight": rnd(inter, d), p + "mlp.up_proj.weight": rnd(inter, d),
                   p + "mlp.down_proj.weight": rnd(d, inter), p + "input_layernorm.weight": rnd(d),
                   p + "post_attention_layernorm.weight": rnd(d)})
    path = tmp_path / "model.safetensors"
    write_safetensors(path, ck)
    load_weights(model, str(path))

    sd = dict(model.named_parameters())
    for i in range(n_layers):
        p = f"model.layers.{i}."
        qkv = torch.cat([ck[p + "self_attn.q_proj.weight"], ck[p + "self_attn.k_proj.weight"],
                         ck[p + "self_attn.v_proj.weight"]])
        assert torch.equal(sd[p + "self_attn.qkv_proj.weight"], qkv)
        gate_up = torch.cat([ck[p + "mlp.gate_proj.weight"], ck[p + "mlp.up_proj.weight"]])
        assert torch.equal(sd[p + "mlp.gate_up_proj.weight"], gate_up)
        for name in ("self_attn.o_proj.weight", "mlp.down_proj.weight", "input_layernorm.weight",
                     "post_attention_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight"):
            assert torch.equal(sd[p + name], ck[p + name].to(torch.bfloat16)), name
    assert torch.equal(sd["model.norm.weight"], ck["model.norm.weight"].to(torch.bfloat16))
    assert torch.equal(sd["model.embed_tokens.weight"], ck["model.embed_tokens.weight"])
    # tied: lm_head shares the embedding's storage, the checkpoint's lm_head.weight is not read
    assert torch.equal(sd["lm_head.weight"], ck["model.embed_tokens.weight"])
    assert not torch.equal(sd["lm_head.weight"], ck["lm_head.weight"])
