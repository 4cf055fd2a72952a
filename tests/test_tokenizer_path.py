"""The tokenizer / chat-template prompt path beside load_weights, on the CPU.

The reference builds its prompts by rendering one user turn through the tokenizer's chat
template with the generation prompt appended and encoding the result
(test_prefix_cache.py:37-43, qwen3_grpo_train.py:317-324), loads tokenizer, config and weights
from one checkpoint directory (test_prefix_cache.py:22-35), and scores a rollout by decoding the
completion with special tokens skipped (qwen3_grpo_train.py:229-232, :141-151).  No Qwen3
tokenizer exists in this container, so a small word-level tokenizer with a ChatML template (the
format of Qwen3's template) stands in for it; the checkpoint is a synthetic safetensors file.
"""
import json

import torch

from qwen3_naive_inference_b200 import qwen3_grpo_train as G
from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config, load_model_and_tokenizer, tokenize

from test_load_weights import write_safetensors  # tests/ is on sys.path (rootdir conftest)

CHATML = ("{% for m in messages %}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n{% endfor %}"
          "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}")
WORDS = ["user", "assistant", "what", "is", "the", "capital", "of", "france", "?", "paris", "it"]
SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]


def make_tokenizer(path):
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast
    vocab = {w: i for i, w in enumerate(SPECIAL + ["[UNK]"] + WORDS)}
    tok = Tokenizer(models.WordLevel(vocab=vocab, unk_token="[UNK]"))
    tok.pre_tokenizer = pre_tokenizers.Sequence([pre_tokenizers.WhitespaceSplit(), pre_tokenizers.Punctuation()])
    fast = PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="[UNK]", eos_token="<|im_end|>",
                                   pad_token="<|endoftext|>", additional_special_tokens=SPECIAL[1:])
    fast.chat_template = CHATML
    fast.save_pretrained(str(path))
    return vocab


def test_tokenize_renders_the_chat_template(tmp_path):
    from transformers import AutoTokenizer
    vocab = make_tokenizer(tmp_path)
    tok = AutoTokenizer.from_pretrained(str(tmp_path))
    ids = tokenize("what is the capital of france?", tok)
    expect = ["<|im_start|>", "user", "what", "is", "the", "capital", "of", "france", "?", "<|im_end|>",
              "<|im_start|>", "assistant"]
    assert ids.dtype == torch.long and ids.shape == (1, len(expect))
    assert ids[0].tolist() == [vocab[w] for w in expect]


def test_reward_decodes_the_completion_without_special_tokens(tmp_path):
    from transformers import AutoTokenizer
    vocab = make_tokenizer(tmp_path)
    tok = AutoTokenizer.from_pretrained(str(tmp_path))
    assert G.compute_reward("  paris  ") == 0.0 and G.compute_reward("it is paris") == 1.0
    long_answer = [vocab[w] for w in ("it", "is", "paris")] + [vocab["<|im_end|>"]]
    short_answer = [vocab["paris"], vocab["<|im_end|>"], vocab["<|im_end|>"]]
    assert G._reward(tok, long_answer, None) == 1.0    # "it is paris"
    assert G._reward(tok, short_answer, None) == 0.0   # "paris": the stop tokens do not count
    assert G._reward(None, short_answer, None) == 0.0  # no tokenizer: the rule on the token count
    assert G._reward(None, long_answer * 2, None) == 1.0
    assert G._reward(tok, short_answer, lambda c: 0.5) == 0.5


def test_load_model_and_tokenizer_from_one_directory(tmp_path):
    make_tokenizer(tmp_path)
    cfg = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=128,
               intermediate_size=256, num_hidden_layers=1, vocab_size=64, max_position_embeddings=512,
               rms_norm_eps=1e-6, rope_theta=1e6, tie_word_embeddings=True, hidden_act="silu",
               attention_bias=False, bos_token_id=151643, eos_token_id=151645, torch_dtype="bfloat16")
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    g = torch.Generator().manual_seed(0)
    rnd = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)
    ck = {"model.embed_tokens.weight": rnd(64, 256), "model.norm.weight": rnd(256),
          "model.layers.0.input_layernorm.weight": rnd(256),
          "model.layers.0.post_attention_layernorm.weight": rnd(256),
          "model.layers.0.self_attn.q_proj.weight": rnd(512, 256),
          "model.layers.0.self_attn.k_proj.weight": rnd(256, 256),
          "model.layers.0.self_attn.v_proj.weight": rnd(256, 256),
          "model.layers.0.self_attn.o_proj.weight": rnd(256, 512),
          "model.layers.0.self_attn.q_norm.weight": rnd(128), "model.layers.0.self_attn.k_norm.weight": rnd(128),
          "model.layers.0.mlp.gate_proj.weight": rnd(256, 256), "model.layers.0.mlp.up_proj.weight": rnd(256, 256),
          "model.layers.0.mlp.down_proj.weight": rnd(256, 256)}
    write_safetensors(tmp_path / "model.safetensors", ck)
    model, tok, config = load_model_and_tokenizer(str(tmp_path), device="cpu")
    assert isinstance(config, Qwen3Config) and config.vocab_size == 64 and config.num_hidden_layers == 1
    assert torch.equal(model.model.embed_tokens.weight, ck["model.embed_tokens.weight"])
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()
    qkv = model.model.layers[0].self_attn.qkv_proj.weight
    assert torch.equal(qkv[512:768], ck["model.layers.0.self_attn.k_proj.weight"])
    assert tokenize("what is paris", tok).shape[1] == 8  # <|im_start|> user what is paris <|im_end|> <|im_start|> assistant
