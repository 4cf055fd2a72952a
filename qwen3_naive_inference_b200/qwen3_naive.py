"""Qwen3 model, paged KV cache and continuous-batching rollout on B200 kernels.

Drop-in for the reference module ``qwen3_naive.py``: same class names,
constructor arguments, public methods, return types and scheduler semantics
(decode-first, 2048-token budget, chunked prefill, LIFO preemption, prefix
caching through ``BlockManager``).  Under the API every op is a kernel of
``libqwen3b200.so`` (see :mod:`.ops`): RMSNorm, QK-Norm+RoPE fused with the
paged KV store, paged prefill/decode attention, SwiGLU, sampling; dense
projections go through :func:`.ops.linear`.

Differences from the reference that do not change observable results:
  * lm_head runs only on the rows that are sampled (the reference's
    ``generate_continuous_with_logprobs`` projects every row, qwen3_naive.py:1607);
  * decode steps of any batch size up to 512 replay a CUDA graph that also
    contains lm_head and the sampler, and each step makes one device->host copy
    (the reference syncs per sequence, qwen3_naive.py:1656,1659);
  * sampling is Gumbel-max on a Philox stream instead of torch.multinomial, so
    sampled tokens match the reference in distribution (greedy, top_k=1, exactly).
"""
from __future__ import annotations

import json
import math
import time
from collections import deque
from dataclasses import dataclass
from functools import lru_cache

import numpy as np
import torch
import torch.nn as nn

from . import _lib, ops


def _pdl_mode() -> int:
    """The library's launch mode (programmatic dependent launch on/off): captured decode graphs
    record it, so a change recaptures them."""
    return int(_lib.load().qb_get_pdl())


# ============================================================================ config
@dataclass
class Qwen3Config:
    """Model shape; field names and defaults follow qwen3_naive.py:109-148."""
    hidden_size: int = 1024
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    vocab_size: int = 151936
    max_position_embeddings: int = 40960
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000
    attention_bias: bool = False
    hidden_act: str = "silu"
    tie_word_embeddings: bool = True
    bos_token_id: int = 151643
    eos_token_id: int = 151645
    dtype: str = "bfloat16"

    @classmethod
    def from_json(cls, path):
        """Reads a HuggingFace ``config.json`` (qwen3_naive.py:128-148)."""
        with open(path, "r") as f:
            d = json.load(f)
        return cls(
            hidden_size=d["hidden_size"],
            num_attention_heads=d["num_attention_heads"],
            num_key_value_heads=d["num_key_value_heads"],
            head_dim=d.get("head_dim", d["hidden_size"] // d["num_attention_heads"]),
            intermediate_size=d["intermediate_size"],
            num_hidden_layers=d["num_hidden_layers"],
            vocab_size=d["vocab_size"],
            max_position_embeddings=d["max_position_embeddings"],
            rms_norm_eps=d["rms_norm_eps"],
            rope_theta=d.get("rope_theta", 1000000),
            attention_bias=d.get("attention_bias", False),
            hidden_act=d["hidden_act"],
            tie_word_embeddings=d.get("tie_word_embeddings", True),
            bos_token_id=d.get("bos_token_id", 151643),
            eos_token_id=d.get("eos_token_id", 151645),
        )


# ============================================================================ paging
class Sequence:
    """State of one request (qwen3_naive.py:191-237): token ids, KV length, page table."""

    BLOCK_SIZE = 256

    def __init__(self, token_ids: list[int], sampling_params: dict = None):
        self.token_ids = list(token_ids)
        self.num_prompt_tokens = len(token_ids)
        self.last_token = token_ids[-1]
        self.status = "WAITING"
        self.block_table: list[int] = []
        self.kv_len = 0                  # tokens whose K/V are in the cache
        self.num_scheduled_tokens = 0    # tokens computed in the current step
        sp = sampling_params or {}
        self.temperature = sp.get("temperature", 0.6)
        self.max_tokens = sp.get("max_tokens", 256)
        self.response_log_probs: list[float] = []

    def append_token(self, token_id: int):
        self.token_ids.append(token_id)
        self.last_token = token_id

    @property
    def num_tokens(self):
        return len(self.token_ids)

    @property
    def num_blocks(self):
        return -(-len(self.token_ids) // self.BLOCK_SIZE)

    def block(self, i: int) -> list[int]:
        """Token ids of logical page i (the input of the prefix-cache hash)."""
        return self.token_ids[i * self.BLOCK_SIZE:(i + 1) * self.BLOCK_SIZE]

    @property
    def num_completion_tokens(self):
        return len(self.token_ids) - self.num_prompt_tokens

    @property
    def unfinished(self):
        return self.status != "FINISHED"

    @property
    def prompt_len(self):
        return self.num_prompt_tokens


class BlockManager:
    """Page allocator with reference counts and a chained-hash prefix cache.

    Observable behaviour equals qwen3_naive.py:240-375: ``free`` is a list used
    as a stack (allocation pops from the end, release appends), a freed page
    keeps its hash so a later prompt with the same prefix can reuse it, and the
    hash of page i is the 64-bit djb2-xor chain over its token ids seeded with
    the hash of page i-1.  The fields are public because callers (and the
    reference's tests) inspect and reset them directly.
    """

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free = list(range(num_blocks))
        self.ref_count = [0] * num_blocks
        self.block_hash = [-1] * num_blocks
        self.block_tokens = [None] * num_blocks
        self.hash_to_block: dict[int, int] = {}

    @staticmethod
    def compute_hash(token_ids: list[int], prefix_hash: int = -1) -> int:
        """h <- 33*h XOR t over the tokens, from the previous page's hash (0 for
        the first page), reduced to 64 bits (qwen3_naive.py:260-267).  Python
        integers are unbounded, so the running value is folded to 64 bits as it
        goes; the low 64 bits of 33*h ^ t depend only on the low 64 bits of h,
        so the result is identical."""
        mask = 0xFFFFFFFFFFFFFFFF
        h = 0 if prefix_hash == -1 else prefix_hash & mask
        for t in token_ids:
            h = ((h * 33) ^ t) & mask
        return h

    def _take_free(self, blk: int | None = None) -> int:
        if blk is None:
            blk = self.free.pop()
        old = self.block_hash[blk]
        if old != -1:  # the page is recycled: forget its cached content
            if self.hash_to_block.get(old) == blk:
                del self.hash_to_block[old]
            self.block_hash[blk] = -1
            self.block_tokens[blk] = None
        self.ref_count[blk] = 1
        return blk

    def allocate(self, seq: Sequence):
        """Give ``seq`` pages for its current tokens, sharing cached full prefix pages."""
        assert not seq.block_table, "block_table must be empty"
        h = -1
        cached = 0
        for i in range(seq.num_blocks - 1):  # the last (maybe partial) page is never shared
            toks = seq.block(i)
            h = self.compute_hash(toks, h)
            blk = self.hash_to_block.get(h, -1)
            if blk == -1 or self.block_tokens[blk] != toks:
                break
            cached += 1
            if blk in self.free:
                self.free.remove(blk)
            self.ref_count[blk] += 1
            seq.block_table.append(blk)
        for _ in range(cached, seq.num_blocks):
            seq.block_table.append(self._take_free())
        seq.kv_len = cached * self.block_size

    def deallocate(self, block_table: list[int]):
        """Drop one reference per page; pages reaching zero return to ``free`` with their hash kept."""
        for b in block_table:
            self.ref_count[b] -= 1
            if self.ref_count[b] == 0:
                self.free.append(b)

    def can_append(self, seq: Sequence) -> bool:
        """True unless writing K/V at position ``kv_len`` needs a page and none is free."""
        return seq.kv_len % self.block_size != 0 or len(self.free) > 0

    def may_append(self, seq: Sequence):
        """Append a fresh page when ``kv_len`` sits on a page boundary."""
        if seq.kv_len % self.block_size == 0:
            seq.block_table.append(self._take_free())

    def hash_blocks(self, seq: Sequence):
        """Register the pages completed by this step's ``num_scheduled_tokens`` in the prefix cache."""
        bs = self.block_size
        first = (seq.kv_len - seq.num_scheduled_tokens) // bs
        last = seq.kv_len // bs
        if first >= last:
            return
        h = self.block_hash[seq.block_table[first - 1]] if first > 0 else -1
        for i in range(first, last):
            blk = seq.block_table[i]
            toks = seq.block(i)
            h = self.compute_hash(toks, h)
            self.block_hash[blk] = h
            self.block_tokens[blk] = toks
            self.hash_to_block[h] = blk

    @property
    def available(self):
        return len(self.free)


# ============================================================================ modules
class RMSNorm(nn.Module):
    """RMSNorm with the reference's rounding points (qwen3_naive.py:150-175)."""

    def __init__(self, hidden_size, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def forward(self, x, residual=None):
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps)
        return ops.add_rmsnorm(x, residual, self.weight, self.eps)


class RotaryEmbedding(nn.Module):
    """fp32 table [max_position, head_dim] = [cos | sin] of pos * theta^(-2i/d) (qwen3_naive.py:380-387).

    The table is built with the same torch expressions as the reference so that it
    is bit-identical on the same device; the rotation itself runs inside the fused
    QK-Norm+RoPE kernel.
    """

    def __init__(self, head_dim, max_position, rope_theta):
        super().__init__()
        inv_freq = 1.0 / (rope_theta ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
        pos = torch.arange(0, max_position, dtype=torch.float)
        freqs = torch.outer(pos, inv_freq)
        self.register_buffer("cos_sin_cache", torch.cat((freqs.cos(), freqs.sin()), dim=-1))


@lru_cache(8)
def get_rope(head_dim: int, max_position: int, rope_theta: float):
    return RotaryEmbedding(head_dim, max_position, rope_theta)


class Qwen3Attention(nn.Module):
    """GQA attention with QK-Norm and RoPE (qwen3_naive.py:413-683)."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.head_dim = config.head_dim
        self.hidden_size = config.hidden_size
        self.q_size = self.num_heads * self.head_dim
        self.kv_size = self.num_kv_heads * self.head_dim
        self.scale = self.head_dim ** -0.5
        self.eps = config.rms_norm_eps
        self.qkv_proj = nn.Linear(self.hidden_size, self.q_size + 2 * self.kv_size, bias=config.attention_bias)
        self.o_proj = nn.Linear(self.q_size, self.hidden_size, bias=False)
        self.q_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_norm = RMSNorm(self.head_dim, eps=config.rms_norm_eps)
        self.k_cache = None
        self.v_cache = None
        self.rotary_emb = get_rope(self.head_dim, config.max_position_embeddings, config.rope_theta)
        self.rope_grad = True  # False reproduces the reference's gradient-blocking RoPE

    def _cos_sin(self, device):
        cs = self.rotary_emb.cos_sin_cache
        if cs.device != device:
            self.rotary_emb.cos_sin_cache = cs = cs.to(device)
        return cs

    def forward_packed(self, x, positions, cu_seqlens, tiles):
        """Training/recompute path over packed sequences (each attends only to itself)."""
        # projection, then QK-norm + RoPE + attention as one node (the GEMM with QK-norm in its epilogue,
        # ops.qkv_attention, is slower at training sizes: its row-per-thread epilogue throttles the LSU)
        qkv = ops.linear(x, self.qkv_proj.weight)
        o = ops.qk_norm_rope_attention(qkv, positions, self._cos_sin(x.device), self.q_norm.weight,
                                       self.k_norm.weight, self.eps, cu_seqlens, tiles, self.num_heads,
                                       self.num_kv_heads, self.scale, rope_grad=self.rope_grad)
        return ops.linear(o, self.o_proj.weight)

    def forward(self, x):
        """Dense path on [batch, seq, hidden] (qwen3_naive.py:553-593): causal per row."""
        B, S, H = x.shape
        positions, cu, tiles = _dense_meta(B, S, x.device)
        return self.forward_packed(x.reshape(B * S, H), positions, cu, tiles).view(B, S, H)

    def forward_prefill(self, x, positions, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                        block_mapping, block_tables=None, *, tiles=None, decode_tail=None):
        """Paged prefill (qwen3_naive.py:597-640): K/V of the new tokens go to the cache rows
        ``block_mapping``, then queries attend to the cache through ``block_tables``.

        ``decode_tail`` = (n_prefill_rows, context_lens, block_tables, decode_plan): the rows from
        n_prefill_rows on are single decode tokens whose attention runs on the decode kernel of
        ``decode_plan`` (cu_seqlens and ``block_tables`` then describe the prefill rows only)."""
        # qkv projection with QK-norm, RoPE and the K/V store in the GEMM's epilogue
        q = ops.qkv_norm_rope_store(x, self.qkv_proj.weight, positions, self._cos_sin(x.device), self.q_norm.weight,
                                    self.k_norm.weight, self.eps, self.num_heads, self.num_kv_heads, self.k_cache,
                                    self.v_cache, block_mapping)
        if block_tables is None:
            raise ValueError("the paged prefill kernel reads K/V through block_tables")
        if decode_tail is None:
            o = ops.attention_paged_prefill(q, self.k_cache, self.v_cache, cu_seqlens_q, cu_seqlens_k,
                                            max_seqlen_q, block_tables, self.scale, tiles=tiles)
        else:
            tp, context_lens, bt_d, plan = decode_tail
            o = torch.empty_like(q)
            if tp:
                ops.attention_paged_prefill(q[:tp], self.k_cache, self.v_cache, cu_seqlens_q, cu_seqlens_k,
                                            max_seqlen_q, block_tables, self.scale, tiles=tiles, out=o[:tp])
            self._decode_attention(q[tp:], context_lens, bt_d, plan, out=o[tp:])
        return ops.linear(o.view(x.shape[0], -1), self.o_proj.weight)

    def _decode_attention(self, q, context_lens, block_tables, decode_plan, out=None):
        if decode_plan is None:
            o = ops.paged_decode_attention(q, self.k_cache, self.v_cache, block_tables, context_lens, self.scale)
        elif decode_plan[0] == "grouped":
            # prompt pages shared by G completions: read once per group (shared-prefix decode)
            _, plan, ws, members, shared_len, kv_start = decode_plan
            return ops.paged_decode_attention_grouped(q, self.k_cache, self.v_cache, block_tables, context_lens,
                                                      self.scale, members, shared_len, kv_start, plan, workspace=ws,
                                                      out=out)
        else:
            _, split_tokens, max_splits, ws = decode_plan
            o = ops.paged_decode_attention(q, self.k_cache, self.v_cache, block_tables, context_lens, self.scale,
                                           split_tokens=split_tokens, max_splits=max_splits, workspace=ws)
        if out is not None:
            out.copy_(o)
            return out
        return o

    def forward_decode(self, x, positions, context_lens, block_tables, slot_mapping=None, *, decode_plan=None):
        """One new token per sequence (qwen3_naive.py:642-683); attends to context_lens + 1 keys."""
        if slot_mapping is None:
            raise ValueError("the decode step stores the new token's K/V through slot_mapping")
        q = ops.qkv_norm_rope_store(x, self.qkv_proj.weight, positions, self._cos_sin(x.device), self.q_norm.weight,
                                    self.k_norm.weight, self.eps, self.num_heads, self.num_kv_heads, self.k_cache,
                                    self.v_cache, slot_mapping)
        o = self._decode_attention(q, context_lens, block_tables, decode_plan)
        return ops.linear(o.view(x.shape[0], -1), self.o_proj.weight)


class Qwen3MLP(nn.Module):
    """SwiGLU with fused gate/up projection (qwen3_naive.py:686-702)."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.gate_up_proj = nn.Linear(config.hidden_size, 2 * config.intermediate_size, bias=False)
        self.down_proj = nn.Linear(config.intermediate_size, config.hidden_size, bias=False)

    def forward(self, x):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        h = ops.swiglu_linear(x2, self.gate_up_proj.weight)  # gate_up GEMM with SwiGLU in its epilogue
        return ops.linear(h, self.down_proj.weight).view(*shape[:-1], -1)


class Qwen3DecoderLayer(nn.Module):
    """Pre-norm block (qwen3_naive.py:705-756)."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.input_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.self_attn = Qwen3Attention(config)
        self.post_attention_layernorm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.mlp = Qwen3MLP(config)

    def forward_packed(self, x, positions, cu_seqlens, tiles):
        # bf16 residual adds, as the reference's dense path (qwen3_naive.py:715-719)
        x = ops.add(self.self_attn.forward_packed(self.input_layernorm(x), positions, cu_seqlens, tiles), x)
        return ops.add(self.mlp(self.post_attention_layernorm(x)), x)

    def forward(self, x):
        B, S, H = x.shape
        positions, cu, tiles = _dense_meta(B, S, x.device)
        return self.forward_packed(x.reshape(B * S, H), positions, cu, tiles).view(B, S, H)

    def forward_prefill(self, x, positions, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                        block_mapping, block_tables=None, residual=None, *, tiles=None, decode_tail=None):
        if residual is None:
            hidden_states, residual = self.input_layernorm(x), x
        else:
            hidden_states, residual = self.input_layernorm(x, residual)
        hidden_states = self.self_attn.forward_prefill(hidden_states, positions, cu_seqlens_q, cu_seqlens_k,
                                                       max_seqlen_q, max_seqlen_k, block_mapping, block_tables,
                                                       tiles=tiles, decode_tail=decode_tail)
        hidden_states, residual = self.post_attention_layernorm(hidden_states, residual)
        return self.mlp(hidden_states), residual

    def forward_decode(self, x, positions, context_lens, block_tables, slot_mapping=None, residual=None, *,
                       decode_plan=None):
        if residual is None:
            hidden_states, residual = self.input_layernorm(x), x
        else:
            hidden_states, residual = self.input_layernorm(x, residual)
        hidden_states = self.self_attn.forward_decode(hidden_states, positions, context_lens, block_tables,
                                                      slot_mapping, decode_plan=decode_plan)
        hidden_states, residual = self.post_attention_layernorm(hidden_states, residual)
        return self.mlp(hidden_states), residual


_DENSE_META: dict = {}


def _dense_meta(B: int, S: int, device):
    """Positions / cu_seqlens / tiles for B rows of S tokens (cached per shape)."""
    key = (B, S, str(device))
    m = _DENSE_META.get(key)
    if m is None:
        positions = torch.arange(S, device=device).repeat(B)
        cu = torch.arange(0, (B + 1) * S, S, dtype=torch.int32, device=device)
        tiles = torch.from_numpy(ops.build_tiles([S] * B)).to(device)
        m = (positions, cu, tiles)
        if len(_DENSE_META) > 16:
            _DENSE_META.clear()
        _DENSE_META[key] = m
    return m


def packed_meta(lengths, device):
    """(positions int64 [T], cu_seqlens int32 [B+1], tiles int32) for packed sequences of ``lengths``."""
    lens = np.asarray(lengths, dtype=np.int64)
    cu = np.zeros(len(lens) + 1, dtype=np.int32)
    np.cumsum(lens, out=cu[1:])
    T = int(cu[-1])
    positions = np.arange(T, dtype=np.int64) - np.repeat(cu[:-1].astype(np.int64), lens)
    tiles = ops.build_tiles(lens)
    return (torch.from_numpy(positions).to(device, non_blocking=True),
            torch.from_numpy(cu).to(device, non_blocking=True),
            torch.from_numpy(tiles).to(device, non_blocking=True))


class Qwen3Model(nn.Module):
    """Embedding -> decoder layers -> final norm (qwen3_naive.py:759-807)."""

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([Qwen3DecoderLayer(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, eps=config.rms_norm_eps)

    def forward_packed(self, input_ids, positions, cu_seqlens, tiles):
        h = ops.embedding(input_ids, self.embed_tokens.weight)
        for layer in self.layers:
            h = layer.forward_packed(h, positions, cu_seqlens, tiles)
        return self.norm(h)

    def forward(self, x):
        B, S = x.shape
        positions, cu, tiles = _dense_meta(B, S, x.device)
        return self.forward_packed(x.reshape(-1), positions, cu, tiles).view(B, S, -1)

    def forward_prefill(self, x, positions, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                        block_mapping, block_tables=None, *, tiles=None, decode_tail=None):
        h = ops.embedding(x, self.embed_tokens.weight)
        residual = None
        for layer in self.layers:
            h, residual = layer.forward_prefill(h, positions, cu_seqlens_q, cu_seqlens_k, max_seqlen_q,
                                                max_seqlen_k, block_mapping, block_tables, residual, tiles=tiles,
                                                decode_tail=decode_tail)
        h, _ = self.norm(h, residual)
        return h

    def forward_decode(self, x, positions, context_lens, block_tables, slot_mapping=None, *, decode_plan=None):
        h = ops.embedding(x, self.embed_tokens.weight)
        residual = None
        for layer in self.layers:
            h, residual = layer.forward_decode(h, positions, context_lens, block_tables, slot_mapping, residual,
                                               decode_plan=decode_plan)
        h, _ = self.norm(h, residual)
        return h


# ============================================================================ host->device staging
class _Staging:
    """Packs several small host arrays into one pinned buffer and one H2D copy.

    Returns typed device views.  The pinned buffer is reused on the next call; the
    generator synchronises once per step (the token read-back), which orders the
    previous copy before the buffer is rewritten.
    """

    def __init__(self, device, nbytes=1 << 20):
        self.device = device
        self._alloc(nbytes)

    def _alloc(self, nbytes):
        self.host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        self.dev = torch.empty(nbytes, dtype=torch.uint8, device=self.device)
        self.nbytes = nbytes

    def put(self, arrays):
        sizes = [(a.nbytes + 15) // 16 * 16 for a in arrays]
        total = sum(sizes)
        if total > self.nbytes:
            torch.cuda.current_stream().synchronize()
            self._alloc(max(total, 2 * self.nbytes))
        hb = self.host.numpy()
        off = 0
        spans = []
        for a, sz in zip(arrays, sizes):
            hb[off:off + a.nbytes] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
            spans.append((off, a))
            off += sz
        self.dev[:total].copy_(self.host[:total], non_blocking=True)
        out = []
        for o, a in spans:
            dt = {np.dtype(np.int64): torch.int64, np.dtype(np.int32): torch.int32,
                  np.dtype(np.float32): torch.float32}[a.dtype]
            out.append(self.dev[o:o + a.nbytes].view(dt).view(a.shape))
        return out


def _round_bs(bs, sizes):
    for s in sizes:
        if s >= bs:
            return s
    return None


# ============================================================================ causal LM
class Qwen3ForCausalLM(nn.Module):
    """Qwen3 with a tied lm_head and the paged continuous-batching generator (qwen3_naive.py:810-1679)."""

    packed_modules_mapping = {
        "q_proj": ("qkv_proj", "q"),
        "k_proj": ("qkv_proj", "k"),
        "v_proj": ("qkv_proj", "v"),
        "gate_proj": ("gate_up_proj", "gate"),
        "up_proj": ("gate_up_proj", "up"),
    }

    BLOCK_SIZE = 256
    MAX_TOKENS_PER_STEP = 2048
    GRAPH_BATCH_SIZES = [1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 160, 192, 256, 320, 384, 448, 512]

    def __init__(self, config: Qwen3Config):
        super().__init__()
        self.config = config
        self.model = Qwen3Model(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        if config.tie_word_embeddings:
            # separate Parameter sharing storage, as the reference (qwen3_naive.py:830-831)
            self.lm_head.weight.data = self.model.embed_tokens.weight.data
        self._num_blocks = 0
        self._graphs = {}
        self._has_cuda_graphs = False
        self.use_cuda_graphs = True  # decode steps replay captured graphs (False: eager launches)
        self.pipeline_decode = True  # grouped rollout: submit decode step k+1 before step k's bookkeeping
        self.rollout_stats: dict = {}  # per generate call: steps, decode steps, host time waiting on the GPU
        self.max_model_len = None  # KV positions a sequence may reach; default = prompt + max_new_tokens

    def forward(self, x):
        """Dense logits [batch, seq, vocab] (qwen3_naive.py:833-835)."""
        return ops.linear(self.model(x), self.lm_head.weight)

    def set_rope_grad(self, enabled: bool):
        """False reproduces the reference's RoPE, which blocks q/k gradients (qwen3_naive.py:74-80)."""
        for layer in self.model.layers:
            layer.self_attn.rope_grad = enabled

    # ---------------------------------------------------------------- KV cache
    def _block_bytes(self):
        a = self.model.layers[0].self_attn
        return 2 * len(self.model.layers) * self.BLOCK_SIZE * a.num_kv_heads * a.head_dim * 2

    def _compute_num_blocks(self, gpu_memory_utilization=0.9):
        """Pages that fit after a 2048-token warm-up (qwen3_naive.py:996-1034)."""
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats()
        dummy = torch.randint(0, self.config.vocab_size, (1, 2048), device="cuda")
        with torch.no_grad():
            _ = self.model(dummy)
        del _, dummy
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        free, total = torch.cuda.mem_get_info()
        used = total - free
        stats = torch.cuda.memory_stats()
        peak_act = stats["allocated_bytes.all.peak"] - stats["allocated_bytes.all.current"]
        available = int(total * gpu_memory_utilization - used - peak_act)
        return max(available // self._block_bytes(), 1)

    def allocate_global_kv_cache(self):
        """K and V caches [layers, num_blocks, 256, kv_heads, head_dim] bf16; each layer gets a view."""
        a0 = self.model.layers[0].self_attn
        if not self._num_blocks:
            self._num_blocks = self._compute_num_blocks()
        shape = (self._num_blocks, self.BLOCK_SIZE, a0.num_kv_heads, a0.head_dim)
        if a0.k_cache is not None and tuple(a0.k_cache.shape) == shape:
            return
        dev = self.lm_head.weight.device
        L = len(self.model.layers)
        for layer in self.model.layers:  # drop old views before allocating the new pool
            layer.self_attn.k_cache = layer.self_attn.v_cache = None
        self._graphs.clear()
        self._has_cuda_graphs = False
        k = torch.empty(L, *shape, dtype=torch.bfloat16, device=dev)
        v = torch.empty(L, *shape, dtype=torch.bfloat16, device=dev)
        for i, layer in enumerate(self.model.layers):
            layer.self_attn.k_cache = k[i]
            layer.self_attn.v_cache = v[i]

    # ---------------------------------------------------------------- metadata (reference signatures)
    def _prepare_step(self, seqs: list[Sequence]):
        """Varlen inputs of a mixed prefill/decode step (qwen3_naive.py:1147-1205).

        Returns (input_ids, positions, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
        block_mapping, block_tables) as device tensors (+ Python ints)."""
        arrays, m_q, m_k = self._step_arrays(seqs)
        ids, pos, cu_q, cu_k, blk_map, bt, _tiles = self._staging().put(arrays)
        return ids, pos, cu_q, cu_k, m_q, m_k, blk_map, bt

    def _step_arrays(self, seqs):
        BS = self.BLOCK_SIZE
        n_new = np.fromiter((s.num_scheduled_tokens for s in seqs), dtype=np.int64, count=len(seqs))
        starts = np.fromiter((s.kv_len for s in seqs), dtype=np.int64, count=len(seqs))
        ends = starts + n_new
        ids = np.fromiter((t for s in seqs for t in s.token_ids[s.kv_len:s.kv_len + s.num_scheduled_tokens]),
                          dtype=np.int64, count=int(n_new.sum()))
        seq_of = np.repeat(np.arange(len(seqs)), n_new)
        pos = np.arange(int(n_new.sum()), dtype=np.int64) - np.repeat(np.cumsum(n_new) - n_new, n_new) + \
            np.repeat(starts, n_new)
        cu_q = np.zeros(len(seqs) + 1, dtype=np.int32)
        np.cumsum(n_new, out=cu_q[1:])
        cu_k = np.zeros(len(seqs) + 1, dtype=np.int32)
        np.cumsum(ends, out=cu_k[1:])
        bt = self._block_table_array(seqs)
        blk_map = (bt[seq_of, pos // BS].astype(np.int64) * BS + pos % BS).astype(np.int32)
        tiles = ops.build_tiles(n_new)
        return [ids, pos, cu_q, cu_k, blk_map, bt, tiles], int(n_new.max(initial=0)), int(ends.max(initial=0))

    @staticmethod
    def _block_table_array(seqs, width=None):
        width = width or max(len(s.block_table) for s in seqs)
        bt = np.full((len(seqs), width), -1, dtype=np.int32)
        for i, s in enumerate(seqs):
            bt[i, :len(s.block_table)] = s.block_table
        return bt

    def _build_block_tables(self, seqs: list[Sequence]):
        """[batch, max_blocks] int32 page table padded with -1 (qwen3_naive.py:1207-1212)."""
        return self._staging().put([self._block_table_array(seqs)])[0]

    def _decode_arrays(self, seqs, width=None):
        BS = self.BLOCK_SIZE
        ids = np.fromiter((s.last_token for s in seqs), dtype=np.int64, count=len(seqs))
        pos = np.fromiter((s.num_tokens - 1 for s in seqs), dtype=np.int64, count=len(seqs))
        ctx = np.fromiter((s.kv_len for s in seqs), dtype=np.int32, count=len(seqs))
        slots = np.fromiter((s.block_table[s.kv_len // BS] * BS + s.kv_len % BS for s in seqs), dtype=np.int32,
                            count=len(seqs))
        return ids, pos, ctx, self._block_table_array(seqs, width), slots

    def _prepare_decode(self, seqs: list[Sequence]):
        """(input_ids, positions, context_lens, block_tables, slot_mapping) for a decode step
        (qwen3_naive.py:1214-1225)."""
        ids, pos, ctx, bt, slots = self._decode_arrays(seqs)
        return tuple(self._staging().put([ids, pos, ctx, bt, slots]))

    def _staging(self):
        st = getattr(self, "_stage", None)
        if st is None:
            st = self._stage = _Staging(self.lm_head.weight.device)
        return st

    # ---------------------------------------------------------------- CUDA graphs
    def _init_cuda_graphs(self, max_bs=512, max_ctx=None, max_shared=0):
        """Static decode buffers for batch sizes up to ``max_bs`` (the reference stops at 64).
        ``max_shared``: longest prompt prefix shared by a group (grouped rollout graphs)."""
        dev = self.lm_head.weight.device
        max_ctx = max_ctx or self.config.max_position_embeddings
        self._graph_max_blocks = -(-max_ctx // self.BLOCK_SIZE)
        self._graph_max_ctx = max_ctx
        self._graph_max_shared = max_shared
        self._graph_bs = [b for b in self.GRAPH_BATCH_SIZES if b <= max_bs]
        mb = self._graph_bs[-1]
        W = self._graph_max_blocks
        # packed inputs: i64 ids[mb] pos[mb] rng[2] feed_src[mb] | i32 ctx[mb] slots[mb] bt[mb*W]
        #                members[mb*8] shared_len[mb] kv_start[mb]
        # (feed_src: per row, the row of the previous step whose sample is its input token, or -1;
        # read by the gather that runs before a step submitted ahead of its predecessor's read-back)
        n64 = 3 * mb + 2
        n32 = 2 * mb + mb * W + 8 * mb + 2 * mb
        # two pinned copies, alternated per step: a step is filled while the one before may still
        # wait for its upload
        self._gin_hosts = [torch.zeros(n64 * 8 + n32 * 4, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self._gin_turn = 0
        self._gin_dev = torch.zeros_like(self._gin_hosts[0], device=dev)

        def views(i64, i32):
            o = 2 * mb + mb * W
            return {"input_ids": i64[:mb], "positions": i64[mb:2 * mb], "rng_state": i64[2 * mb:2 * mb + 2],
                    "feed_src": i64[2 * mb + 2:3 * mb + 2],
                    "context_lens": i32[:mb], "slot_mapping": i32[mb:2 * mb],
                    "block_tables": i32[2 * mb:o].reshape(mb, W), "members": i32[o:o + 8 * mb].reshape(mb, 8),
                    "shared_len": i32[o + 8 * mb:o + 9 * mb], "kv_start": i32[o + 9 * mb:o + 10 * mb]}

        self._graph_bufs = views(self._gin_dev[:n64 * 8].view(torch.int64), self._gin_dev[n64 * 8:].view(torch.int32))
        self._graph_bufs["tokens"] = torch.zeros(mb, dtype=torch.int64, device=dev)
        self._graph_bufs["logp"] = torch.zeros(mb, dtype=torch.float32, device=dev)
        self._graph_hosts = [views(h[:n64 * 8].numpy().view(np.int64), h[n64 * 8:].numpy().view(np.int32))
                             for h in self._gin_hosts]
        self._graphs = {}
        self._graph_pool = None
        self._has_cuda_graphs = False

    def _decode_plan(self, bs, grouped=False):
        a = self.model.layers[0].self_attn
        dev = self.lm_head.weight.device
        if grouped:
            b = self._graph_bufs
            plan = ops.grouped_decode_plan(bs, a.num_kv_heads, self._graph_max_shared, self._graph_max_ctx)
            ws = ops.grouped_workspace(bs, a.num_heads, a.head_dim, plan, dev)
            return ("grouped", plan, ws, b["members"][:bs], b["shared_len"][:bs], b["kv_start"][:bs])
        split_tokens, max_splits = ops.decode_split_plan(bs, a.num_kv_heads, self._graph_max_ctx)
        ws = None
        if max_splits > 1:
            nb = ops.lib().qb_paged_decode_workspace_bytes(bs, a.num_heads, a.head_dim, max_splits)
            ws = torch.empty(nb // 4, dtype=torch.float32, device=dev)
        return ("split", split_tokens, max_splits, ws)

    def _decode_body(self, bs, plan, temperature, top_k):
        b = self._graph_bufs
        h = self.model.forward_decode(b["input_ids"][:bs], b["positions"][:bs], b["context_lens"][:bs],
                                      b["block_tables"][:bs], b["slot_mapping"][:bs], decode_plan=plan)
        logits = ops.linear(h, self.lm_head.weight)
        ops.sample(logits, temperature, top_k, 0, b["rng_state"], tokens=b["tokens"][:bs], logp=b["logp"][:bs])

    def _capture_decode_graphs(self, temperature=1.0, top_k=None, grouped=False):
        """Capture decode+lm_head+sampling graphs for every bucket (largest first, one shared pool)."""
        self._graph_key = (float(temperature), top_k, bool(grouped), _pdl_mode())
        self._graphs = {}
        self._graph_pool = None
        self._gin_dev.zero_()
        b = self._graph_bufs
        mb = b["members"].shape[0]
        # warm-up inputs: every row its own group with no keys (its attention reads nothing: pages
        # not yet written may hold any bits), nothing shared, cache writes skipped
        b["context_lens"].fill_(-1)
        b["slot_mapping"].fill_(-1)
        b["members"].fill_(-1)
        b["members"][:, 0] = torch.arange(mb, dtype=torch.int32, device=b["members"].device)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for bs in reversed(self._graph_bs):
                plan = self._decode_plan(bs, grouped)
                self._decode_body(bs, plan, temperature, top_k)  # warm-up outside capture
                g = torch.cuda.CUDAGraph()
                n0 = _lib.LAUNCHES[0]
                with torch.cuda.graph(g, pool=self._graph_pool, stream=s):
                    self._decode_body(bs, plan, temperature, top_k)
                if self._graph_pool is None:
                    self._graph_pool = g.pool()
                self._graphs[bs] = (g, plan, _lib.LAUNCHES[0] - n0)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self._has_cuda_graphs = True

    def _graph_fits(self, bs, width=0):
        """A captured decode graph covers ``bs`` rows with block tables ``width`` pages wide."""
        if not self._has_cuda_graphs or _round_bs(bs, self._graph_bs) is None:
            return False
        return width <= self._graph_max_blocks

    def _run_decode_graph(self, seqs, rng_counter, rng_seed, groups=None, arrays=None, feed=None):
        """Fill the static inputs with one H2D copy, replay, return (tokens, logp) device views.

        ``groups`` (grouped graphs): list of (member row indices, shared key count, first own key).
        ``arrays``: (ids, positions, context_lens, block_tables, slots) already built for ``seqs``.
        ``feed``: (src, prev_tokens) -- row i's input token is prev_tokens[src[i]] (the previous
        step's sample, still on the device) where src[i] >= 0, else ids[i]; gathered on the device
        after the upload, so this step can be enqueued before the previous one is read back."""
        bs = len(seqs)
        gbs = _round_bs(bs, self._graph_bs)
        if gbs is None or (arrays is not None and arrays[3].shape[1] > self._graph_max_blocks):
            return None
        turn = self._gin_turn
        self._gin_turn ^= 1
        hb = self._graph_hosts[turn]
        if arrays is None:
            ids, pos, ctx, bt, slots = self._decode_arrays(seqs, width=self._graph_max_blocks)
        else:
            ids, pos, ctx, bt, slots = arrays
            hb["block_tables"][:bs] = -1
        hb["input_ids"][:bs] = ids
        hb["positions"][:bs] = pos
        hb["context_lens"][:bs] = ctx
        hb["slot_mapping"][:bs] = slots
        hb["block_tables"][:bs, :bt.shape[1]] = bt
        if gbs > bs:  # padding rows: no keys (zero attention output, nothing read), cache writes skipped
            hb["input_ids"][bs:gbs] = 0
            hb["positions"][bs:gbs] = 0
            hb["context_lens"][bs:gbs] = -1
            hb["slot_mapping"][bs:gbs] = -1
            hb["block_tables"][bs:gbs] = 0
        if self._graph_key[2]:
            mem, sl, ks = hb["members"], hb["shared_len"], hb["kv_start"]
            mem[:gbs] = -1
            sl[:gbs] = 0
            ks[:gbs] = 0
            g_i = _fill_groups(groups or [([i], 0, 0) for i in range(bs)], mem, sl, ks)
            for r in range(bs, gbs):  # padding rows are singleton groups
                mem[g_i, 0] = r
                g_i += 1
        hb["rng_state"][0] = rng_counter
        hb["rng_state"][1] = rng_seed
        if feed is not None:
            hb["feed_src"][:bs] = feed[0]
        self._gin_dev.copy_(self._gin_hosts[turn], non_blocking=True)
        if feed is not None:
            b = self._graph_bufs
            ids, src = b["input_ids"][:bs], b["feed_src"][:bs]
            fed = feed[1].index_select(0, src.clamp(min=0))
            ids.copy_(torch.where(src >= 0, fed, ids))
        g, _, n_kernels = self._graphs[gbs]
        g.replay()
        _lib.LAUNCHES[0] += n_kernels
        return self._graph_bufs["tokens"][:bs], self._graph_bufs["logp"][:bs]

    # ---------------------------------------------------------------- non-paged generation modes
    def _sample_rows(self, h, temperature, top_k, rng, step):
        """One token per row of hidden states h: lm_head, then the sampler kernel (the reference's
        logits / T -> top-k -> softmax -> multinomial as one pass); host ints."""
        logits = ops.linear(h, self.lm_head.weight)
        rng[0].fill_(step)
        toks, _ = ops.sample(logits, temperature, top_k, 0, rng)
        return toks.tolist()

    def _new_rng(self):
        seed = int(torch.randint(0, 2**62, (1,)).item())
        return torch.tensor([0, seed], dtype=torch.int64, device=self.lm_head.weight.device)

    def _recompute_step(self, seqs, temperature, top_k, rng, step):
        """Packed forward over the full token lists ``seqs`` (dense varlen causal attention, no KV
        cache) and one sampled token per sequence from its last position."""
        dev = self.lm_head.weight.device
        lens = [len(t) for t in seqs]
        flat = np.fromiter((t for seq in seqs for t in seq), dtype=np.int64, count=sum(lens))
        positions, cu, tiles = packed_meta(lens, dev)
        h = self.model.forward_packed(torch.from_numpy(flat).to(dev), positions, cu, tiles)
        return self._sample_rows(h.index_select(0, (cu[1:] - 1).long()), temperature, top_k, rng, step)

    @torch.no_grad()
    def generate_varlen(self, prompt_ids_list, max_new_tokens=256, temperature=0.6, top_k=20, eos_token_ids=None):
        """Varlen batch generation without a KV cache (qwen3_naive.py:915-990): every step re-runs
        the packed forward over each unfinished sequence's whole token list and samples one token
        from its last position.  A sequence that samples an EOS keeps it and finishes.  Finished
        sequences leave the batch (the reference recomputes them and drops the draws, which changes
        no other sequence's result).  Returns (seq_tokens, generated) as lists of token-id lists."""
        seq_tokens = [p[0].tolist() if isinstance(p, torch.Tensor) else list(p[0]) for p in prompt_ids_list]
        generated = [[] for _ in seq_tokens]
        eos = set(eos_token_ids) if eos_token_ids is not None else None
        active = list(range(len(seq_tokens)))
        rng = self._new_rng()
        for step in range(max_new_tokens):
            if not active:
                break
            toks = self._recompute_step([seq_tokens[i] for i in active], temperature, top_k, rng, step)
            still = []
            for i, t in zip(active, toks):
                seq_tokens[i].append(t)
                generated[i].append(t)
                if eos is None or t not in eos:
                    still.append(i)
            active = still
        ops.check_device_errors()
        return seq_tokens, generated

    @staticmethod
    def _eos_hit(toks, eos_token_ids):
        """The reference tests ``next_token.item() in eos_token_ids``: one row only."""
        if eos_token_ids is None:
            return False
        if len(toks) != 1:
            raise RuntimeError("EOS check reads a single sampled token (next_token.item()): batch size 1 only")
        return toks[0] in eos_token_ids

    @torch.no_grad()
    def generate_naive(self, prompt, max_new_tokens=256, temperature=0.6, top_k=20, eos_token_ids=None):
        """Autoregressive generation by full recomputation (qwen3_naive.py:892-913): prompt [B, L]
        -> [B, L + n]; every step runs the whole sequences; an EOS stops generation before it is
        appended."""
        rows = prompt.tolist()
        rng = self._new_rng()
        for step in range(max_new_tokens):
            toks = self._recompute_step(rows, temperature, top_k, rng, step)
            if self._eos_hit(toks, eos_token_ids):
                break
            for r, t in zip(rows, toks):
                r.append(t)
        ops.check_device_errors()
        return torch.tensor(rows, dtype=torch.long, device=prompt.device)

    @torch.no_grad()
    def generate_kvcache(self, prompt, max_new_tokens=256, temperature=0.6, top_k=20, eos_token_ids=None):
        """Prefill once, then one decode step per token (qwen3_naive.py:842-889): prompt [B, L] ->
        [B, L + n].  The reference's per-layer contiguous cache becomes a run of pages of the paged
        pool for each row (prefill and decode on the paged kernels).  As in the reference, the first
        sampled token is always appended and a later EOS stops generation before it is appended."""
        dev = self.lm_head.weight.device
        B, L = prompt.shape
        pages = -(-(L + max_new_tokens) // self.BLOCK_SIZE)
        self.allocate_global_kv_cache()
        if self._num_blocks < B * pages:
            raise ValueError(f"KV pool holds {self._num_blocks} pages; generate_kvcache needs {B * pages}")
        bt = torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages)
        pos = torch.arange(L, dtype=torch.int64, device=dev)
        slots = (bt[:, pos // self.BLOCK_SIZE].long() * self.BLOCK_SIZE + pos % self.BLOCK_SIZE).reshape(-1).int()
        cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device=dev)
        h = self.model.forward_prefill(prompt.to(dev).reshape(-1), pos.repeat(B), cu, cu, L, L, slots, bt)
        rng = self._new_rng()
        toks = self._sample_rows(h.index_select(0, (cu[1:] - 1).long()), temperature, top_k, rng, 0)
        rows = prompt.tolist()
        for r, t in zip(rows, toks):
            r.append(t)
        for step in range(max_new_tokens - 1):
            p = L + step
            ids = torch.tensor(toks, dtype=torch.long, device=dev)
            positions = torch.full((B,), p, dtype=torch.int64, device=dev)
            ctx = torch.full((B,), p, dtype=torch.int32, device=dev)  # keys already cached
            slot = (bt[:, p // self.BLOCK_SIZE] * self.BLOCK_SIZE + p % self.BLOCK_SIZE).int()
            h = self.model.forward_decode(ids, positions, ctx, bt, slot)
            toks = self._sample_rows(h, temperature, top_k, rng, step + 1)
            if self._eos_hit(toks, eos_token_ids):
                break
            for r, t in zip(rows, toks):
                r.append(t)
        ops.check_device_errors()
        return torch.tensor(rows, dtype=torch.long, device=prompt.device)

    # ---------------------------------------------------------------- generation
    @torch.no_grad()
    def generate_continuous(self, prompt_ids_list, max_new_tokens=256, temperature=0.6, top_k=20,
                            eos_token_ids=None):
        """Continuous batching + chunked prefill (qwen3_naive.py:1228-1471).

        Returns (seq_tokens, generated) as lists of token-id lists."""
        seqs = self._generate(prompt_ids_list, max_new_tokens, temperature, top_k, eos_token_ids, False)
        return [s.token_ids for s in seqs], [s.token_ids[s.num_prompt_tokens:] for s in seqs]

    @torch.no_grad()
    def generate_continuous_with_logprobs(self, prompt_ids_list, max_new_tokens=256, temperature=0.6, top_k=20,
                                          eos_token_ids=None):
        """As generate_continuous, also recording each sampled token's log-prob under the
        temperature-scaled, top-k-filtered distribution (qwen3_naive.py:1474-1679).

        Returns (seq_tokens, generated, log_probs, prompt_lens)."""
        seqs = self._generate(prompt_ids_list, max_new_tokens, temperature, top_k, eos_token_ids, True)
        return ([s.token_ids for s in seqs], [s.token_ids[s.num_prompt_tokens:] for s in seqs],
                [s.response_log_probs for s in seqs], [s.num_prompt_tokens for s in seqs])

    def _grouped_setup(self, max_ctx, max_shared, temperature, top_k):
        """KV pool and grouped decode graphs for a grouped rollout; returns the step context."""
        dev = self.lm_head.weight.device
        self.allocate_global_kv_cache()
        seed = int(torch.randint(0, 2**62, (1,)).item())
        key = (float(temperature), top_k, True, _pdl_mode())
        if not self.use_cuda_graphs:
            self._has_cuda_graphs = False
        elif (not self._has_cuda_graphs or self._graph_max_ctx < max_ctx or getattr(self, "_graph_key", None) != key
                or getattr(self, "_graph_max_shared", -1) < max_shared):
            # the shared-prefix bound is the whole context, so later prompts never force a recapture
            ctx_cap = max(max_ctx, 1024)
            self._init_cuda_graphs(max_bs=512, max_ctx=ctx_cap, max_shared=ctx_cap)
            self._capture_decode_graphs(temperature, top_k, grouped=True)
        cap = 2 * self.MAX_TOKENS_PER_STEP + 512 * 8
        ctx = {"dev": dev, "seed": seed, "temperature": temperature, "top_k": top_k,
               "rng": torch.tensor([0, seed], dtype=torch.int64, device=dev),
               "rb": [(torch.empty(cap, dtype=torch.int64, pin_memory=True),
                       torch.empty(cap, dtype=torch.float32, pin_memory=True),
                       torch.zeros(1, dtype=torch.int32, pin_memory=True)) for _ in range(2)],
               "rb_turn": 0, "err": ops.err_flag(dev)}
        ctx["tok_host"], ctx["lp_host"], ctx["err_host"] = ctx["rb"][0]  # the synchronous steps' slot
        return ctx

    def _grouped_launch(self, ctx, prefill, done, decode_rows, groups_rows, step, G, n_samples):
        """Enqueues one grouped-rollout step: a grouped-decode graph when only decode
        rows run, else one forward over the donors' prompt chunks (paged varlen attention) and
        the decode rows (shared-prefix decode attention); then lm_head + sampling (G draws from each finished
        prefill's last row) and the read-back."""
        dev, temperature, top_k = ctx["dev"], ctx["temperature"], ctx["top_k"]
        r = None
        a = self.model.layers[0].self_attn
        nd = len(decode_rows)
        if not prefill:
            if self._has_cuda_graphs:
                r = self._run_decode_graph(decode_rows, step, ctx["seed"], groups=groups_rows)
            if r is None:  # eager decode with the same shared-prefix attention
                r = self._grouped_decode_eager(ctx, self._decode_arrays(decode_rows), groups_rows, step)
        else:
            # prefill rows (the donors' prompt chunks) on the paged varlen kernel; decode rows,
            # whose keys skip the unused tail of the shared prompt page, on the grouped decode
            donors = [g.donor for g in prefill]
            (ids, pos, cu_q, cu_k, blk_map, bt, tiles), m_q, m_k = self._step_arrays(donors)
            tp = len(ids)
            ends = np.cumsum([d.num_scheduled_tokens for d in donors]) - 1
            rows_np = np.asarray([ends[prefill.index(g)] for g in done for _ in range(G)]
                                 + [tp + j for j in range(nd)], dtype=np.int64)
            if nd:
                ids_d, pos_d, cl, bt_d, slots = self._decode_arrays(decode_rows)
                mem, sl, ks = _group_arrays(groups_rows, nd)
                plan = ops.grouped_decode_plan(nd, a.num_kv_heads, int(sl.max(initial=0)),
                                               int((cl + 1 - ks).max(initial=1)))
                (ids, pos, blk_map, cu_q, cu_k, bt, tiles, rows, cl_d, bt_d, mem_d, sl_d, ks_d) = self._staging().put(
                    [np.concatenate([ids, ids_d]), np.concatenate([pos, pos_d]), np.concatenate([blk_map, slots]),
                     cu_q, cu_k, bt, tiles, rows_np, cl, bt_d, mem, sl, ks])
                ws = ops.grouped_workspace(nd, a.num_heads, a.head_dim, plan, dev)
                tail = (tp, cl_d, bt_d, ("grouped", plan, ws, mem_d, sl_d, ks_d))
            else:
                ids, pos, cu_q, cu_k, blk_map, bt, tiles, rows = self._staging().put(
                    [ids, pos, cu_q, cu_k, blk_map, bt, tiles, rows_np])
                tail = None
            h = self.model.forward_prefill(ids, pos, cu_q, cu_k, m_q, m_k, blk_map, bt, tiles=tiles,
                                           decode_tail=tail)
            logits = ops.linear(h.index_select(0, rows), self.lm_head.weight)
            ctx["rng"][0].fill_(step)
            r = ops.sample(logits, temperature, top_k, 0, ctx["rng"])
        toks_dev, logp_dev = r
        ctx["tok_host"][:n_samples].copy_(toks_dev, non_blocking=True)
        ctx["lp_host"][:n_samples].copy_(logp_dev, non_blocking=True)
        ctx["err_host"].copy_(ctx["err"], non_blocking=True)

    def _grouped_decode_eager(self, ctx, arrays, groups_rows, step):
        """One grouped decode step without graphs (shared-prefix attention); returns (tokens, logp) on the device."""
        dev = ctx["dev"]
        a = self.model.layers[0].self_attn
        ids, pos, cl, bt, slots = arrays
        nd = len(ids)
        mem, sl, ks = _group_arrays(groups_rows, nd)
        plan = ops.grouped_decode_plan(nd, a.num_kv_heads, int(sl.max(initial=0)), int((cl + 1 - ks).max(initial=1)))
        ids, pos, cl, bt, slots, mem_d, sl_d, ks_d = self._staging().put([ids, pos, cl, bt, slots, mem, sl, ks])
        ws = ops.grouped_workspace(nd, a.num_heads, a.head_dim, plan, dev)
        h = self.model.forward_decode(ids, pos, cl, bt, slots, decode_plan=("grouped", plan, ws, mem_d, sl_d, ks_d))
        logits = ops.linear(h, self.lm_head.weight)
        ctx["rng"][0].fill_(step)
        return ops.sample(logits, ctx["temperature"], ctx["top_k"], 0, ctx["rng"])

    # -- pipelined decode steps of the grouped rollout: the host submits step k+1 right after step k's
    #    read-back and does step k's bookkeeping while step k+1 runs (_generate_grouped)
    def _decode_step_arrays(self, rows):
        """(positions, context_lens, block_tables, slots) of a decode step over ``rows``; a row's
        position counts its tokens still in flight (``inflight`` submitted steps not yet read back)."""
        BS = self.BLOCK_SIZE
        n = len(rows)
        pos = np.fromiter((len(s.token_ids) + s.inflight - 1 for s in rows), dtype=np.int64, count=n)
        cl = np.fromiter((s.kv_len for s in rows), dtype=np.int32, count=n)
        slots = np.fromiter((s.block_table[s.kv_len // BS] * BS + s.kv_len % BS for s in rows), dtype=np.int32,
                            count=n)
        return pos, cl, self._block_table_array(rows), slots

    def _decode_submit(self, ctx, rows, groups_rows, step, ids, arrays, feed=None):
        """Enqueue one decode step over ``rows`` (input token ``ids``, metadata ``arrays`` from
        _decode_step_arrays) and the read-back of its samples; returns a handle for _decode_collect.

        ``feed`` = (src, handle of the step before, not yet read back): the inputs of rows with
        src >= 0 are that step's samples, gathered on the device (graph replays only: the caller
        checks _graph_fits).  Read-backs alternate between two pinned slots, so a step can be
        collected while the next one is already queued."""
        pos, cl, bt, slots = arrays
        full = (ids, pos, cl, bt, slots)
        r = None
        if self._has_cuda_graphs:
            fd = None if feed is None else (feed[0], feed[1]["tokens"])
            r = self._run_decode_graph(rows, step, ctx["seed"], groups=groups_rows, arrays=full, feed=fd)
        if r is None:
            if feed is not None:
                raise RuntimeError("a device-fed decode step needs a captured graph")
            r = self._grouped_decode_eager(ctx, full, groups_rows, step)
        n = len(rows)
        toks_dev, logp_dev = r
        slot = ctx["rb_turn"]
        ctx["rb_turn"] ^= 1
        tok_h, lp_h, err_h = ctx["rb"][slot]
        tok_h[:n].copy_(toks_dev, non_blocking=True)
        lp_h[:n].copy_(logp_dev, non_blocking=True)
        err_h.copy_(ctx["err"], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        return {"n": n, "event": ev, "slot": slot, "tokens": toks_dev}

    def _decode_collect(self, ctx, handle):
        """Waits for a submitted step; returns its (tokens, log-probs) as numpy arrays."""
        t0 = time.perf_counter()
        handle["event"].synchronize()
        st = self.rollout_stats
        st["gpu_wait_s"] = st.get("gpu_wait_s", 0.0) + time.perf_counter() - t0
        st["steps"] = st.get("steps", 0) + 1
        tok_h, lp_h, err_h = ctx["rb"][handle["slot"]]
        if int(err_h[0]):
            ops.check_device_errors(ctx["dev"])
        n = handle["n"]
        return tok_h[:n].numpy().copy(), lp_h[:n].numpy().copy()

    @torch.no_grad()
    def generate_grouped_with_logprobs(self, prompt_ids_list, group_size, max_new_tokens=256, temperature=0.6,
                                       top_k=20, eos_token_ids=None):
        """GRPO rollout: ``group_size`` (<= 8) completions of every prompt, the prompt prefilled once
        per group and its K/V pages shared (the grouped decode attention reads them once per step).

        Returns the 4-tuple of :meth:`generate_continuous_with_logprobs` for the list in which each
        prompt is repeated ``group_size`` times consecutively.  Sampling and log-probs follow the same
        distribution; page ids and step boundaries differ from the reference's scheduler, which
        prefills every completion separately (use generate_continuous_with_logprobs for that)."""
        if not 1 <= group_size <= 8:
            raise ValueError("group_size must be in [1, 8]")
        prompts = [p[0].tolist() if isinstance(p, torch.Tensor) else list(p[0]) for p in prompt_ids_list]
        seqs = _generate_grouped(self, prompts, group_size, max_new_tokens, temperature, top_k, eos_token_ids)
        return ([s.token_ids for s in seqs], [s.token_ids[s.num_prompt_tokens:] for s in seqs],
                [s.response_log_probs for s in seqs], [s.num_prompt_tokens for s in seqs])

    # -- device side of one generation step (kept behind two methods so the host
    #    scheduler can be exercised on its own)
    def _gen_setup(self, prompts, max_new_tokens, temperature, top_k):
        """Allocates the KV pool, (re)captures decode graphs, returns the per-call device context."""
        dev = self.lm_head.weight.device
        self.allocate_global_kv_cache()
        max_ctx = self.max_model_len or (max((len(p) for p in prompts), default=1) + max_new_tokens)
        seed = int(torch.randint(0, 2**62, (1,)).item())
        if not self.use_cuda_graphs:
            self._has_cuda_graphs = False
        elif (not self._has_cuda_graphs or self._graph_max_ctx < max_ctx
                or getattr(self, "_graph_key", None) != (float(temperature), top_k, False, _pdl_mode())):
            if not self._has_cuda_graphs or self._graph_max_ctx < max_ctx:
                self._init_cuda_graphs(max_bs=512, max_ctx=max(max_ctx, 1024))
            self._capture_decode_graphs(temperature, top_k)
        cap = self.MAX_TOKENS_PER_STEP + 512
        return {"dev": dev, "seed": seed, "temperature": temperature, "top_k": top_k,
                "rng": torch.tensor([0, seed], dtype=torch.int64, device=dev),  # {counter, seed}
                "tok_host": torch.empty(cap, dtype=torch.int64, pin_memory=True),
                "lp_host": torch.empty(cap, dtype=torch.float32, pin_memory=True),
                "err_host": torch.zeros(1, dtype=torch.int32, pin_memory=True),
                "err": ops.err_flag(dev)}

    def _launch_step(self, ctx, scheduled, n_sampled, all_decode, step):
        """Enqueues forward + lm_head + sampling for ``scheduled`` and the async read-back."""
        toks_dev = logp_dev = None
        if all_decode and self._has_cuda_graphs:
            r = self._run_decode_graph(scheduled, step, ctx["seed"])
            if r is not None:
                toks_dev, logp_dev = r
        if toks_dev is None:
            if all_decode:
                ids, pos, cl, bt, slots = self._prepare_decode(scheduled)
                h = self.model.forward_decode(ids, pos, cl, bt, slots)
                rows = None
            else:
                arrays, m_q, m_k = self._step_arrays(scheduled)
                offsets = np.cumsum([s.num_scheduled_tokens for s in scheduled]) - 1
                rows_np = np.asarray([offsets[j] for j, s in enumerate(scheduled)
                                      if s.num_scheduled_tokens == 1
                                      or s.kv_len + s.num_scheduled_tokens >= s.num_prompt_tokens], dtype=np.int64)
                ids, pos, cu_q, cu_k, blk_map, bt, tiles, rows = self._staging().put(arrays + [rows_np])
                h = self.model.forward_prefill(ids, pos, cu_q, cu_k, m_q, m_k, blk_map, bt, tiles=tiles)
            if n_sampled:
                hs = h if rows is None else h.index_select(0, rows)
                logits = ops.linear(hs, self.lm_head.weight)
                ctx["rng"][0].fill_(step)
                toks_dev, logp_dev = ops.sample(logits, ctx["temperature"], ctx["top_k"], 0, ctx["rng"])
        if n_sampled:  # one read-back per step: tokens, log-probs and the device error word
            ctx["tok_host"][:n_sampled].copy_(toks_dev, non_blocking=True)
            ctx["lp_host"][:n_sampled].copy_(logp_dev, non_blocking=True)
        ctx["err_host"].copy_(ctx["err"], non_blocking=True)
        return None

    def _finish_step(self, ctx, pending, n, record_logprobs):
        """Waits for the step, surfaces device-side bounds errors, returns host lists."""
        t0 = time.perf_counter()
        torch.cuda.current_stream().synchronize()
        st = self.rollout_stats
        st["gpu_wait_s"] = st.get("gpu_wait_s", 0.0) + time.perf_counter() - t0
        st["steps"] = st.get("steps", 0) + 1
        if int(ctx["err_host"][0]):
            ops.check_device_errors(ctx["dev"])
        if not n:
            return [], []
        toks = ctx["tok_host"][:n].tolist()
        lps = ctx["lp_host"][:n].tolist() if record_logprobs else None
        return toks, lps

    def _generate(self, prompt_ids_list, max_new_tokens, temperature, top_k, eos_token_ids, record_logprobs):
        BS = self.BLOCK_SIZE
        budget_max = self.MAX_TOKENS_PER_STEP
        prompts = [p[0].tolist() if isinstance(p, torch.Tensor) else list(p[0]) for p in prompt_ids_list]
        self.rollout_stats = {"t_start": time.perf_counter()}
        ctx = self._gen_setup(prompts, max_new_tokens, temperature, top_k)
        bm = BlockManager(self._num_blocks, BS)
        eos = set(eos_token_ids) if eos_token_ids is not None else None
        sp = {"temperature": temperature, "max_tokens": max_new_tokens}
        waiting: deque[Sequence] = deque(Sequence(t, sp) for t in prompts)
        running: list[Sequence] = []
        all_seqs = list(waiting)
        step = 0

        def finish(seq):
            seq.status = "FINISHED"
            bm.deallocate(seq.block_table)
            seq.block_table.clear()
            running.remove(seq)

        while waiting or running:
            scheduled = []
            budget = budget_max
            # ---- Step 1: running sequences, decode first (qwen3_naive.py:1513-1552)
            i = 0
            while i < len(running) and budget > 0:
                seq = running[i]
                if seq.kv_len >= seq.num_prompt_tokens:
                    if seq.num_completion_tokens >= seq.max_tokens:
                        seq.status = "FINISHED"
                        bm.deallocate(seq.block_table)
                        seq.block_table.clear()
                        running.pop(i)
                        continue
                    if seq.kv_len % BS == 0:
                        if not bm.free:
                            while not bm.can_append(seq):  # LIFO preemption
                                victim = running[-1]
                                victim.status = "WAITING"
                                bm.deallocate(victim.block_table)
                                victim.block_table.clear()
                                victim.kv_len = 0
                                victim.token_ids = victim.token_ids[:victim.num_prompt_tokens]
                                victim.response_log_probs.clear()
                                running.pop()
                                waiting.appendleft(victim)
                                if victim is seq:
                                    break
                            if seq.status == "WAITING":
                                continue
                        bm.may_append(seq)
                    seq.num_scheduled_tokens = 1
                else:
                    seq.num_scheduled_tokens = min(seq.num_prompt_tokens - seq.kv_len, budget)
                scheduled.append(seq)
                budget -= seq.num_scheduled_tokens
                i += 1
            # ---- Step 2: admit waiting sequences with the remaining budget (:1557-1580)
            while waiting and budget > 0:
                seq = waiting[0]
                if not seq.block_table:
                    if bm.available < seq.num_blocks:
                        break
                    bm.allocate(seq)
                waiting.popleft()
                seq.status = "RUNNING"
                running.append(seq)
                remaining = seq.num_prompt_tokens - seq.kv_len
                if remaining <= budget:
                    seq.num_scheduled_tokens = remaining
                elif not scheduled:
                    seq.num_scheduled_tokens = budget
                else:
                    waiting.appendleft(seq)
                    running.pop()
                    break
                scheduled.append(seq)
                budget -= seq.num_scheduled_tokens
            if not scheduled:
                continue

            # ---- Step 3: forward + lm_head + sampling, launched on the device
            all_decode = all(s.num_scheduled_tokens == 1 for s in scheduled)
            sampled = [s for s in scheduled
                       if s.num_scheduled_tokens == 1 or s.kv_len + s.num_scheduled_tokens >= s.num_prompt_tokens]
            step += 1
            pending = self._launch_step(ctx, scheduled, len(sampled), all_decode, step)

            # ---- Step 4: KV bookkeeping and prefix-cache registration (overlaps the GPU)
            if all_decode:
                for seq in scheduled:
                    seq.kv_len += 1
            else:
                for seq in scheduled:
                    seq.kv_len += seq.num_scheduled_tokens
                    bm.hash_blocks(seq)

            n = len(sampled)
            toks, lps = self._finish_step(ctx, pending, n, record_logprobs)
            if not n:
                for seq in scheduled:
                    seq.num_scheduled_tokens = 0
                continue
            # ---- Step 5: append sampled tokens, finish on EOS / max_tokens (:1653-1673)
            for j, seq in enumerate(sampled):
                tok = toks[j]
                seq.append_token(tok)
                if record_logprobs:
                    seq.response_log_probs.append(lps[j])
                if eos is not None and tok in eos:
                    finish(seq)
                elif seq.num_completion_tokens >= seq.max_tokens:
                    finish(seq)
            for seq in scheduled:
                seq.num_scheduled_tokens = 0
        self.rollout_stats["total_s"] = time.perf_counter() - self.rollout_stats.pop("t_start")
        return all_seqs


class _Group:
    """G completions of one prompt: one prefill (``donor``) into pages that all members share.

    Every prompt page, the partially filled last one included, is shared; a member's own
    tokens start on a fresh page at key position ``own_start`` of its page table (positions
    for RoPE stay the true token positions).  The unused tail of the last prompt page is
    never read: decode attention takes keys [0, L) from the shared pages and
    [own_start, kv_len] from the member's own."""

    def __init__(self, idx, prompt, G, sp):
        self.idx = idx
        self.prompt = list(prompt)
        self.L = len(prompt)
        self.G = G
        self.sp = sp
        self.members = [Sequence(prompt, sp) for _ in range(G)]
        self.reset()

    def reset(self):
        self.state = "WAITING"
        self.donor = Sequence(self.prompt, self.sp)
        self.shared = []
        for m in self.members:
            m.token_ids = list(self.prompt)
            m.last_token = self.prompt[-1]
            m.kv_len = 0
            m.block_table = []
            m.response_log_probs = []
            m.status = "WAITING"
            m.num_scheduled_tokens = 0
            m.inflight = 0  # decode steps submitted for this member and not yet read back

    @property
    def n_shared(self):
        return -(-self.L // Sequence.BLOCK_SIZE)

    @property
    def own_start(self):
        return self.n_shared * Sequence.BLOCK_SIZE

    def pages_needed(self):
        return self.n_shared


def _group_arrays(groups_rows, n_rows):
    """(members [n_groups, 8], shared_len [n_groups], kv_start [n_rows]) int32 for the grouped decode attention."""
    mem = np.full((len(groups_rows), 8), -1, dtype=np.int32)
    sl = np.zeros(len(groups_rows), dtype=np.int32)
    ks = np.zeros(n_rows, dtype=np.int32)
    _fill_groups(groups_rows, mem, sl, ks)
    return mem, sl, ks


def _fill_groups(groups_rows, mem, sl, ks):
    g_i = 0
    for rows, shared, start in groups_rows:
        mem[g_i, :len(rows)] = rows
        sl[g_i] = shared
        ks[rows] = start
        g_i += 1
    return g_i


def _generate_grouped(model, prompts, G, max_new_tokens, temperature, top_k, eos_token_ids, record_logprobs=True):
    """Continuous-batching rollout of G completions per prompt with the prompt computed once.

    Scheduling follows the reference's loop (decode first, 2048-token budget, chunked prefill,
    LIFO preemption) at the granularity of a group.  A group's prompt pages are shared by its
    members (reference-counted once per member); each member owns the pages of what it
    generates, starting on a fresh page (see _Group).  The first token of every member is
    sampled from the single prefill's last row (G independent draws)."""
    BS = model.BLOCK_SIZE
    sp = {"temperature": temperature, "max_tokens": max_new_tokens}
    groups = [_Group(i, p, G, sp) for i, p in enumerate(prompts)]
    # key positions run up to own_start + max_new_tokens (own tokens start page-aligned)
    max_ctx = (model.max_model_len or (max((len(p) for p in prompts), default=1) + max_new_tokens)) + BS
    max_shared = max((g.L for g in groups), default=0)
    model.rollout_stats = {"t_start": time.perf_counter()}
    ctx = model._grouped_setup(max_ctx, max_shared, temperature, top_k)
    model.rollout_stats["setup_s"] = time.perf_counter() - model.rollout_stats["t_start"]
    bm = BlockManager(model._num_blocks, BS)
    eos = set(eos_token_ids) if eos_token_ids is not None else None
    waiting = deque(groups)
    running: list[_Group] = []
    step = 0

    def release(grp):
        for m in grp.members:
            if m.block_table:
                bm.deallocate(m.block_table)
                m.block_table = []

    def preempt(grp):
        release(grp)
        grp.reset()
        running.remove(grp)
        waiting.appendleft(grp)

    def accept(m, tok, lp):
        m.append_token(tok)
        if record_logprobs:
            m.response_log_probs.append(lp)
        if (eos is not None and tok in eos) or m.num_completion_tokens >= m.max_tokens:
            m.status = "FINISHED"
            bm.deallocate(m.block_table)
            m.block_table = []

    def groups_of(rows):
        pos_of = {id(m): i for i, m in enumerate(rows)}
        out = []  # (decode row indices, shared prompt keys, first own key) per group
        for grp in running:
            idx = [pos_of[id(m)] for m in grp.members if id(m) in pos_of]
            if idx:
                out.append((idx, grp.L, grp.own_start))
        return out

    # ---- pipelined decode: with no group waiting and every running group decoding, the rows of
    # step k+1 are known before step k's tokens are (a member leaves only by EOS, found after
    # the fact, or by its token budget, known ahead).  Step k+1 is planned while step k runs and
    # queued behind it before step k is read back: its input tokens are step k's samples,
    # gathered on the device from the decode graph's output, so the GPU goes from step k to
    # step k+1 without waiting for the host.  Step k's read-back and bookkeeping, and step
    # k+2's planning, then overlap step k+1.  (Without a captured graph for step k+1 it is
    # submitted after step k's read-back with the tokens from the host.)  A member that sampled
    # EOS at step k has already been submitted for step k+1: that sample is discarded.  The
    # rows' random draws are independent, so the others are unaffected; pages it still writes at
    # step k+1 are freed on the host first but reused only by steps that run after it on the
    # stream.
    def plan_step(prev_rows=None):
        """Rows, groups, metadata and, per row, its index in ``prev_rows`` (the step in flight,
        whose samples are this step's inputs) of the next decode step; None when no row is left
        or a page is missing (the synchronous loop then preempts)."""
        rows = [m for g in running for m in g.members
                if m.status == "RUNNING" and m.num_completion_tokens + m.inflight < m.max_tokens]
        if not rows or len(rows) > model.MAX_TOKENS_PER_STEP:
            return None
        for m in rows:
            if len(m.block_table) * BS <= m.kv_len:
                if not bm.free:
                    return None
                m.block_table.append(bm._take_free())
        src = None
        if prev_rows is not None:
            pos_of = {id(m): i for i, m in enumerate(prev_rows)}
            src = np.fromiter((pos_of.get(id(m), -1) for m in rows), dtype=np.int64, count=len(rows))
        return rows, groups_of(rows), model._decode_step_arrays(rows), src

    def submit(plan, ids, feed=None):
        nonlocal step
        rows, grows, arrays, _ = plan
        step += 1
        model.rollout_stats["decode_steps"] = model.rollout_stats.get("decode_steps", 0) + 1
        h = model._decode_submit(ctx, rows, grows, step, ids, arrays, feed=feed)
        for m in rows:
            m.kv_len += 1
            m.inflight += 1
        return h

    def run_pipelined():
        plan = plan_step()
        if plan is None:
            return False
        rows = plan[0]
        h = submit(plan, np.fromiter((m.last_token for m in rows), dtype=np.int64, count=len(rows)))
        while True:
            nplan = plan_step(rows)  # overlaps the step in flight
            h_nxt = None
            if nplan is not None and model._graph_fits(len(nplan[0]), nplan[2][2].shape[1]):
                # step k+1 is queued behind step k before k is read back: its input tokens are
                # step k's samples, gathered on the device (a row new to k+1 brings its own)
                src = nplan[3]
                own = np.fromiter((0 if j >= 0 else m.last_token for j, m in zip(src, nplan[0])), dtype=np.int64,
                                  count=len(src))
                h_nxt = submit(nplan, own, feed=(src, h))
            toks, lps = model._decode_collect(ctx, h)
            if nplan is not None and h_nxt is None:
                src = nplan[3]
                if (src >= 0).all():
                    ids = toks[src]
                else:
                    ids = np.array([toks[j] if j >= 0 else m.last_token for j, m in zip(src, nplan[0])], dtype=np.int64)
                h_nxt = submit(nplan, ids)
            for j, m in enumerate(rows):  # overlaps the step just submitted
                m.inflight -= 1
                if m.status == "RUNNING":
                    accept(m, int(toks[j]), float(lps[j]))
            for g in list(running):
                if all(m.status == "FINISHED" for m in g.members):
                    g.state = "FINISHED"
                    running.remove(g)
            if h_nxt is None:
                return True
            rows, h = nplan[0], h_nxt

    while waiting or running:
        if (getattr(model, "pipeline_decode", True) and not waiting and running
                and all(g.state == "DECODE" for g in running) and run_pipelined()):
            continue
        budget = model.MAX_TOKENS_PER_STEP
        decode_rows: list[Sequence] = []
        prefill: list[_Group] = []
        # ---- running groups: decoding members first, then a group still in prefill
        gi = 0
        while gi < len(running) and budget > 0:
            grp = running[gi]
            if grp.state == "DECODE":
                preempted = False
                for m in grp.members:
                    if m.status != "RUNNING" or budget <= 0:
                        continue
                    if m.num_completion_tokens >= m.max_tokens:
                        m.status = "FINISHED"
                        bm.deallocate(m.block_table)
                        m.block_table = []
                        continue
                    if len(m.block_table) * BS <= m.kv_len:  # the next key needs a new page
                        while not bm.free:
                            victim = running[-1]
                            preempt(victim)
                            if victim is grp:
                                preempted = True
                                break
                        if preempted:
                            break
                        m.block_table.append(bm._take_free())
                    m.num_scheduled_tokens = 1
                    decode_rows.append(m)
                    budget -= 1
                if preempted:
                    decode_rows = [r for r in decode_rows if r not in grp.members]
                    continue
                if all(m.status == "FINISHED" for m in grp.members):
                    grp.state = "FINISHED"
                    running.pop(gi)
                    continue
            elif grp.state == "PREFILL":
                d = grp.donor
                d.num_scheduled_tokens = min(grp.L - d.kv_len, budget)
                budget -= d.num_scheduled_tokens
                prefill.append(grp)
            gi += 1
        # ---- admit waiting groups
        while waiting and budget > 0:
            grp = waiting[0]
            if grp.state == "WAITING":
                if bm.available < grp.pages_needed():
                    break
                grp.shared = [bm._take_free() for _ in range(grp.n_shared)]
                for p in grp.shared:
                    bm.ref_count[p] = G  # one reference per member
                for m in grp.members:
                    m.block_table = list(grp.shared)
                grp.donor.block_table = grp.shared
                grp.state = "PREFILL"
            waiting.popleft()
            running.append(grp)
            d = grp.donor
            remaining = grp.L - d.kv_len
            if remaining <= budget:
                d.num_scheduled_tokens = remaining
            elif not decode_rows and not prefill:
                d.num_scheduled_tokens = budget
            else:
                waiting.appendleft(grp)
                running.pop()
                break
            budget -= d.num_scheduled_tokens
            prefill.append(grp)
        if not decode_rows and not prefill:
            continue

        # ---- device step (Step 4 bookkeeping below overlaps it)
        step += 1
        done = [g for g in prefill if g.donor.kv_len + g.donor.num_scheduled_tokens >= g.L]
        n_samples = len(decode_rows) + G * len(done)
        groups_rows = groups_of(decode_rows)
        if not prefill:
            model.rollout_stats["decode_steps"] = model.rollout_stats.get("decode_steps", 0) + 1
        model._grouped_launch(ctx, prefill, done, decode_rows, groups_rows, step, G, n_samples)
        for g in prefill:
            g.donor.kv_len += g.donor.num_scheduled_tokens
            g.donor.num_scheduled_tokens = 0
        for m in decode_rows:
            m.kv_len += 1
            m.num_scheduled_tokens = 0
        toks, lps = model._finish_step(ctx, None, n_samples, True)
        k = 0
        for g in done:
            g.state = "DECODE"
            for m in g.members:
                m.kv_len = g.own_start  # next key goes to a fresh page
                m.status = "RUNNING"
                accept(m, toks[k], lps[k])
                k += 1
        for m in decode_rows:
            accept(m, toks[k], lps[k])
            k += 1
        for g in list(running):
            if g.state == "DECODE" and all(m.status == "FINISHED" for m in g.members):
                g.state = "FINISHED"
                running.remove(g)
    if bm.available != bm.num_blocks or any(bm.ref_count):
        raise RuntimeError("grouped rollout finished with KV pages still referenced")
    st = model.rollout_stats
    st["total_s"] = time.perf_counter() - st.pop("t_start")
    return [m for g in groups for m in g.members]


def use_reference_defaults():
    """The reference module sets these process-wide at import (qwen3_naive.py:1786-1787) so that
    ``Qwen3ForCausalLM(config)`` is built in bf16 on the GPU; here it is an explicit call."""
    torch.set_default_dtype(torch.bfloat16)
    torch.set_default_device("cuda")


def build_model(config: Qwen3Config, device="cuda", dtype=torch.bfloat16, seed: int | None = 0,
                std: float = 0.02) -> Qwen3ForCausalLM:
    """Constructs the model directly in ``dtype`` on ``device`` (so the lm_head/embedding tie
    survives) and, with a seed, draws every Linear and the embedding from N(0, std) with RMSNorm
    weights 1 -- the random-init Qwen3-0.6B shape the benchmarks use."""
    prev = torch.get_default_dtype()
    torch.set_default_dtype(dtype)
    try:
        with torch.device(device):
            model = Qwen3ForCausalLM(config)
    finally:
        torch.set_default_dtype(prev)
    if seed is not None:
        g = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name == "lm_head.weight" and config.tie_word_embeddings:
                    continue
                if name.endswith("norm.weight"):
                    p.fill_(1.0)
                else:
                    p.normal_(0.0, std, generator=g)
    return model


def load_weights(model, checkpoint_path):
    """Loads a single-file safetensors checkpoint, packing q/k/v and gate/up into the fused
    projections (qwen3_naive.py:1682-1730).  lm_head.weight is skipped (tied)."""
    import struct

    dtype_map = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}
    device = next(model.parameters()).device
    packed = getattr(model, "packed_modules_mapping", {})
    with open(checkpoint_path, "rb") as f:
        header_size = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(header_size).decode("utf-8"))
        for name, info in header.items():
            if name == "__metadata__" or name == "lm_head.weight":
                continue
            start, end = info["data_offsets"]
            f.seek(8 + header_size + start)
            raw = f.read(end - start)
            t = torch.frombuffer(bytearray(raw), dtype=dtype_map[info["dtype"]]).reshape(info["shape"]).to(device)
            for key, (fused, shard) in packed.items():
                if key in name:
                    param = model.get_parameter(name.replace(key, fused))
                    if shard in ("q", "gate"):
                        off = 0
                    elif shard == "k":
                        off = param.shape[0] - 2 * t.shape[0]
                    else:
                        off = param.shape[0] - t.shape[0]
                    param.data[off:off + t.shape[0]] = t
                    break
            else:
                model.get_parameter(name).data.copy_(t)


def tokenize(text, tokenizer, device=None):
    """One user turn in the tokenizer's chat template, generation prompt appended, encoded to a
    [1, L] int64 tensor (test_prefix_cache.py:37-43, test_chunked_prefill.py:38-44,
    qwen3_grpo_train.py:317-324)."""
    messages = [{"role": "user", "content": text}]
    formatted = tokenizer.apply_chat_template(messages, tokenize=False, add_generation_prompt=True)
    ids = tokenizer.encode(formatted, return_tensors="pt")
    return ids.to(device) if device is not None else ids


def load_model_and_tokenizer(model_path, device="cuda"):
    """Tokenizer, config and weights of a Qwen3 checkpoint directory (config.json,
    model.safetensors and the tokenizer files), as test_prefix_cache.py:22-35 loads them.
    Returns (model, tokenizer, config)."""
    from pathlib import Path

    from transformers import AutoTokenizer
    tokenizer = AutoTokenizer.from_pretrained(model_path)
    config = Qwen3Config.from_json(str(Path(model_path) / "config.json"))
    model = build_model(config, device=device, seed=None)
    load_weights(model, str(Path(model_path) / "model.safetensors"))
    return model, tokenizer, config
