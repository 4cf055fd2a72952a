"""The structural checks of the reference's own GPU tests, restated on the host arrays (CPU; token
ids are synthetic since the tokenizer and weights are absent):
* test_chunked_prefill.py Case 3 (:180-205): a long prompt prefilled in 512-token chunks; each
  step's cu_q[-1] is the chunk and cu_k[-1] the keys before it plus the chunk;
* Case 4 (:228-305): two short sequences decode their first token while a long prompt's first
  chunk is prefilled in the same step: cu_q = [0, 1, 2, 2 + n], cu_k the running kv lengths,
  block tables [3, max_blocks];
* test_prefix_cache.py (:95-190): a prompt whose leading full pages were registered by an earlier
  sequence hits the prefix cache: kv_len > 0, the shared pages' ref_count is 2 and the step's
  cu_k exceeds its cu_q.  (The reference test builds the step with a _prepare_prefill the
  reference does not define; the step builder both share is _prepare_step.)"""
import numpy as np

from qwen3_naive_inference_b200.qwen3_naive import BlockManager, Qwen3ForCausalLM, Sequence

PAGE = 256


def step_arrays(seqs):
    meta = Qwen3ForCausalLM.__new__(Qwen3ForCausalLM)
    arrays, _, _ = Qwen3ForCausalLM._step_arrays(meta, seqs)
    return arrays  # ids, positions, cu_q, cu_k, block_mapping, block_tables, tiles


def prompt(n, seed):
    return np.random.default_rng(seed).integers(0, 151643, n).tolist()


def test_case3_chunked_prefill_cu_seqlens():
    bm = BlockManager(64, PAGE)
    seq = Sequence(prompt(1200, 1), {"temperature": 0.6, "max_tokens": 64})
    bm.allocate(seq)
    chunks = []
    while seq.kv_len < seq.num_prompt_tokens:
        seq.num_scheduled_tokens = min(seq.num_prompt_tokens - seq.kv_len, 512)
        kv_before = seq.kv_len
        _, pos, cu_q, cu_k, blk, _, _ = step_arrays([seq])
        assert cu_q[-1] == seq.num_scheduled_tokens
        assert cu_k[-1] == kv_before + seq.num_scheduled_tokens
        assert pos.tolist() == list(range(kv_before, kv_before + seq.num_scheduled_tokens))
        assert blk.tolist() == [seq.block_table[p // PAGE] * PAGE + p % PAGE for p in pos.tolist()]
        seq.kv_len += seq.num_scheduled_tokens
        bm.hash_blocks(seq)
        chunks.append(seq.num_scheduled_tokens)
        seq.num_scheduled_tokens = 0
    assert chunks == [512, 512, 176]


def test_case4_mixed_decode_and_prefill_chunk():
    bm = BlockManager(64, PAGE)
    seq1 = Sequence(prompt(3, 2), {"temperature": 0.6, "max_tokens": 16})
    seq2 = Sequence(prompt(8, 3), {"temperature": 0.6, "max_tokens": 16})
    seq_long = Sequence(prompt(1200, 4), {"temperature": 0.6, "max_tokens": 16})
    for s in (seq1, seq2):
        bm.allocate(s)
        s.status = "RUNNING"
        s.num_scheduled_tokens = s.num_prompt_tokens - s.kv_len
    step_arrays([seq1, seq2])
    for i, s in enumerate((seq1, seq2)):  # the first sampled token, as after the prefill
        s.append_token(100 + i)
        s.kv_len = s.num_prompt_tokens
        bm.hash_blocks(s)
        s.num_scheduled_tokens = 0
    bm.allocate(seq_long)
    seq_long.status = "RUNNING"
    for s in (seq1, seq2):
        s.num_scheduled_tokens = 1  # decode: kv_len already points at the next position
    seq_long.num_scheduled_tokens = min(512, seq_long.num_prompt_tokens - seq_long.kv_len)
    mixed = [seq1, seq2, seq_long]
    ids, pos, cu_q, cu_k, _, bt, _ = step_arrays(mixed)
    for s in mixed:
        s.kv_len += s.num_scheduled_tokens
    assert cu_q.tolist() == [0, 1, 2, 2 + seq_long.num_scheduled_tokens]
    assert cu_k.tolist() == [0, seq1.kv_len, seq1.kv_len + seq2.kv_len, seq1.kv_len + seq2.kv_len + seq_long.kv_len]
    assert bt.shape == (3, max(len(s.block_table) for s in mixed))
    assert ids[:2].tolist() == [100, 101] and pos[:2].tolist() == [3, 8]


def test_prefix_cache_hit_shares_pages():
    bm = BlockManager(64, PAGE)
    shared = prompt(600, 5)  # two full pages + a partial one
    seq1 = Sequence(shared, {"temperature": 0.6, "max_tokens": 64})
    bm.allocate(seq1)
    seq1.num_scheduled_tokens = seq1.num_prompt_tokens
    step_arrays([seq1])
    seq1.kv_len = seq1.num_prompt_tokens
    bm.hash_blocks(seq1)
    seq5 = Sequence(shared[:540] + prompt(100, 6), {"temperature": 0.6, "max_tokens": 64})
    bm.allocate(seq5)
    assert seq5.kv_len == 2 * PAGE  # both full pages of the common prefix hit
    for i in range(seq5.kv_len // PAGE):
        assert seq5.block_table[i] == seq1.block_table[i]
        assert bm.ref_count[seq5.block_table[i]] == 2
    seq5.num_scheduled_tokens = seq5.num_prompt_tokens - seq5.kv_len
    _, pos, cu_q, cu_k, _, _, _ = step_arrays([seq5])
    assert cu_k[-1] > cu_q[-1]
    assert cu_q[-1] == seq5.num_prompt_tokens - 2 * PAGE and cu_k[-1] == seq5.num_prompt_tokens
    assert pos[0] == 2 * PAGE
