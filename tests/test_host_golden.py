"""Host logic vs golden traces recorded from the reference (CPU only, bit-exact).

Covers Sequence/BlockManager (qwen3_naive.py:191-375), the metadata builders
_prepare_step/_prepare_decode (:1147-1225) and the whole continuous-batching scheduler
of generate_continuous_with_logprobs (:1474-1679): admission, chunked prefill,
decode-first budget, prefix-cache hits, LIFO preemption, EOS / max-token finish.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from qwen3_naive_inference_b200.qwen3_naive import BlockManager, Qwen3Config, Qwen3ForCausalLM, Sequence

GOLD = Path(__file__).parent / "golden"


def load(name):
    with open(GOLD / name) as f:
        return json.load(f)


def bm_state(bm, seqs):
    return {"free": list(bm.free), "ref_count": list(bm.ref_count), "block_hash": [str(h) for h in bm.block_hash],
            "hash_to_block": sorted([str(h), b] for h, b in bm.hash_to_block.items()),
            "tables": [list(s.block_table) for s in seqs], "kv_len": [s.kv_len for s in seqs]}


def test_compute_hash_golden():
    for case in load("block_manager.json")["hashes"]:
        h1 = BlockManager.compute_hash(case["tokens"])
        assert str(h1) == case["h"]
        assert str(BlockManager.compute_hash(case["tokens"], h1)) == case["h_chain"]


def test_block_manager_trace_golden():
    g = load("block_manager.json")
    bm = BlockManager(12, 256)
    seqs = {k: Sequence(v) for k, v in g["prompts"].items()}
    order = g["order"]
    trace = iter(g["trace"])

    def prefill(s):
        s.num_scheduled_tokens = s.num_prompt_tokens - s.kv_len
        s.kv_len += s.num_scheduled_tokens
        bm.hash_blocks(s)
        s.num_scheduled_tokens = 0

    for op in ["alloc A", "prefill A", "alloc B", "prefill B", "alloc C", "prefill C", "dealloc A", "alloc D",
               "prefill D", "append D x300", "can_append C", "dealloc B", "alloc E", "prefill E", "append C x600"]:
        kind, name = op.split()[:2]
        s = seqs[name]
        if kind == "alloc":
            bm.allocate(s)
        elif kind == "prefill":
            prefill(s)
        elif kind == "dealloc":
            bm.deallocate(s.block_table)
            s.block_table = []
            s.kv_len = 0
        elif kind == "can_append":
            assert next(trace) == {"op": op, "result": bm.can_append(s)}
            continue
        elif kind == "append":
            n = int(op.split()[2][1:])
            for i in range(n):
                if not bm.can_append(s):
                    assert next(trace) == {"op": f"{op} stopped at {i}", "result": False}
                    break
                bm.may_append(s)
                s.append_token(1000 + i)
                s.num_scheduled_tokens = 1
                s.kv_len += 1
                bm.hash_blocks(s)
                s.num_scheduled_tokens = 0
        exp = next(trace)
        assert exp["op"] == op
        got = bm_state(bm, [seqs[k] for k in order])
        for key in got:
            assert got[key] == exp[key], (op, key)


def _model_meta():
    m = Qwen3ForCausalLM.__new__(Qwen3ForCausalLM)
    return m


def test_prepare_step_and_decode_golden():
    for case in load("prepare.json"):
        seqs = []
        for d in case["seqs"]:
            s = Sequence(d["token_ids"][:d["prompt_len"]])
            s.token_ids = list(d["token_ids"])
            s.last_token = s.token_ids[-1]
            s.kv_len = d["kv_len"]
            s.num_scheduled_tokens = d["n"]
            s.block_table = list(d["block_table"])
            seqs.append(s)
        arrays, mq, mk = Qwen3ForCausalLM._step_arrays(_model_meta(), seqs)
        ids, pos, cu_q, cu_k, blk, bt, _tiles = arrays
        st = case["step"]
        assert ids.tolist() == st["input_ids"]
        assert pos.tolist() == st["positions"]
        assert cu_q.tolist() == st["cu_q"] and cu_k.tolist() == st["cu_k"]
        assert (mq, mk) == (st["max_q"], st["max_k"])
        assert blk.tolist() == st["block_mapping"]
        assert bt.tolist() == st["block_tables"]
        assert ids.dtype == np.int64 and pos.dtype == np.int64
        assert cu_q.dtype == np.int32 and blk.dtype == np.int32 and bt.dtype == np.int32
        if "decode" in case:
            dec = [seqs[i] for i in case["decode_idx"]]
            got = Qwen3ForCausalLM._decode_arrays(_model_meta(), dec)
            for k, v in zip(["input_ids", "positions", "context_lens", "block_tables", "slot_mapping"], got):
                assert v.tolist() == case["decode"][k], k


def _fake_next(input_id, position, vocab):
    return (input_id * 7 + position * 13 + 1) % vocab


class _HostOnlyModel(Qwen3ForCausalLM):
    """The product scheduler with the device step replaced by the golden generator's stand-in."""

    def __init__(self, num_blocks, vocab):
        torch.nn.Module.__init__(self)
        self._num_blocks = num_blocks
        self.vocab = vocab
        self.trace = []

    def _gen_setup(self, prompts, max_new_tokens, temperature, top_k):
        return {}

    def _launch_step(self, ctx, scheduled, n_sampled, all_decode, step):
        if all_decode:
            ids, pos, cl, bt, slots = self._decode_arrays(scheduled)
            self.trace.append({"kind": "decode", "input_ids": ids.tolist(), "positions": pos.tolist(),
                               "context_lens": cl.tolist(), "block_tables": bt.tolist(),
                               "slot_mapping": slots.tolist()})
            rows = list(range(len(scheduled)))
        else:
            arrays, _, _ = self._step_arrays(scheduled)
            ids, pos, cu_q, cu_k, blk, bt, _ = arrays
            self.trace.append({"kind": "step", "n": [s.num_scheduled_tokens for s in scheduled],
                               "input_ids": ids.tolist(), "positions": pos.tolist(), "cu_q": cu_q.tolist(),
                               "cu_k": cu_k.tolist(), "block_mapping": blk.tolist(), "block_tables": bt.tolist()})
            ends = np.cumsum([s.num_scheduled_tokens for s in scheduled]) - 1
            rows = [int(ends[j]) for j, s in enumerate(scheduled)
                    if s.num_scheduled_tokens == 1 or s.kv_len + s.num_scheduled_tokens >= s.num_prompt_tokens]
        ctx["toks"] = [_fake_next(int(ids[r]), int(pos[r]), self.vocab) for r in rows]
        assert len(ctx["toks"]) == n_sampled

    def _finish_step(self, ctx, pending, n, record_logprobs):
        return ctx.get("toks", [])[:n], [0.0] * n


@pytest.mark.parametrize("case", range(3))
def test_scheduler_trace_golden(case):
    g = load("scheduler.json")[case]
    m = _HostOnlyModel(g["num_blocks"], g["vocab"])
    toks, gen, lps, plens = m.generate_continuous_with_logprobs(
        [torch.tensor([p]) for p in g["prompts"]], max_new_tokens=g["max_new"], temperature=1.0, top_k=1,
        eos_token_ids=g["eos"])
    assert len(m.trace) == len(g["steps"])
    for i, (a, b) in enumerate(zip(m.trace, g["steps"])):
        assert a == b, f"step {i} differs ({a['kind']} vs {b['kind']})"
    assert toks == g["seq_tokens"]
    assert gen == g["generated"]
    assert plens == g["prompt_lens"]
    assert [len(x) for x in lps] == g["n_logprobs"]


def test_scheduler_golden_exercises_preemption_and_chunking():
    """The recorded traces cover the interesting scheduler paths."""
    g = load("scheduler.json")
    # case 1: tight pool -> LIFO preemption happened
    assert g[1]["preemptions"] > 0
    # case 2: a 2100-token prompt is split into chunks of the 2048 budget
    assert any(max(s["n"]) == 2048 for s in g[2]["steps"] if s["kind"] == "step")
    # case 2 uses EOS ids: some generation ends before max_new tokens
    assert any(len(x) < g[2]["max_new"] for x in g[2]["generated"])
