"""Host logic of the grouped (shared-prompt) rollout, CPU only.

The device step is replaced by a deterministic stand-in: member i's first token is a
function of the prompt and i, every later token a function of the previous token and its
position.  Whatever the scheduling (chunked prefill, preemption), each completion must
come out identical to a direct chain; pages must be shared exactly within a group, owned
pages never shared, and the pool must be fully released at the end.
"""
import numpy as np
import pytest
import torch

from qwen3_naive_inference_b200 import qwen3_naive as QN
from qwen3_naive_inference_b200.qwen3_naive import Qwen3ForCausalLM

V = 4096


def nxt(tok, pos):
    return (tok * 7 + pos * 13 + 1) % V


class HostGrouped(Qwen3ForCausalLM):
    def __init__(self, num_blocks):
        torch.nn.Module.__init__(self)
        self._num_blocks = num_blocks
        self.max_model_len = None
        self.checks = 0
        self.resets = 0
        self.pipelined = 0
        self.fed = 0
        self.feed_on_device = True  # steps queued ahead take their inputs from the step before

    def _grouped_setup(self, max_ctx, max_shared, temperature, top_k):
        return {}

    def _grouped_launch(self, ctx, prefill, done, decode_rows, groups_rows, step, G, n_samples):
        toks = []
        for g in done:
            for i in range(G):
                toks.append((nxt(g.prompt[-1], g.L - 1) + i) % V)
        for m in decode_rows:
            toks.append(nxt(m.last_token, m.num_tokens - 1))
        self._check(decode_rows, groups_rows)
        ctx["toks"] = toks
        assert len(toks) == n_samples

    def _graph_fits(self, bs, width=0):
        return self.feed_on_device

    # pipelined decode steps: the input token of a row comes from the host (the previous step's
    # read-back) or, for a step queued before that read-back, from the previous step's samples
    # (the device gather: row i takes sample src[i] where src[i] >= 0); its position from the
    # step's metadata
    def _decode_submit(self, ctx, rows, groups_rows, step, ids, arrays, feed=None):
        pos, cl, bt, slots = arrays
        assert list(cl) == [m.kv_len for m in rows]
        self._check(rows, groups_rows)
        self.pipelined += 1
        if feed is not None:
            src, prev = feed
            assert len(src) == len(rows)
            ids = [prev[j] if j >= 0 else t for j, t in zip(src, ids)]
            self.fed += 1
        return [nxt(int(t), int(p)) for t, p in zip(ids, pos)]

    def _decode_collect(self, ctx, handle):
        return np.asarray(handle, dtype=np.int64), np.zeros(len(handle), dtype=np.float32)

    def _check(self, decode_rows, groups_rows):
        # structural checks on the page tables of everything that runs this step: the whole
        # prompt is shared, own tokens start on a fresh page, own pages belong to one member
        own_seen = set()
        seen_rows = set()
        for rows, shared, start in groups_rows:
            members = [decode_rows[r] for r in rows]
            n_sh = -(-shared // 256)
            assert shared == members[0].num_prompt_tokens and start == n_sh * 256
            first = members[0].block_table[:n_sh]
            for m in members:
                assert m.block_table[:n_sh] == first
                assert start <= m.kv_len < len(m.block_table) * 256
                for p in m.block_table[n_sh:]:
                    assert p not in own_seen and p not in first
                    own_seen.add(p)
            seen_rows.update(rows)
        assert seen_rows == set(range(len(decode_rows)))  # every decode row is in one group
        self.checks += 1

    def _finish_step(self, ctx, pending, n, record_logprobs):
        return ctx.get("toks", [])[:n], [0.0] * n


EOS = set(range(0, V, 97))  # ~1% of token values end a completion


def expected(prompt, i, n, eos=None):
    L = len(prompt)
    t = (nxt(prompt[-1], L - 1) + i) % V
    out = [t]
    for k in range(n - 1):
        if eos is not None and t in eos:
            break
        t = nxt(t, L + k)
        out.append(t)
    return out


@pytest.mark.parametrize("num_blocks,lens,G,new,eos", [
    (400, [5, 256, 300, 700, 2100, 512, 1], 8, 40, None),  # roomy pool, chunked prefill of a long prompt
    (30, [600, 300, 200, 256], 4, 300, None),                # tight pool: group preemption
    (60, [100] * 12, 8, 20, None),                           # many groups, all partial pages
    (400, [5, 256, 300, 700, 512, 1], 8, 200, EOS),          # completions end at EOS mid-pipeline
    (14, [600, 300, 200, 256], 4, 300, EOS),                 # EOS and preemption
])
def test_grouped_rollout_host_logic(num_blocks, lens, G, new, eos):
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, V, L).tolist() for L in lens]
    m = HostGrouped(num_blocks)
    resets = [0]
    orig = QN._Group.reset

    def counting_reset(self):
        resets[0] += 1
        orig(self)

    QN._Group.reset = counting_reset
    try:
        toks, gen, lps, plens = m.generate_grouped_with_logprobs([torch.tensor([p]) for p in prompts], G,
                                                                 max_new_tokens=new, temperature=1.0, top_k=None,
                                                                 eos_token_ids=eos)
    finally:
        QN._Group.reset = orig
    assert plens == [len(p) for p in prompts for _ in range(G)]
    for gi, p in enumerate(prompts):
        for i in range(G):
            k = gi * G + i
            assert gen[k] == expected(p, i, new, eos), (gi, i)
            assert toks[k] == p + gen[k]
            assert len(lps[k]) == len(gen[k])
    assert m.checks > 0 and m.pipelined > 0
    if num_blocks in (14, 30):
        assert resets[0] > len(prompts)  # at least one group was preempted and restarted


@pytest.mark.parametrize("eos", [None, EOS])
def test_pipelined_decode_matches_synchronous(eos):
    """Submitting step k+1 before step k's bookkeeping (speculating on EOS) -- with its inputs
    from the host after step k's read-back, or gathered from step k's samples before it -- gives
    exactly the synchronous scheduler's completions and leaves no page referenced."""
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, V, int(L)).tolist() for L in rng.integers(64, 513, 16)]
    outs = []
    for pipe, fed in ((False, False), (True, False), (True, True)):
        m = HostGrouped(400)
        m.pipeline_decode = pipe
        m.feed_on_device = fed
        outs.append(m.generate_grouped_with_logprobs([torch.tensor([p]) for p in prompts], 8, max_new_tokens=300,
                                                     temperature=1.0, top_k=None, eos_token_ids=eos))
        assert (m.pipelined > 0) == pipe
        assert (m.fed > 0) == fed
    for o in outs[1:]:
        assert outs[0][0] == o[0] and outs[0][1] == o[1]
