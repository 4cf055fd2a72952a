"""Model-level parity on the GPU: the product path (CUDA kernels) vs the CPU oracle.

A tiny Qwen3 shape (head_dim 128, GQA 4q/2kv, 2 layers) shares seeded weights with the
oracle.  Tolerances follow the north star: log-probs and loss within 2e-3 relative
(bf16), gradients within 1e-2 cosine distance, greedy tokens exact where the oracle's
top-2 logits are separated by more than bf16 noise.
"""
import math

import numpy as np
import pytest
import torch

from oracle import ref_model
from oracle import ref_ops as R
from qwen3_naive_inference_b200 import ops
from qwen3_naive_inference_b200 import qwen3_grpo_train as G
from qwen3_naive_inference_b200.qwen3_naive import BlockManager, Qwen3Config, Sequence, build_model

pytestmark = pytest.mark.gpu

TINY = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=128, intermediate_size=256,
            num_hidden_layers=2, vocab_size=512, max_position_embeddings=4096)


@pytest.fixture(scope="module")
def setup(cuda):
    cfg = Qwen3Config(**TINY)
    params = ref_model.init_params(cfg, seed=0)
    model = build_model(cfg, device=cuda, seed=None)
    sd = model.state_dict()
    with torch.no_grad():
        for k, v in params.items():
            sd[k].copy_(v)
    model._num_blocks = 64
    return cfg, params, model


def rel_err(a, b):
    return ((a.float().cpu() - b.float()).abs().max() / (b.float().abs().max() + 1e-9)).item()


def test_tied_weights_share_storage(setup):
    _, _, model = setup
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()
    assert model.lm_head.weight is not model.model.embed_tokens.weight


def test_dense_logits_vs_oracle(setup, cuda):
    cfg, params, model = setup
    ids = torch.randint(0, cfg.vocab_size, (3, 77), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        mine = model(ids.to(cuda))
        ref = ref_model.logits(params, cfg, ids)
    assert rel_err(mine, ref) < 0.05
    assert (mine.float().cpu().argmax(-1) == ref.float().argmax(-1)).float().mean() > 0.95


@pytest.mark.parametrize("shift", [False, True])
def test_forward_logprob_vs_oracle(setup, cuda, shift):
    cfg, params, model = setup
    ids = torch.randint(0, cfg.vocab_size, (2, 150), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        mine = G.forward_logprob(model, ids.to(cuda), shift=shift).cpu()
        ref = ref_model.forward_logprob(params, cfg, ids, shift=shift)
    rel = ((mine - ref).abs() / ref.abs().clamp_min(1e-3))
    assert rel.mean().item() < 2e-3, rel.mean().item()
    assert (mine - ref).abs().max().item() < 0.05


@pytest.mark.parametrize("rope_grad", [False, True])
def test_grpo_grads_vs_oracle(setup, cuda, rope_grad):
    cfg, params, model = setup
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, cfg.vocab_size, (2, 96), generator=g)
    mask = torch.zeros(2, 96)
    mask[0, 40:] = 1
    mask[1, 10:80] = 1
    with torch.no_grad():
        base = ref_model.forward_logprob(params, cfg, ids)
    old = base + 0.05 * torch.randn(base.shape, generator=g)
    tok_adv = torch.tensor([0.9, -1.1])[:, None] * mask
    # oracle autograd
    p = {k: v.clone().requires_grad_(True) for k, v in params.items() if k != "lm_head.weight"}
    p["lm_head.weight"] = params["lm_head.weight"].clone().requires_grad_(True)
    lp = ref_model.forward_logprob(p, cfg, ids, rope_grad=rope_grad)
    loss_ref = R.ppo_loss(old, lp, tok_adv, mask)
    loss_ref.backward()
    # product
    model.set_rope_grad(rope_grad)
    model.zero_grad(set_to_none=True)
    lpm = G.forward_logprob(model, ids.to(cuda))
    loss = G.ppo_clipped_loss(old.to(cuda), lpm, tok_adv.to(cuda), mask.to(cuda))
    loss.backward()
    model.set_rope_grad(True)
    assert abs(loss.item() - loss_ref.item()) <= 2e-3 * abs(loss_ref.item()) + 1e-4
    named = dict(model.named_parameters())
    for name, pr in p.items():
        gm = named[name].grad
        if pr.grad is None or pr.grad.float().norm() == 0:
            assert gm is None or gm.float().norm().item() < 1e-5, name
            continue
        cos = torch.nn.functional.cosine_similarity(gm.float().cpu().reshape(-1), pr.grad.float().reshape(-1), 0)
        assert 1 - cos.item() < 1e-2, (name, cos.item())


def _prefill(model, seqs):
    ids, pos, cu_q, cu_k, mq, mk, blk, bt = model._prepare_step(seqs)
    h = model.model.forward_prefill(ids, pos, cu_q, cu_k, mq, mk, blk, bt)
    return h, cu_q


def test_paged_prefill_matches_dense_and_chunking(setup, cuda):
    """Reference Case 1 (test_chunked_prefill.py:63-155) on random weights: chunked and
    unchunked prefill agree (top-1 equal, top-20 overlap >= 19), and both match the dense path."""
    cfg, params, model = setup
    model.allocate_global_kv_cache()
    g = torch.Generator().manual_seed(4)
    toks = torch.randint(0, cfg.vocab_size, (700,), generator=g).tolist()
    bm = BlockManager(model._num_blocks, 256)
    s = Sequence(toks)
    bm.allocate(s)
    s.num_scheduled_tokens = len(toks)
    with torch.no_grad():
        h, _ = _prefill(model, [s])
        full = torch.nn.functional.linear(h, model.lm_head.weight)[-1].float()
        dense = model(torch.tensor([toks], device=cuda))[0, -1].float()
    assert rel_err(full, dense.cpu()) < 0.03
    bm2 = BlockManager(model._num_blocks, 256)
    s2 = Sequence(toks)
    bm2.allocate(s2)
    with torch.no_grad():
        while s2.kv_len < s2.num_prompt_tokens:
            s2.num_scheduled_tokens = min(256, s2.num_prompt_tokens - s2.kv_len)
            h2, _ = _prefill(model, [s2])
            s2.kv_len += s2.num_scheduled_tokens
            bm2.hash_blocks(s2)
        chunked = torch.nn.functional.linear(h2, model.lm_head.weight)[-1].float()
    assert full.argmax().item() == chunked.argmax().item()
    overlap = len(set(full.topk(20).indices.tolist()) & set(chunked.topk(20).indices.tolist()))
    assert overlap >= 19


def _oracle_lp(params, cfg, tokens, temperature=1.0):
    with torch.no_grad():
        lg = ref_model.logits(params, cfg, torch.tensor([tokens]))[0].float()
    return lg, torch.log_softmax(lg / temperature, -1)


def test_generate_greedy_teacher_forced(setup, cuda):
    cfg, params, model = setup
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g) for L in (3, 250, 256, 300)]
    torch.manual_seed(0)
    seq_tokens, gen = model.generate_continuous([p.to(cuda) for p in prompts], max_new_tokens=24, top_k=1,
                                                temperature=1.0)
    checked = 0
    for toks, p in zip(seq_tokens, prompts):
        L = p.shape[1]
        lg, _ = _oracle_lp(params, cfg, toks)
        for t in range(L, len(toks)):
            top2 = lg[t - 1].topk(2).values
            if (top2[0] - top2[1]).item() > 0.05:
                assert toks[t] == lg[t - 1].argmax().item(), (L, t)
                checked += 1
    assert checked > 40


@pytest.mark.parametrize("top_k,temp", [(None, 1.0), (20, 0.8)])
def test_generate_logprobs_teacher_forced(setup, cuda, top_k, temp):
    cfg, params, model = setup
    g = torch.Generator().manual_seed(6)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g) for L in (17, 260)]
    torch.manual_seed(1)
    toks, gen, lps, plens = model.generate_continuous_with_logprobs([p.to(cuda) for p in prompts],
                                                                    max_new_tokens=20, temperature=temp, top_k=top_k)
    checked = 0
    for t, lp, pl in zip(toks, lps, plens):
        assert len(lp) == len(t) - pl == 20
        lg, _ = _oracle_lp(params, cfg, t)
        for j, v in enumerate(lp):
            pos = pl + j
            row = lg[pos - 1]
            if top_k is not None:
                srt = row.sort(descending=True).values
                # GPU and CPU logits differ at bf16 noise level; a near-tie at the k-th value
                # can swap which token is kept, so such positions are not comparable
                if (srt[top_k - 1] - srt[top_k]).item() < 0.01:  # ~5 bf16 ulps at this logit scale
                    continue
            probs, logps = R.sample_distribution(row[None].to(torch.bfloat16), temp, top_k)
            ref = logps[0, t[pos]].item()
            assert math.isfinite(ref), "sampled a token outside the oracle's support"
            assert abs(v - ref) < 2e-3 * abs(ref) + 0.05, (pos, v, ref)
            checked += 1
    assert checked >= 5


def test_cuda_graph_decode_matches_eager(setup, cuda):
    cfg, params, model = setup
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (5, 40, 70)]
    torch.manual_seed(3)
    a = model.generate_continuous(prompts, max_new_tokens=16, top_k=1)[1]
    saved = model._has_cuda_graphs
    model._run_decode_graph = lambda *args, **kw: None  # force the eager decode path
    try:
        torch.manual_seed(3)
        b = model.generate_continuous(prompts, max_new_tokens=16, top_k=1)[1]
    finally:
        del model._run_decode_graph
    flat_a = sum(a, [])
    flat_b = sum(b, [])
    assert len(flat_a) == len(flat_b)
    assert np.mean([x == y for x, y in zip(flat_a, flat_b)]) > 0.95
    assert saved


def test_fused_grpo_step_matches_autograd_path(setup, cuda):
    """policy_loss_backward (fused lm_head/log-prob/loss/backward, microbatched) gives the
    same loss and gradients as forward_logprob + ppo_clipped_loss + autograd."""
    cfg, params, model = setup
    g = torch.Generator().manual_seed(8)
    N, G_ = 6, 3
    lens = [40, 77, 130, 64, 200, 90]
    plens = [10, 30, 50, 20, 60, 45]
    toks = [torch.randint(0, cfg.vocab_size, (L,), generator=g).tolist() for L in lens]
    olds = [(-5 + 0.1 * torch.randn(L - pl, generator=g)).tolist() for L, pl in zip(lens, plens)]
    rewards = torch.tensor([1., 0., 1., 1., 1., 0.])
    gids = [0, 0, 0, 1, 1, 1]
    batch = G.PackedBatch(toks, plens, olds, rewards, gids, cuda, shift=True)
    model.zero_grad(set_to_none=True)
    loss, new_lp = G.policy_loss_backward(model, batch, microbatch_tokens=256, chunk_rows=100)
    fused = {k: p.grad.detach().clone() for k, p in model.named_parameters() if p.grad is not None}
    # autograd path on padded rows with shift=True
    S = batch.S
    ids = torch.zeros(N, S, dtype=torch.long)
    for i, t in enumerate(toks):
        ids[i, :len(t)] = torch.tensor(t)
    model.zero_grad(set_to_none=True)
    lp = G.forward_logprob(model, ids.to(cuda), shift=True)
    adv = G.compute_grpo_advantage(rewards.to(cuda), torch.tensor(gids, device=cuda))
    tok_adv = adv[:, None] * batch.mask
    loss2 = G.ppo_clipped_loss(batch.old_lp, lp, tok_adv, batch.mask)
    loss2.backward()
    assert abs(loss[0].item() - loss2.item()) <= 2e-3 * abs(loss2.item()) + 1e-5
    m = batch.mask.bool()
    assert torch.allclose(new_lp[m], lp.detach()[m], rtol=2e-3, atol=2e-2)
    for k, p in model.named_parameters():
        if k not in fused:
            continue
        cos = torch.nn.functional.cosine_similarity(fused[k].float().reshape(-1), p.grad.float().reshape(-1), 0)
        assert 1 - cos.item() < 1e-2, (k, cos.item())


def test_grouped_rollout_teacher_forced(setup, cuda):
    """Shared-prompt rollout (one prefill per group, shared-prefix decode attention): greedy tokens and
    full-vocabulary log-probs match the oracle teacher-forced on the produced sequences."""
    cfg, params, model = setup
    g = torch.Generator().manual_seed(10)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g) for L in (30, 260, 520)]
    torch.manual_seed(4)
    toks, gen, lps, plens = model.generate_grouped_with_logprobs([p.to(cuda) for p in prompts], 4,
                                                                 max_new_tokens=16, temperature=1.0, top_k=1)
    assert plens == [30] * 4 + [260] * 4 + [520] * 4
    checked = 0
    for t, pl in zip(toks, plens):
        lg, _ = _oracle_lp(params, cfg, t)
        for pos in range(pl, len(t)):
            top2 = lg[pos - 1].topk(2).values
            if (top2[0] - top2[1]).item() > 0.05:
                assert t[pos] == lg[pos - 1].argmax().item(), (pl, pos)
                checked += 1
    assert checked > 60
    torch.manual_seed(5)
    toks, gen, lps, plens = model.generate_grouped_with_logprobs([p.to(cuda) for p in prompts], 4,
                                                                 max_new_tokens=12, temperature=1.0, top_k=None)
    members_differ = len({tuple(x) for x in gen[:4]}) > 1
    assert members_differ  # independent draws per member
    for t, lp, pl in zip(toks, lps, plens):
        lg, _ = _oracle_lp(params, cfg, t)
        for j, v in enumerate(lp):
            _, logps = R.sample_distribution(lg[pl + j - 1][None].to(torch.bfloat16), 1.0, None)
            ref = logps[0, t[pl + j]].item()
            assert abs(v - ref) < 2e-3 * abs(ref) + 0.05, (pl, j, v, ref)
    ops.check_device_errors()


@pytest.mark.parametrize("graphs", [True, False])
def test_grouped_rollout_mixed_steps(setup, cuda, graphs):
    """Prompts longer in total than one step's 2048-token budget: the last prompt's prefill
    runs in the same step as the other groups' first decode tokens (prefill rows on the paged
    varlen kernel, decode rows on the grouped decode, whose keys skip the unused tail of the
    shared last prompt page).  Greedy tokens match the oracle teacher-forced; eager decode
    (graphs=False) and graph replay produce the same tokens."""
    cfg, params, model = setup
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (30, 260, 520, 1400)]
    model.use_cuda_graphs = graphs
    try:
        toks, gen, lps, plens = model.generate_grouped_with_logprobs(prompts, 4, max_new_tokens=10,
                                                                     temperature=1.0, top_k=1)
    finally:
        model.use_cuda_graphs = True
    assert model.rollout_stats["steps"] > model.rollout_stats.get("decode_steps", 0) + 1  # a mixed step ran
    checked = 0
    for t, pl in zip(toks, plens):
        lg, _ = _oracle_lp(params, cfg, t)
        for pos in range(pl, len(t)):
            top2 = lg[pos - 1].topk(2).values
            if (top2[0] - top2[1]).item() > 0.05:
                assert t[pos] == lg[pos - 1].argmax().item(), (pl, pos, graphs)
                checked += 1
    assert checked > 60
    ops.check_device_errors()


def test_grouped_rollout_matches_plain_greedy(setup, cuda):
    cfg, params, model = setup
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (77, 300)]
    torch.manual_seed(6)
    _, grouped, _, _ = model.generate_grouped_with_logprobs(prompts, 2, max_new_tokens=20, top_k=1, temperature=1.0)
    torch.manual_seed(6)
    _, plain = model.generate_continuous([p for p in prompts for _ in range(2)], max_new_tokens=20, top_k=1,
                                         temperature=1.0)
    a, b = sum(grouped, []), sum(plain, [])
    assert len(a) == len(b)
    assert np.mean([x == y for x, y in zip(a, b)]) > 0.95


def test_generation_reads_only_written_cache_slots(setup, cuda):
    """Every K/V slot a step reads was written first: with the page pool filled with NaN
    beforehand (memory left by earlier work can hold any bits), greedy generation -- the decode
    graphs' capture warm-up and padded batch rows, which must read no keys, included -- and the
    grouped rollout give the same tokens as on a zeroed pool, and no device error is raised."""
    cfg, params, model = setup
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (3, 250, 256, 300, 17)]
    model.allocate_global_kv_cache()

    def run(fill):
        for layer in model.model.layers:
            layer.self_attn.k_cache.fill_(fill)
            layer.self_attn.v_cache.fill_(fill)
        model._has_cuda_graphs = False  # recapture: the capture warm-up runs on this pool too
        torch.manual_seed(0)
        plain = model.generate_continuous(prompts, max_new_tokens=20, top_k=1, temperature=1.0)[1]
        torch.manual_seed(0)
        grouped = model.generate_grouped_with_logprobs(prompts[:3], 3, max_new_tokens=20, top_k=1,
                                                       temperature=1.0)[1]
        ops.check_device_errors()
        return plain, grouped

    assert run(float("nan")) == run(0.0)


def _greedy_checked(params, cfg, toks, L):
    """Positions of toks[L:] whose greedy choice the oracle confirms (top-2 logits more than bf16
    noise apart); asserts every confirmed position matches.  Returns how many were confirmed."""
    lg, _ = _oracle_lp(params, cfg, toks)
    checked = 0
    for t in range(L, len(toks)):
        top2 = lg[t - 1].topk(2).values
        if (top2[0] - top2[1]).item() > 0.05:
            assert toks[t] == lg[t - 1].argmax().item(), (L, t)
            checked += 1
    return checked


def test_non_paged_generation_modes(setup, cuda):
    """generate_varlen (packed recompute), generate_naive (recompute) and generate_kvcache (prefill
    + paged decode), qwen3_naive.py:842-990: greedy tokens match the oracle teacher-forced, and each
    mode treats EOS as the reference does (naive: stop before appending; kvcache: the first token is
    always appended, a later EOS stops before it; varlen: append, then the sequence finishes)."""
    cfg, params, model = setup
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (5, 70, 260)]
    seqs, gen = model.generate_varlen(prompts, max_new_tokens=12, top_k=1, temperature=1.0)
    assert [len(x) for x in gen] == [12, 12, 12]
    assert sum(_greedy_checked(params, cfg, t, p.shape[1]) for t, p in zip(seqs, prompts)) > 15
    checked, naive = 0, []
    for p in prompts:
        out = model.generate_naive(p, max_new_tokens=12, top_k=1, temperature=1.0)
        assert out.shape == (1, p.shape[1] + 12)
        checked += _greedy_checked(params, cfg, out[0].tolist(), p.shape[1])
        naive.append(out)
    assert checked > 15
    two = torch.cat([prompts[1], torch.randint(0, cfg.vocab_size, (1, 70), generator=g).to(cuda)])
    out = model.generate_kvcache(two, max_new_tokens=12, top_k=1, temperature=1.0)
    assert out.shape == (2, 82)
    assert sum(_greedy_checked(params, cfg, row, 70) for row in out.tolist()) > 10
    # EOS rules, each mode with its own first greedy token of prompts[0] as the EOS id
    eos_n = naive[0][0, 5].item()
    assert model.generate_naive(prompts[0], max_new_tokens=12, top_k=1, temperature=1.0,
                                eos_token_ids=[eos_n]).shape == (1, 5)
    eos_k = model.generate_kvcache(prompts[0], max_new_tokens=12, top_k=1, temperature=1.0)[0, 5].item()
    kv = model.generate_kvcache(prompts[0], max_new_tokens=12, top_k=1, temperature=1.0, eos_token_ids=[eos_k])
    assert kv[0, 5].item() == eos_k and eos_k not in kv[0, 6:].tolist()
    eos_v = seqs[0][5]
    _, g2 = model.generate_varlen(prompts, max_new_tokens=12, top_k=1, temperature=1.0, eos_token_ids=[eos_v])
    assert g2[0] == [eos_v] and all(eos_v not in x[:-1] for x in g2[1:])
    with pytest.raises(RuntimeError):
        model.generate_naive(two, max_new_tokens=2, top_k=1, temperature=1.0, eos_token_ids=[eos_n])
    ops.check_device_errors()


def test_grpo_step_end_to_end(setup, cuda):
    cfg, params, model = setup
    ref = G.make_reference_copy(model)
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (12, 300)]
    before = model.model.layers[0].mlp.down_proj.weight.detach().clone()
    torch.manual_seed(2)
    out = G.grpo_step(model, opt, prompts, ref_model=ref, group_size=4, max_new_tokens=24, temperature=1.0,
                      beta=0.04, reward_gen=torch.Generator().manual_seed(0), microbatch_tokens=512)
    assert math.isfinite(out["loss"]) and abs(out["kl"]) < 1e-3
    assert out["completion_tokens"] == 8 * 24
    assert not torch.equal(before, model.model.layers[0].mlp.down_proj.weight)
    ops.check_device_errors()


def test_rollout_single_and_batch_reference_signatures(setup, cuda):
    """rollout_single(model, prompt_ids, tokenizer) and rollout_batch(model, tokenizer, prompts)
    with the reference's signatures (qwen3_grpo_train.py:69-120, :212-258): prompt + response ids,
    each response token's log-prob at its own position, the response mask, per-completion rewards
    and prompt ids; greedy completions equal generate_continuous's."""
    cfg, params, model = setup
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab_size, (1, L), generator=g).to(cuda) for L in (20, 33)]
    ids, old, mask = G.rollout_single(model, prompts[0], None, max_new_tokens=6, top_k=1, temperature=1.0,
                                      eos_token_ids=None)
    assert ids.shape == (1, 26) and old.shape == (26,) and mask.shape == (26,)
    assert torch.equal(ids[0, :20], prompts[0][0])
    assert mask[:20].sum().item() == 0 and mask[20:].sum().item() == 6
    assert torch.all(old[:20] == 0) and torch.all(old[20:] == 0)  # greedy: log-prob 0
    toks, _ = model.generate_continuous([prompts[0]], max_new_tokens=6, top_k=1, temperature=1.0)
    assert ids[0].tolist() == toks[0]
    ids, old, mask, rewards, pid = G.rollout_batch(model, None, prompts, n_rollout=2, max_new_tokens=7,
                                                   temperature=1.0, top_k=20, eos_token_ids=None)
    assert ids.shape == (4, 40) and old.shape == (4, 40) and mask.shape == (4, 40)
    assert pid.tolist() == [0, 0, 1, 1]
    assert mask.sum(1).tolist() == [7.0, 7.0, 7.0, 7.0]
    assert torch.all(old[mask.bool()] <= 0) and torch.all(old[~mask.bool()] == 0)
    assert rewards.tolist() == [1.0] * 4  # 7 completion tokens > 5 (no tokenizer: the token-count rule)
