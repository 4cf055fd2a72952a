"""Generates the golden fixtures of tests/golden/ by running the reference itself.

Run in the build container, where the reference source is present:

    python tests/golden/make_golden.py /path/to/qwen3-naive-inference

Everything runs on the CPU.  The reference module is imported unmodified; to make
its CUDA-only pieces run here:
  * TORCHDYNAMO_DISABLE=1 (torch.compile'd RMSNorm / MLP run eagerly);
  * TRITON_INTERPRET=1: the reference's own Triton kernels (_apply_rope_kernel,
    _store_kvcache_kernel) execute in Triton's CPU interpreter.  The interpreter
    truncates on fp32->bf16 casts, unlike the GPU (round to nearest even), so RoPE
    is run with fp32 output and rounded to bf16 by torch (RNE) -- the GPU's
    semantics;
  * pinned host tensors and .cuda() become plain CPU tensors in the metadata
    builders (_prepare_step/_prepare_decode);
  * for the scheduler trace, the model's forward/lm_head are replaced by a
    deterministic stand-in whose logits put all mass on f(input id, position),
    so torch.multinomial is deterministic and the trace pins scheduling,
    paging, preemption and bookkeeping exactly.
Inputs are seeded synthetic data (no dataset, no tokenizer, no checkpoint).
"""
from __future__ import annotations

import json
import os
import random
import sys
from pathlib import Path

os.environ["TORCHDYNAMO_DISABLE"] = "1"
os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
if len(sys.argv) != 2 or not (Path(sys.argv[1]) / "qwen3_naive.py").is_file():
    sys.exit("usage: python tests/golden/make_golden.py <reference checkout holding qwen3_naive.py>")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE.parents[1]))

import qwen3_naive as qn  # noqa: E402  (the reference)
import qwen3_grpo_train as qg  # noqa: E402  (the reference)

torch.set_default_device("cpu")
torch.set_default_dtype(torch.float32)

from oracle import ref_model  # noqa: E402  (only for init_params: same seeded weights as the tests)

BF = torch.bfloat16

# ---------------------------------------------------------------- shims
_orig_tensor = torch.tensor


def _tensor_no_pin(*a, **k):
    k.pop("pin_memory", None)
    return _orig_tensor(*a, **k)


def _rope_gpu_semantics(x, positions, cos_sin_cache, out_dtype):
    out32 = qn.apply_rope_kernel.__wrapped__(x, positions, cos_sin_cache, torch.float32)
    return out32.to(out_dtype)


def _mlp_compiled_numerics(self, x):
    """Qwen3MLP.forward (qwen3_naive.py:695-701) is @torch.compile'd in the reference; Inductor
    evaluates silu(gate) * up in fp32 and rounds once.  With dynamo disabled the eager path
    would round silu(gate) to bf16 first, so the generator reproduces the compiled numerics."""
    gate_up = self.gate_up_proj(x)
    gate, up = gate_up.chunk(2, dim=-1)
    hidden = (torch.nn.functional.silu(gate.float()) * up.float()).to(gate_up.dtype)
    return self.down_proj(hidden)


def install_shims():
    torch.tensor = _tensor_no_pin
    torch.Tensor.cuda = lambda self, *a, **k: self
    if not hasattr(qn.apply_rope_kernel, "__wrapped__"):
        orig = qn.apply_rope_kernel
        _rope_gpu_semantics.__wrapped__ = orig
        qn.apply_rope_kernel = _rope_gpu_semantics
    qn.Qwen3MLP.forward = _mlp_compiled_numerics


def remove_shims():
    torch.tensor = _orig_tensor


# ---------------------------------------------------------------- 1. kernels of the reference
def golden_kernels():
    g = torch.Generator().manual_seed(100)
    x = torch.randn(9, 4, 128, generator=g).to(BF)
    pos = torch.tensor([0, 1, 2, 7, 100, 255, 256, 1000, 4095])
    rope = qn.RotaryEmbedding(128, 4096, 1e6)
    rope32 = qn.apply_rope_kernel(x, pos, rope.cos_sin_cache, torch.float32)
    k = torch.randn(6, 8, 128, generator=g).to(BF)
    v = torch.randn(6, 8, 128, generator=g).to(BF)
    kc = torch.zeros(5, 8, 128, dtype=BF)
    vc = torch.zeros(5, 8, 128, dtype=BF)
    slots = torch.tensor([3, -1, 0, 4, -1, 1], dtype=torch.int32)
    qn.store_kvcache(k, v, kc, vc, slots)
    return {"rope_x": x, "rope_pos": pos, "rope_out_fp32": rope32,
            "rope_cache_row_4095": rope.cos_sin_cache[4095].clone(),
            "store_k": k, "store_v": v, "store_slots": slots, "store_kc": kc, "store_vc": vc}


# ---------------------------------------------------------------- 2. BlockManager / Sequence
def bm_state(bm, seqs):
    return {"free": list(bm.free), "ref_count": list(bm.ref_count), "block_hash": [str(h) for h in bm.block_hash],
            "hash_to_block": sorted([str(h), b] for h, b in bm.hash_to_block.items()),
            "tables": [list(s.block_table) for s in seqs], "kv_len": [s.kv_len for s in seqs]}


def golden_block_manager():
    rng = random.Random(7)
    hashes = []
    for n in [0, 1, 5, 256, 300]:
        toks = [rng.randrange(0, 151936) for _ in range(n)]
        h1 = qn.BlockManager.compute_hash(toks)
        h2 = qn.BlockManager.compute_hash(toks, h1)
        hashes.append({"tokens": toks, "h": str(h1), "h_chain": str(h2)})
    # scripted scenario over 12 pages: shared prefixes, prefix hits from the free list,
    # appends across page boundaries, exhaustion
    base = [rng.randrange(0, 151936) for _ in range(700)]
    prompts = {
        "A": base[:600],
        "B": base[:512] + [rng.randrange(0, 151936) for _ in range(40)],
        "C": [rng.randrange(0, 151936) for _ in range(300)],
        "D": base[:600],
        "E": base[:256],
    }
    bm = qn.BlockManager(12, 256)
    seqs = {k: qn.Sequence(v) for k, v in prompts.items()}
    order = list(seqs)
    trace = []

    def snap(op):
        trace.append({"op": op, **bm_state(bm, [seqs[k] for k in order])})

    def prefill(name):
        s = seqs[name]
        s.num_scheduled_tokens = s.num_prompt_tokens - s.kv_len
        s.kv_len += s.num_scheduled_tokens
        bm.hash_blocks(s)
        s.num_scheduled_tokens = 0

    for op in ["alloc A", "prefill A", "alloc B", "prefill B", "alloc C", "prefill C", "dealloc A", "alloc D",
               "prefill D", "append D x300", "can_append C", "dealloc B", "alloc E", "prefill E", "append C x600"]:
        parts = op.split()
        s = seqs[parts[1]]
        if parts[0] == "alloc":
            bm.allocate(s)
        elif parts[0] == "prefill":
            prefill(parts[1])
        elif parts[0] == "dealloc":
            bm.deallocate(s.block_table)
            s.block_table = []
            s.kv_len = 0
        elif parts[0] == "can_append":
            trace.append({"op": op, "result": bm.can_append(s)})
            continue
        elif parts[0] == "append":
            n = int(parts[2][1:])
            for i in range(n):
                if not bm.can_append(s):
                    trace.append({"op": f"{op} stopped at {i}", "result": False})
                    break
                bm.may_append(s)
                s.append_token(1000 + i)
                s.num_scheduled_tokens = 1
                s.kv_len += 1
                bm.hash_blocks(s)
                s.num_scheduled_tokens = 0
        snap(op)
    return {"hashes": hashes, "prompts": prompts, "order": order, "trace": trace}


# ---------------------------------------------------------------- 3. metadata builders
class _Meta:
    BLOCK_SIZE = 256
    _build_block_tables = qn.Qwen3ForCausalLM._build_block_tables


def golden_prepare():
    rng = random.Random(11)
    out = []
    m = _Meta()
    for case in range(4):
        bm = qn.BlockManager(64, 256)
        seqs = []
        for j in range(3 + case):
            L = rng.choice([1, 5, 255, 256, 257, 700])
            s = qn.Sequence([rng.randrange(0, 151936) for _ in range(L)])
            bm.allocate(s)
            # some sequences already decoding, some mid-prefill
            if j % 3 == 0:
                s.kv_len = s.num_prompt_tokens
                s.append_token(rng.randrange(0, 151936))
                if s.kv_len % 256 == 0:
                    bm.may_append(s)
                s.num_scheduled_tokens = 1
            elif j % 3 == 1 and s.num_prompt_tokens > 10:
                s.kv_len = 7
                s.num_scheduled_tokens = min(100, s.num_prompt_tokens - 7)
            else:
                s.num_scheduled_tokens = s.num_prompt_tokens - s.kv_len
            seqs.append(s)
        ids, pos, cu_q, cu_k, mq, mk, blk, bt = qn.Qwen3ForCausalLM._prepare_step(m, seqs)
        entry = {"seqs": [{"token_ids": s.token_ids, "kv_len": s.kv_len, "n": s.num_scheduled_tokens,
                           "block_table": s.block_table, "prompt_len": s.num_prompt_tokens} for s in seqs],
                 "step": {"input_ids": ids.tolist(), "positions": pos.tolist(), "cu_q": cu_q.tolist(),
                          "cu_k": cu_k.tolist(), "max_q": mq, "max_k": mk, "block_mapping": blk.tolist(),
                          "block_tables": bt.tolist()}}
        dec = [s for s in seqs if s.num_scheduled_tokens == 1 and s.kv_len >= s.num_prompt_tokens]
        if dec:
            d = qn.Qwen3ForCausalLM._prepare_decode(m, dec)
            entry["decode_idx"] = [seqs.index(s) for s in dec]
            entry["decode"] = {k: t.tolist() for k, t in zip(
                ["input_ids", "positions", "context_lens", "block_tables", "slot_mapping"], d)}
        out.append(entry)
    return out


# ---------------------------------------------------------------- 4. scheduler trace
def fake_next_token(input_id, position, vocab):
    return (input_id * 7 + position * 13 + 1) % vocab


def golden_scheduler(num_blocks, prompt_lens, max_new, eos, seed):
    """Runs the reference's generate_continuous_with_logprobs with the device work replaced."""
    V = 4096
    cfg = qn.Qwen3Config(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                         intermediate_size=256, num_hidden_layers=1, vocab_size=V, max_position_embeddings=8192)
    model = qn.Qwen3ForCausalLM(cfg)
    model._num_blocks = num_blocks
    model.allocate_global_kv_cache = lambda: None
    model._init_cuda_graphs = lambda: None
    model._capture_decode_graphs = lambda: setattr(model, "_has_cuda_graphs", False)
    model._has_cuda_graphs = False
    steps = []
    orig_step, orig_dec = qn.Qwen3ForCausalLM._prepare_step, qn.Qwen3ForCausalLM._prepare_decode

    def prep_step(self, seqs):
        r = orig_step(self, seqs)
        steps.append({"kind": "step", "n": [s.num_scheduled_tokens for s in seqs],
                      "input_ids": r[0].tolist(), "positions": r[1].tolist(), "cu_q": r[2].tolist(),
                      "cu_k": r[3].tolist(), "block_mapping": r[6].tolist(), "block_tables": r[7].tolist()})
        return r

    def prep_dec(self, seqs):
        r = orig_dec(self, seqs)
        steps.append({"kind": "decode", "input_ids": r[0].tolist(), "positions": r[1].tolist(),
                      "context_lens": r[2].tolist(), "block_tables": r[3].tolist(),
                      "slot_mapping": r[4].tolist()})
        return r

    model._prepare_step = prep_step.__get__(model)
    model._prepare_decode = prep_dec.__get__(model)

    def fake_forward(input_ids, positions, *rest):
        nxt = [fake_next_token(i, p, V) for i, p in zip(input_ids.tolist(), positions.tolist())]
        return torch.tensor(nxt, dtype=torch.float32)[:, None]

    model.model.forward_prefill = fake_forward
    model.model.forward_decode = fake_forward

    class FakeHead(torch.nn.Module):
        def forward(self, h):
            logits = torch.full((h.shape[0], V), -30.0)
            logits[torch.arange(h.shape[0]), h[:, 0].long()] = 30.0
            return logits

    model.lm_head = FakeHead()
    rng = random.Random(seed)
    prompts = [[rng.randrange(0, V) for _ in range(L)] for L in prompt_lens]
    torch.manual_seed(seed)
    n_dealloc = [0]
    orig_dealloc = qn.BlockManager.deallocate

    def counting_dealloc(self, table):
        n_dealloc[0] += 1
        return orig_dealloc(self, table)

    qn.BlockManager.deallocate = counting_dealloc
    try:
        toks, gen, lps, plens = model.generate_continuous_with_logprobs(
            [torch.tensor([p]) for p in prompts], max_new_tokens=max_new, temperature=1.0, top_k=1,
            eos_token_ids=eos)
    finally:
        qn.BlockManager.deallocate = orig_dealloc
    # every sequence is released once when it finishes; any extra release is a preemption
    return {"num_blocks": num_blocks, "prompts": prompts, "max_new": max_new, "eos": eos, "vocab": V,
            "steps": steps, "seq_tokens": toks, "generated": gen, "prompt_lens": plens,
            "n_logprobs": [len(x) for x in lps], "preemptions": n_dealloc[0] - len(prompts)}


# ---------------------------------------------------------------- 5. GRPO math
def golden_grpo():
    g = torch.Generator().manual_seed(123)
    G, groups, S = 4, 5, 64
    N = G * groups
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    rewards[:G] = 1.0
    pid = torch.arange(groups).repeat_interleave(G)
    perm = torch.randperm(N, generator=g)
    rewards, pid = rewards[perm], pid[perm]  # groups interleaved
    new = -torch.rand(N, S, generator=g) * 6
    old = new + 0.05 * torch.randn(N, S, generator=g)
    mask = torch.zeros(N, S)
    for i in range(N):
        L = int(torch.randint(1, S + 1, (1,), generator=g))
        mask[i, S - L:] = 1.0
    adv = qg.compute_grpo_advantage(rewards, pid)
    tok = adv.unsqueeze(-1) * mask
    newp = new.clone().requires_grad_(True)
    loss = qg.ppo_clipped_loss(old, newp, tok, mask)
    loss.backward()
    return {"rewards": rewards, "prompt_ids": pid, "new": new, "old": old, "mask": mask, "adv": adv,
            "loss": loss.detach(), "grad_new": newp.grad}


# ---------------------------------------------------------------- 6. tiny model
TINY = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, head_dim=128, intermediate_size=256,
            num_hidden_layers=2, vocab_size=512, max_position_embeddings=1024)


def golden_model():
    cfg = qn.Qwen3Config(**TINY)
    torch.set_default_dtype(BF)
    model = qn.Qwen3ForCausalLM(cfg)
    torch.set_default_dtype(torch.float32)
    params = ref_model.init_params(cfg, seed=0)
    sd = model.state_dict()
    for k in sd:
        if k in params:  # the rest are the shared RoPE table buffers
            sd[k].copy_(params[k])
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (2, 40), generator=g)
    with torch.no_grad():
        logits = model(ids)
    lp = qg.forward_logprob(model, ids)
    # GRPO loss through the reference's own training math; RoPE blocks q/k grads as in the reference
    old = lp.detach() + 0.05 * torch.randn(lp.shape, generator=g)
    mask = torch.zeros(2, 40)
    mask[0, 20:] = 1
    mask[1, 10:35] = 1
    tok_adv = torch.tensor([0.7, -1.3])[:, None] * mask
    loss = qg.ppo_clipped_loss(old, lp, tok_adv, mask)
    model.zero_grad()
    loss.backward()
    grads = {k: (p.grad.clone() if p.grad is not None else None) for k, p in model.named_parameters()}
    return {"config": TINY, "ids": ids, "logits": logits, "logprob": lp.detach(), "old": old, "mask": mask,
            "tok_adv": tok_adv, "loss": loss.detach(), "grads": grads}


def main():
    install_shims()
    try:
        out = {}
        torch.save(golden_kernels(), HERE / "kernels.pt")
        with open(HERE / "block_manager.json", "w") as f:
            json.dump(golden_block_manager(), f)
        with open(HERE / "prepare.json", "w") as f:
            json.dump(golden_prepare(), f)
        sched = [golden_scheduler(40, [5, 300, 700, 256, 1, 512, 90], 40, None, 1),
                 golden_scheduler(9, [600, 600, 300, 200, 100], 300, None, 2),       # preemption
                 golden_scheduler(60, [2100, 30, 30, 1500, 999], 20, list(range(3, 4096, 9)), 3)]  # chunked + EOS
        with open(HERE / "scheduler.json", "w") as f:
            json.dump(sched, f)
        torch.save(golden_grpo(), HERE / "grpo.pt")
        torch.save(golden_model(), HERE / "model_tiny.pt")
    finally:
        remove_shims()
    for p in sorted(HERE.iterdir()):
        if p.suffix in (".pt", ".json"):
            print(f"{p.name}: {p.stat().st_size / 1024:.1f} KiB")


if __name__ == "__main__":
    main()
