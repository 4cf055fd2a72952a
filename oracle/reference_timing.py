"""Times config 1 (the GRPO loss / advantage path) through the reference's own functions on the
host cores -- test infrastructure, run where the reference source is present:

    python oracle/reference_timing.py <reference checkout holding qwen3_grpo_train.py>

Config 1: 2 prompts x G=4 completions x 128 tokens = 1024 rows of bf16 logits [1024, 151936]
~N(0,1); targets U[0, 151643); rewards Bernoulli(0.5); old/ref log-probs = current + N(0, 0.05);
clip 0.2; random tail masks.  Each pass runs the reference's forward_logprob
(qwen3_grpo_train.py:46-53; its model is a stand-in returning the config's logits, which gathers
the target ids exactly as the reference gathers input_ids), compute_grpo_advantage (:162-173),
the token advantage of grpo_train_step (:266-269) and ppo_clipped_loss (:184-199), plus the k3
KL term the north star adds (beta 0.04; the reference has none), then the backward to the logits.
Prints one JSON line with the mean time per pass and the thread count.  The GPU box has no copy
of the reference, so bench.py times the oracle's restatement of the same pass there.
"""
from __future__ import annotations

import json
import os
import sys
import time
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")


def main():
    if len(sys.argv) != 2 or not (Path(sys.argv[1]) / "qwen3_grpo_train.py").is_file():
        sys.exit("usage: python oracle/reference_timing.py <reference checkout holding qwen3_grpo_train.py>")
    sys.path.insert(0, sys.argv[1])
    import torch
    torch.set_num_threads(os.cpu_count())
    import qwen3_grpo_train as ref  # the reference, unmodified
    # importing it runs qwen3_naive.py:1786-1787 (default device cuda, default dtype bf16); the
    # timing runs on the host cores in the reference's fp32 loss arithmetic
    torch.set_default_device("cpu")
    torch.set_default_dtype(torch.float32)

    N, S, V = 8, 128, 151936
    g = torch.Generator().manual_seed(1)
    logits0 = torch.randn(N, S, V, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 151643, (N, S), generator=g)
    lens = torch.randint(1, S + 1, (N,), generator=g)
    mask = (torch.arange(S)[None, :] < lens[:, None]).float()
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    prompt_ids = torch.arange(N) // 4
    with torch.no_grad():
        base = ref.forward_logprob(lambda x: logits0, ids)
    old = base + 0.05 * torch.randn(N, S, generator=g)
    ref_lp = base + 0.05 * torch.randn(N, S, generator=g)
    times = []
    for i in range(4):
        t0 = time.perf_counter()
        logits = logits0.clone().requires_grad_(True)
        new = ref.forward_logprob(lambda x: logits, ids)
        adv = ref.compute_grpo_advantage(rewards, prompt_ids)
        loss = ref.ppo_clipped_loss(old, new, adv.unsqueeze(-1) * mask, mask)
        d = ref_lp - new
        loss = loss + 0.04 * ((d.exp() - d - 1) * mask).sum() / (mask.sum() + 1e-8)
        loss.backward()
        if i:
            times.append(time.perf_counter() - t0)
    ms = 1000 * sum(times) / len(times)
    print(json.dumps({"config": 1, "impl": "reference (imported)", "ms_per_pass": ms, "tokens_per_s": N * S / (ms / 1e3),
                      "threads": torch.get_num_threads(), "cpu_count": os.cpu_count()}))


if __name__ == "__main__":
    main()
