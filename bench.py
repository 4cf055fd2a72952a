"""Benchmark of the GRPO step (the north-star path) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload per GPU ("grpo_step_cfg4"): Qwen3-0.6B-shaped random-init bf16 model (hidden
1024, 28 layers, 16 q / 8 kv heads, head_dim 128, SwiGLU 3072, vocab 151936 tied,
rope theta 1e6, weights N(0, 0.02)); 64 prompts x G=8 completions, prompt length
U[64, 512], ids U[0, 151643); 512 new tokens (no EOS), temperature 1.0, no top-k,
paged KV pages of 256; then log-prob recompute of the policy and a frozen reference
copy, group advantages, clipped surrogate + 0.04 * k3 KL, backward, AdamW lr 1e-6.
Rewards are Bernoulli(0.5).  Under torchrun each rank runs its own 64 prompt groups
(weak scaling), sums the response-token count and the fp32 gradients with NCCL, and
steps AdamW on the global loss.  Inputs are synthetic (no dataset exists for this path).

metric: GRPO step tokens/s = (prompt + completion tokens of all ranks) / step time.

Kernel microbenchmarks (one GPU, each prints its own JSON line): --rollout-attn (decode attention
mid-rollout, plain vs grouped layout), --decode-only (plain paged decode, config 3), --gemm-only
(projection shapes, tcgen05 vs cuBLAS, graph-timed), --attn-only (training attention fwd/bwd),
--loss-only (config 1: log-prob, GRPO loss and logit gradient, with the config-1 CPU baseline),
--rollout-only (config 2: the grouped rollout alone, with its roofline and a CPU baseline);
--kernel-profile PATH writes the per-kernel time of one step, split by phase.  The main line also
carries the whole-step roofline fraction and the dominant kernel's in-step bandwidth, measured on
one extra untimed step under CUPTI (--no-inner-profile skips it).
"""
from __future__ import annotations

import argparse
import contextlib
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GRPO step tokens/s"
UNIT = "tokens/s"
WORKLOAD = "grpo_step_cfg4: 64 prompts x G=8 per GPU, prompt U[64,512], 512 new tokens, Qwen3-0.6B shape"
WORKLOAD5 = ("grpo_step_cfg5: 512 prompts x G=8 in total, groups sharded round-robin over the ranks, prompt "
             "U[64,1024], 512 new tokens, Qwen3-0.6B shape")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompts", type=int, default=64, help="prompt groups per GPU")
    ap.add_argument("--workload", default="cfg4", choices=["cfg4", "cfg5"],
                    help="cfg4: 64 groups per GPU, prompt U[64,512] (weak scaling, the default); cfg5: 512 groups "
                         "in total sharded over the ranks, prompt U[64,1024] (strong scaling)")
    ap.add_argument("--group", type=int, default=8)
    ap.add_argument("--new-tokens", type=int, default=512)
    ap.add_argument("--prompt-min", type=int, default=64)
    ap.add_argument("--prompt-max", type=int, default=512)
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--microbatch-tokens", type=int, default=32768)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--decode-only", action="store_true",
                    help="only the config-3 paged-decode microbenchmark (for kernel profiling)")
    ap.add_argument("--decode-batch", type=int, default=256, help="batch of the decode microbenchmark")
    ap.add_argument("--gemm-only", action="store_true",
                    help="only the tcgen05 GEMM microbenchmark on the model's projection shapes")
    ap.add_argument("--gemm-shape", default=None, help="M,N,K: run --gemm-only on this one shape")
    ap.add_argument("--rollout-attn", action="store_true",
                    help="only plain vs grouped decode attention on a mid-rollout batch")
    ap.add_argument("--no-graphs", action="store_true",
                    help="eager decode launches (for launch-list profiling; ncu and graph replays do not mix)")
    ap.add_argument("--attn-only", action="store_true",
                    help="training attention forward + backward on one microbatch of the bench's sequences")
    ap.add_argument("--gemm-qk", action="store_true",
                    help="qkv GEMM with the QK-norm + RoPE epilogue against GEMM + standalone kernel (decode "
                         "step and training sizes)")
    ap.add_argument("--elementwise", action="store_true",
                    help="the row kernels (QK-norm/RoPE fwd+bwd, SwiGLU fwd+bwd, RMSNorm bwd) on a training "
                         "microbatch")
    ap.add_argument("--loss-only", action="store_true",
                    help="config 1: fused log-prob -> GRPO loss -> logit gradient over 1024 rows of logits")
    ap.add_argument("--kernel-profile", default=None, metavar="PATH",
                    help="after the timed steps, run one more step under torch.profiler (CUPTI kernel records) and "
                         "write per-kernel launches / device time / share to PATH")
    ap.add_argument("--rollout-only", action="store_true",
                    help="config 2: the grouped rollout alone (generated tokens/s, rollout roofline, CPU baseline)")
    ap.add_argument("--no-inner-profile", action="store_true",
                    help="skip the extra untimed step under CUPTI that measures the dominant kernel inside the step")
    ap.add_argument("--no-share-prefix", action="store_true",
                    help="roll out with the reference's scheduler (every completion prefilled and stored)")
    ap.add_argument("--no-pdl", action="store_true",
                    help="launch every kernel with plain stream ordering (no programmatic dependent launch)")
    return ap.parse_args()


# ------------------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        import tempfile
        try:
            fd, name = tempfile.mkstemp(prefix=f"clocks_gpu{self.index}_", suffix=".csv")
            self.path = Path(name)
            self.f = os.fdopen(fd, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        text = self.path.read_text()
        self.path.unlink()
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        mx = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------------------ workload
def make_prompts(args, rank, step, device=None):
    """This rank's prompt groups of one step.  cfg4: args.prompts groups per rank drawn per rank;
    cfg5: one global list of args.total_prompts groups per step, rank r taking groups r, r+N, ..."""
    import torch
    if args.workload == "cfg5":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        g = torch.Generator().manual_seed(1 + step)
        lens = torch.randint(args.prompt_min, args.prompt_max + 1, (args.total_prompts,), generator=g)
        prompts = [torch.randint(0, 151643, (1, int(L)), generator=g) for L in lens][rank::world]
    else:
        g = torch.Generator().manual_seed(1 + 1000 * rank + step)
        lens = torch.randint(args.prompt_min, args.prompt_max + 1, (args.prompts,), generator=g)
        prompts = [torch.randint(0, 151643, (1, int(L)), generator=g) for L in lens]
    if device is not None:
        prompts = [p.to(device) for p in prompts]
    return prompts


def decode_microbench(torch, ops, device, n_iter=20, batch=256):
    """Config 3: paged decode attention, batch 256, context U[1k, 8k], 16q/8kv, head_dim 128,
    bf16 K/V ~ N(0,1) in 256-token pages randomly permuted in a pool 1.25x the need.
    Returns (kernel ms per launch, algorithmic bytes per launch)."""
    g = torch.Generator().manual_seed(3)
    B, hq, hkv, D = batch, 16, 8, 128
    ctx = torch.randint(1024, 8193, (B,), generator=g)
    pages = [(int(c) + 255) // 256 for c in ctx]
    pool = int(sum(pages) * 1.25)
    perm = torch.randperm(pool, generator=g)
    width = max(pages)
    bt = torch.full((B, width), -1, dtype=torch.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    kc = torch.randn(pool, 256, hkv, D, device=device, dtype=torch.bfloat16)
    vc = torch.randn(pool, 256, hkv, D, device=device, dtype=torch.bfloat16)
    q = torch.randn(B, hq, D, device=device, dtype=torch.bfloat16)
    btd = bt.to(device)
    cl = (ctx - 1).to(torch.int32).to(device)  # context_lens; the kernel attends context + 1 keys
    split_tokens, max_splits = ops.decode_split_plan(B, hkv, int(ctx.max()))
    ws_bytes = ops.lib().qb_paged_decode_workspace_bytes(B, hq, D, max_splits)
    ws = torch.empty(max(ws_bytes // 4, 1), device=device, dtype=torch.float32)
    run = lambda: ops.paged_decode_attention(q, kc, vc, btd, cl, D ** -0.5, split_tokens=split_tokens,
                                             max_splits=max_splits, workspace=ws)
    for _ in range(3):
        run()
    # K/V (GBs) are far larger than the 126 MB L2, so launches run back to back between two
    # events on the launching stream: no launch gaps in the average, no L2 reuse either.
    st = torch.cuda.current_stream()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(n_iter):
        run()
    b.record(st)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n_iter
    nbytes = int(ctx.sum()) * hkv * D * 2 * 2 + B * hq * D * 2 * 2 + B * width * 4 + B * 4
    ops.check_device_errors()
    del kc, vc
    return ms, nbytes, int(ctx.sum())


def profiled_traffic(profile, key, scale=1):
    """DRAM bytes (read + write) of one launch from a committed ncu summary under profiles/: the
    figure after ``key:`` times ``scale`` (per-token figures are scaled to the launch); None if
    the summary is absent."""
    import re
    f = ROOT / "profiles" / profile
    if not f.exists():
        return None
    m = re.search(key + r":\s*([0-9.]+)", f.read_text())
    return float(m.group(1)) * scale if m else None


def cpu_baseline_sample(steps=1, threads=None):
    """The oracle (CPU restatement of the reference) on a bounded sample of the GRPO step:
    1 prompt x G=2 completions at the full Qwen3-0.6B shape, prompt 48 tokens, 4 new
    tokens sampled by full recompute (the reference rollout's scheme), then reference-policy
    and policy log-probs, the loss and its backward.  Returns (tokens/s, sample text, threads)."""
    import torch
    from oracle import ref_model
    from oracle import ref_ops as R
    from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config
    if threads:
        torch.set_num_threads(threads)
    cfg = Qwen3Config()
    params = ref_model.init_params(cfg, seed=0)
    g = torch.Generator().manual_seed(11)
    P, G, new = 48, 2, 4
    cs = R.rope_cache(cfg.head_dim, P + new + 1, cfg.rope_theta)
    tok_total, t_total = 0, 0.0
    for _ in range(steps):
        prompt = torch.randint(0, 151643, (1, P), generator=g)
        t0 = time.perf_counter()
        ids = prompt.repeat(G, 1)
        old = []
        with torch.no_grad():
            for _t in range(new):
                lg = ref_model.logits(params, cfg, ids, cos_sin=cs)[:, -1].float()
                probs, logp = R.sample_distribution(lg, 1.0, None)
                nxt = torch.multinomial(probs, 1, generator=g)
                old.append(logp.gather(-1, nxt))
                ids = torch.cat([ids, nxt], 1)
            ref_lp = ref_model.forward_logprob(params, cfg, ids, shift=True, cos_sin=cs)
        p = {k: v.clone().requires_grad_(True) for k, v in params.items()}
        lp = ref_model.forward_logprob(p, cfg, ids, shift=True, cos_sin=cs)
        mask = torch.zeros_like(lp)
        mask[:, P:] = 1
        oldp = torch.zeros_like(lp)
        oldp[:, P:] = torch.cat(old, 1)
        rewards = torch.bernoulli(torch.full((G,), 0.5), generator=g)
        adv = R.grpo_advantage(rewards, torch.zeros(G, dtype=torch.long))
        loss = R.ppo_loss(oldp, lp, adv[:, None] * mask, mask, 0.2, ref_lp, 0.04)
        loss.backward()
        t_total += time.perf_counter() - t0
        tok_total += G * (P + new)
    sample = (f"oracle GRPO step on 1 prompt x G={G}, prompt {P} + {new} new tokens, Qwen3-0.6B shape "
              f"(rollout by full recompute, ref + policy log-probs, clipped+KL loss, backward)")
    return tok_total / t_total, sample, torch.get_num_threads()


# ------------------------------------------------------------------------------ whole-step roofline
H, I, HQ, HKV, D, VOCAB = 1024, 3072, 16, 8, 128, 151936
LAYER_PARAMS = (HQ + 2 * HKV) * D * H + H * HQ * D + 2 * I * H + H * I  # qkv, o, gate_up, down
LM_HEAD_PARAMS = VOCAB * H
KV_BYTES_PER_KEY_LAYER = 2 * HKV * D * 2                               # K and V, bf16


def step_roofline(prompt_lens, group, new, layers, step_s, peaks):
    """Roofline time of one GRPO step of this rank's workload, phase by phase: each phase costs
    max(FLOP / tensor peak, bytes / HBM peak) at the sustained measured peaks, summed; the
    fraction is that sum over the measured step time.  FLOPs are 2 per weight per token for
    every projection (lm_head only where a token is scored or sampled) plus the causal attention
    products; rollout bytes are the weights and the K/V each decode step must read (each group's
    prompt once, every completion's own tokens)."""
    tf = peaks.get("bf16_tflops_sustained", 1404.4) * 1e12
    bw = peaks.get("hbm_gbs", 6539.5) * 1e9
    lin = 2 * LAYER_PARAMS * layers
    attn = lambda q_pairs: 4 * HQ * D * layers * q_pairs  # QK^T and PV over (query, key) pairs
    # rollout: prefill of each prompt once (grouped), then `new` decode steps of every completion
    pre_flop = sum(lin * L + attn(L * (L + 1) / 2) + 2 * LM_HEAD_PARAMS for L in prompt_lens)
    t_roll = pre_flop / tf
    weights = 2 * (LAYER_PARAMS * layers + LM_HEAD_PARAMS)
    B = len(prompt_lens) * group
    for s in range(new - 1):
        keys_read = sum(prompt_lens) + B * (s + 1)  # shared prompts once + each completion's own keys
        ctx_total = sum(L + s + 1 for L in prompt_lens) * group
        flop = B * (lin + 2 * LM_HEAD_PARAMS) + attn(ctx_total)
        byts = weights + keys_read * KV_BYTES_PER_KEY_LAYER * layers
        t_roll += max(flop / tf, byts / bw)
    # log-prob recompute (frozen reference) and the policy's forward + backward, packed sequences
    seqs = [L + new for L in prompt_lens for _ in range(group)]
    tokens = sum(seqs)
    scored = B * new
    fwd = lin * tokens + 2 * LM_HEAD_PARAMS * scored + attn(sum(L * (L + 1) / 2 for L in seqs))
    attn_fwd = attn(sum(L * (L + 1) / 2 for L in seqs))
    t_ref = fwd / tf
    t_train = (3 * (fwd - attn_fwd) + 3.5 * attn_fwd) / tf  # backward: 2x the projections, 2.5x attention
    total = t_roll + t_ref + t_train
    return {"rollout_s": t_roll, "ref_logprob_s": t_ref, "train_s": t_train, "total_s": total,
            "measured_s": step_s, "frac": total / step_s,
            "peaks": {"bf16_tflops_sustained": tf / 1e12, "hbm_gbs": bw / 1e9},
            "basis": "sum over phases of max(FLOP/peak, bytes/peak); decode steps HBM-bound, the rest tensor-bound"}


def progress(msg):
    """Phase marker on stderr (the JSON line alone goes to stdout)."""
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


@contextlib.contextmanager
def plain_launches():
    """Steps run under torch.profiler (CUPTI activity records) launch every kernel with plain
    stream order: CUPTI tracing and programmatic dependent launches are kept apart.  The decode
    graphs record the launch mode, so they are recaptured for the profiled step."""
    from qwen3_naive_inference_b200._lib import load
    lib = load()
    old = lib.qb_get_pdl()
    lib.qb_set_pdl(0)
    try:
        yield
    finally:
        lib.qb_set_pdl(old)


def in_step_kernel_profile(torch, run_step):
    """Device time per kernel name over one GRPO step (CUPTI records via torch.profiler, graph
    replays included).  Returns ({name: (launches, total_us)}, step outputs)."""
    from collections import defaultdict

    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with plain_launches(), profile(activities=[ProfilerActivity.CUDA]) as prof:
        out = run_step()
        torch.cuda.synchronize()
    agg = defaultdict(lambda: [0, 0.0])
    for e in prof.events():
        if str(getattr(e, "device_type", "")).endswith("CUDA"):
            name = e.name
            for pre in ("void ", "(anonymous namespace)::", "<unnamed>::"):
                name = name.replace(pre, "")
            name = name.split("(")[0].split("<")[0]
            agg[name][0] += 1
            agg[name][1] += e.time_range.elapsed_us()
    return dict(agg), out


def grouped_decode_alg_bytes(prompt_lens, group, new, layers):
    """Algorithmic bytes of every grouped decode attention call of one rollout: per layer and
    decode step, each group's prompt K/V once and each completion's own keys, plus q, out and
    the page tables (as in rollout_attn_case)."""
    B = len(prompt_lens) * group
    total = 0
    for s in range(new - 1):
        keys = sum(prompt_lens) + B * (s + 1)
        total += keys * KV_BYTES_PER_KEY_LAYER + 2 * B * HQ * D * 2 + B * 4 * (4 + 2)
    return total * layers


# ------------------------------------------------------------------------------ arms
def run_reference(args):
    """CPU baseline arm: the oracle port of the reference's GRPO step on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    threads = os.cpu_count()
    torch.set_num_threads(threads)
    for _ in range(args.warmup):
        cpu_baseline_sample(1)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, sample, th = cpu_baseline_sample(1)
        vals.append(v)
    elapsed = time.perf_counter() - t0
    value = sum(vals) / len(vals)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "sample": sample, "cores": threads},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": th, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from qwen3_naive_inference_b200 import _lib, ops
    from qwen3_naive_inference_b200 import qwen3_grpo_train as G
    from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config, build_model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    cfg = Qwen3Config(num_hidden_layers=args.layers)
    policy = build_model(cfg, device=dev, seed=0)
    ref = G.make_reference_copy(policy)
    max_ctx = args.prompt_max + args.new_tokens
    # pages for every sequence of the step at once (64*8 seqs x 4 pages) plus slack; a larger
    # share (cfg5 on few GPUs) gets what fits in memory and the scheduler admits groups in waves
    need = len(make_prompts(args, rank, 0)) * args.group * math.ceil(max_ctx / 256) + 64
    free, _ = torch.cuda.mem_get_info(dev)
    # keep room for the training pass, which runs with the pool still allocated: ~48 KB of saved
    # activations per token and layer for a microbatch, plus 16 GB for the optimizer state, the
    # gradient buffer, the logits chunk and the backward's transient buffers
    reserve = (16 << 30) + args.microbatch_tokens * args.layers * (48 << 10)
    fit = int((free - reserve) // policy._block_bytes())
    policy._num_blocks = max(64, min(need, fit))
    policy.max_model_len = max_ctx
    policy.use_cuda_graphs = not args.no_graphs
    opt = torch.optim.AdamW(policy.parameters(), lr=1e-6)
    reward_gen = torch.Generator().manual_seed(2 + rank)
    torch.manual_seed(1234 + rank)

    def step(i, prompts):
        return G.grpo_step(policy, opt, prompts, ref_model=ref, group_size=args.group,
                           max_new_tokens=args.new_tokens, temperature=1.0, top_k=None, eos_token_ids=None,
                           reward_gen=reward_gen, beta=0.04, shift=True,
                           microbatch_tokens=args.microbatch_tokens, share_prefix=not args.no_share_prefix)

    for i in range(args.warmup):
        step(i, make_prompts(args, rank, i, dev))

    def timed(n, host_inputs):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        tokens = 0
        h2d = d2h = 0
        launches0 = _lib.LAUNCHES[0]
        host = [make_prompts(args, rank, 100 + j) for j in range(n)]
        if host_inputs:
            host = [[p.pin_memory() for p in ps] for ps in host]
        else:
            host = [[p.to(dev) for p in ps] for ps in host]
            torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")  # ncu --nvtx --nvtx-include "timed/" selects this region
        a.record(st)
        wall0 = time.perf_counter()
        for j in range(n):
            prompts = host[j]
            if host_inputs:  # the step's inputs cross PCIe inside the timed region
                prompts = [p.to(dev, non_blocking=True) for p in prompts]
                h2d += sum(p.numel() * p.element_size() for p in host[j])
            out = step(j, prompts)
            tokens += out["tokens"]
            d2h += 3 * 4 + out["completion_tokens"] * 12  # loss[3] + sampled tokens/log-probs read back
        b.record(st)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        wall = time.perf_counter() - wall0
        launches = _lib.LAUNCHES[0] - launches0
        if world > 1:
            t = torch.tensor([ms, float(tokens)], device=dev, dtype=torch.float64)
            mx = t.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            dist.all_reduce(t, op=dist.ReduceOp.SUM)
            ms, tokens = float(mx[0]), int(t[1])
        return ms, tokens, wall, launches, h2d, d2h, out

    sampler = ClockSampler(local)
    sampler.start()
    progress("warm-up done")
    ms, tokens, wall, launches, _, _, last = timed(args.steps, host_inputs=False)
    clocks = sampler.stop()
    progress("timed steps done")
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    # whole-step roofline of the timed steps (this rank's workload; the time is the max over ranks)
    roof_s = 0.0
    for j in range(args.steps):
        lens = [p.shape[1] for p in make_prompts(args, rank, 100 + j)]
        roof_s += step_roofline(lens, args.group, args.new_tokens, args.layers, 1.0, peaks)["total_s"]
    whole_step = step_roofline([p.shape[1] for p in make_prompts(args, rank, 100)], args.group, args.new_tokens,
                               args.layers, ms / 1000.0 / args.steps, peaks)
    whole_step["frac"] = roof_s / (ms / 1000.0)
    whole_step["total_s_all_timed_steps"] = roof_s
    e2e = None
    if not args.no_e2e:
        ems, etok, _, _, h2d, d2h, _ = timed(args.steps, host_inputs=True)
        e2e = {"value": etok / (ems / 1000.0), "unit": UNIT, "h2d_bytes_per_step": h2d // max(1, args.steps),
               "d2h_bytes_per_step": d2h // max(1, args.steps)}
    progress("e2e steps done")
    # the dominant kernel inside the step: one more (untimed) step under CUPTI; every rank runs it
    in_step = None
    if not args.no_inner_profile:
        prof_prompts = make_prompts(args, rank, 300, dev)
        agg, _ = in_step_kernel_profile(torch, lambda: step(0, prof_prompts))
        if rank == 0 and "paged_decode_grouped_kernel" in agg:
            n_g, us_g = agg["paged_decode_grouped_kernel"]
            n_c, us_c = agg.get("paged_decode_combine_kernel", (0, 0.0))
            alg = grouped_decode_alg_bytes([p.shape[1] for p in prof_prompts], args.group, args.new_tokens,
                                           args.layers)
            tot_us = sum(v[1] for v in agg.values())
            in_step = {"calls": n_g, "tile_kernel_us": us_g, "combine_us": us_c,
                       "us_per_call": (us_g + us_c) / max(1, n_g), "algorithmic_bytes": alg,
                       "achieved_gbs": alg / ((us_g + us_c) * 1e-6) / 1e9,
                       "frac": alg / ((us_g + us_c) * 1e-6) / 1e9 / peaks.get("hbm_gbs", 6650.0),
                       "share_of_step_kernel_time": (us_g + us_c) / max(tot_us, 1.0),
                       "source": "CUPTI kernel records of one untimed bench step (all decode steps, all layers)"}
    if args.kernel_profile and rank == 0:
        kernel_profile(args, torch, lambda: step(0, make_prompts(args, rank, 200, dev)), args.kernel_profile)
    progress("profiles done")
    value = tokens / (ms / 1000.0)
    # roofline of the dominant kernel: the grouped (shared-prefix) decode attention, on the
    # mid-rollout case, launches back to back between events on its stream; the timed call is the
    # tile kernel plus its small split-K combine
    hbm = peaks.get("hbm_gbs", 6650.0)
    case = rollout_attn_case(torch, ops, dev)
    grp_ms = time_launches(torch, case["runs"]["grouped"])
    plain_ms = time_launches(torch, case["runs"]["plain"])
    ops.check_device_errors()
    achieved = case["alg_grouped"] / (grp_ms / 1000.0) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": profiled_traffic("paged_decode_grouped_kernel_rollout.md", "traffic_bytes_per_launch"),
                "kernel": "paged_decode_grouped_kernel",
                "case": "mid-rollout: 64 groups x 8, prompt U[64,512] shared per group, 256 own tokens per "
                        "completion, 16q/8kv, d128; back-to-back launches, K/V 4.7x L2",
                "algorithmic_bytes": case["alg_grouped"], "ms_per_launch": grp_ms,
                "traffic_source": "profiles/paged_decode_grouped_kernel_rollout.md (ncu, same case, "
                                  "tile kernel + combine)",
                "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)" if pk.exists() else "fallback",
                "vs_reference_layout": {"kernel": "paged_decode_kernel", "ms_per_launch": plain_ms,
                                        "kv_bytes": case["kv_plain"],
                                        "effective_gbs_of_grouped": case["kv_plain"] / (grp_ms / 1000.0) / 1e9},
                "in_step": in_step}
    del case
    # the plain paged decode kernel alone on config-3 shapes (long contexts)
    dec_ms, dec_bytes, dec_tokens = decode_microbench(torch, ops, dev)
    decode_plain = {"kernel": "paged_decode_kernel", "case": "config 3: batch 256, ctx U[1k,8k]",
                    "ms_per_launch": dec_ms, "achieved_gbs": dec_bytes / (dec_ms / 1000.0) / 1e9,
                    "traffic": profiled_traffic("paged_decode_kernel_config3.md", "traffic_bytes_per_kv_token",
                                                dec_tokens)}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, sample, th = cpu_baseline_sample(1)
        cpu = {"value": v, "unit": UNIT, "cores": th, "kind": "port", "sample": sample}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
                "scaling": "strong" if args.workload == "cfg5" else "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic",
                "config": {"workload": WORKLOAD if args.workload == "cfg4" else WORKLOAD5,
                           "prompts_per_gpu": len(make_prompts(args, rank, 0)), "group": args.group,
                           "kv_pages": policy._num_blocks,
                           "new_tokens": args.new_tokens, "prompt_len": [args.prompt_min, args.prompt_max],
                           "layers": args.layers, "parallelism": f"dp{world}", "beta_kl": 0.04,
                           "rollout": "reference scheduler" if args.no_share_prefix else
                           "grouped: prompt prefilled once per group, shared KV pages, shared-prefix decode attention",
                           "l2": "inputs far larger than L2 (weights + 60+ GB KV cache per step)",
                           "launch": "plain stream order" if args.no_pdl else "programmatic dependent launch",
                           "tokens_per_step": tokens // max(1, args.steps)},
                "phases_s": {"rollout": last["t_rollout"], "ref_logprob": last["t_ref"], "train": last["t_train"],
                             "rollout_detail": last.get("rollout_stats")},
                "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "roofline": roofline,
                "whole_step_roofline": whole_step,
                "cpu_baseline": cpu, "decode_attn_plain": decode_plain}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_rollout_only(args):
    """Config 2 on one GPU: the grouped rollout alone (64 prompts x G=8, prompt U[64,512], 512 new
    tokens, temperature 1, no top-k, 256-token pages) on the bench's model.  value = generated
    tokens/s; the roofline is the rollout phase's (prefill tensor-bound, decode steps HBM-bound:
    weights + the K/V each step must read) over the measured rollout time; the CPU baseline is the
    oracle's rollout by full recompute (the reference's rollout_single scheme) on a bounded sample."""
    import torch

    from qwen3_naive_inference_b200 import ops
    from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config, build_model
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cfg = Qwen3Config(num_hidden_layers=args.layers)
    model = build_model(cfg, device=dev, seed=0)
    max_ctx = args.prompt_max + args.new_tokens
    model._num_blocks = args.prompts * args.group * math.ceil(max_ctx / 256) + 64
    model.max_model_len = max_ctx
    model.use_cuda_graphs = not args.no_graphs
    torch.manual_seed(1234)

    def roll(prompts):
        return model.generate_grouped_with_logprobs(prompts, args.group, max_new_tokens=args.new_tokens,
                                                    temperature=1.0, top_k=None, eos_token_ids=None)

    for i in range(args.warmup):
        roll(make_prompts(args, 0, i, dev))
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    host = [make_prompts(args, 0, 100 + j) for j in range(args.steps)]
    dev_prompts = [[p.to(dev) for p in ps] for ps in host]
    sampler = ClockSampler(0)
    sampler.start()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    gen_tokens = all_tokens = 0
    for ps in dev_prompts:
        seq_tokens, gen, _, _ = roll(ps)
        gen_tokens += sum(len(x) for x in gen)
        all_tokens += sum(len(x) for x in seq_tokens)
    b.record(st)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = a.elapsed_time(b)
    ops.check_device_errors()
    roof = sum(step_roofline([p.shape[1] for p in ps], args.group, args.new_tokens, args.layers, 1.0,
                             peaks)["rollout_s"] for ps in host)
    cpu = None
    if not args.no_cpu_baseline:
        v, sample, th = cpu_rollout_sample()
        cpu = {"value": v, "unit": "generated tokens/s", "cores": th, "kind": "port", "sample": sample}
    print(json.dumps({"metric": "rollout generated tokens/s", "value": gen_tokens / (ms / 1000),
                      "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": ms / args.steps, "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": "config 2: grouped rollout, 64 prompts x G=8, prompt U[64,512], "
                                             "512 new tokens, temperature 1, paged KV 256",
                                 "prompts": args.prompts, "group": args.group, "new_tokens": args.new_tokens,
                                 "layers": args.layers},
                      "all_tokens_per_s": all_tokens / (ms / 1000),
                      "roofline": {"bound": "hbm (decode) + tensor (prefill)", "roofline_s": roof,
                                   "measured_s": ms / 1000, "frac": roof / (ms / 1000),
                                   "basis": "sum over prefill and decode steps of max(FLOP/peak, bytes/peak)"},
                      "clocks": clocks, "cpu_baseline": cpu}), flush=True)


def cpu_rollout_sample(new=4, G=2, P=48):
    """The oracle's rollout by full recompute (one forward of the whole sequence per new token, as
    the reference's rollout_single, qwen3_grpo_train.py:69-120) at the Qwen3-0.6B shape on the host
    cores: 1 prompt x G completions.  Returns (generated tokens/s, sample text, threads)."""
    import torch

    from oracle import ref_model
    from oracle import ref_ops as R
    from qwen3_naive_inference_b200.qwen3_naive import Qwen3Config
    torch.set_num_threads(os.cpu_count())
    cfg = Qwen3Config()
    params = ref_model.init_params(cfg, seed=0)
    g = torch.Generator().manual_seed(11)
    cs = R.rope_cache(cfg.head_dim, P + new + 1, cfg.rope_theta)
    ids = torch.randint(0, 151643, (1, P), generator=g).repeat(G, 1)
    t0 = time.perf_counter()
    with torch.no_grad():
        for _ in range(new):
            lg = ref_model.logits(params, cfg, ids, cos_sin=cs)[:, -1].float()
            probs, _ = R.sample_distribution(lg, 1.0, None)
            ids = torch.cat([ids, torch.multinomial(probs, 1, generator=g)], 1)
    sec = time.perf_counter() - t0
    return (G * new / sec, f"oracle rollout by full recompute, 1 prompt x G={G}, prompt {P}, {new} new tokens, "
            "Qwen3-0.6B shape", torch.get_num_threads())


def kernel_profile(args, torch, run_step, path):
    """One GRPO step under torch.profiler: every kernel's device time from CUPTI activity records
    (graph replays included), summed per kernel name.  Not a timed number: it gives shares."""
    from collections import Counter
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with plain_launches():
        run_step()  # recaptures the decode graphs in this launch mode, outside the profile
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            out = run_step()
            torch.cuda.synchronize()
    tot, cnt = Counter(), Counter()
    recs = []
    for e in prof.events():
        if str(getattr(e, "device_type", "")).endswith("CUDA"):
            name = e.name
            for pre in ("void ", "(anonymous namespace)::", "<unnamed>::"):
                name = name.replace(pre, "")
            name = name.split("(")[0]
            tot[name] += e.time_range.elapsed_us()
            cnt[name] += 1
            recs.append((e.time_range.start, name, e.time_range.elapsed_us()))
    # The rollout ends with a device->host read of its tokens, so every rollout kernel runs before
    # the first kernel of the log-prob/training phases; the rollout's last sampling launch marks it.
    ends = [t for t, n, _ in recs if n == "sample_kernel"]
    split = max(ends) if ends else float("inf")
    phase_tot = {"rollout": Counter(), "ref log-probs + train": Counter()}
    phase_cnt = {"rollout": Counter(), "ref log-probs + train": Counter()}
    for t, n, d in recs:
        ph = "rollout" if t <= split else "ref log-probs + train"
        phase_tot[ph][n] += d
        phase_cnt[ph][n] += 1
    T = sum(tot.values()) or 1.0
    lines = [f"# Kernel time of one GRPO step (CUPTI records via torch.profiler)", "",
             f"Command: python bench.py --warmup {args.warmup} --steps {args.steps}"
             + (" --no-e2e" if args.no_e2e else "") + (" --no-cpu-baseline" if args.no_cpu_baseline else "")
             + f" --kernel-profile {path}"
             + (" --no-graphs" if args.no_graphs else ""), "",
             f"Workload: {WORKLOAD}.  Phases of this step (host wall clock): rollout {out['t_rollout']:.2f} s, "
             f"ref log-probs {out['t_ref']:.2f} s, train {out['t_train']:.2f} s.", "",
             f"Total kernel time {T / 1e3:.1f} ms over {sum(cnt.values())} kernel records.", "",
             "| kernel | launches | total ms | share |", "|---|---|---|---|"]
    for k, v in tot.most_common(40):
        lines.append(f"| {k[:90]} | {cnt[k]} | {v / 1e3:.2f} | {100 * v / T:.1f}% |")
    recs.sort()
    gaps = {"rollout": [0.0, 0], "ref log-probs + train": [0.0, 0]}
    long_gaps = {"rollout": [], "ref log-probs + train": []}
    for (t0, n0, d0), (t1, n1, _) in zip(recs, recs[1:]):
        g = t1 - (t0 + d0)
        ph = "rollout" if t1 <= split else "ref log-probs + train"
        if 0 < g < 100:  # idle time between back-to-back launches (longer gaps are host waits)
            gaps[ph][0] += g
            gaps[ph][1] += 1
        elif g >= 100:
            long_gaps[ph].append((g, n0, n1))
    for ph in phase_tot:
        PT = sum(phase_tot[ph].values()) or 1.0
        lines += ["", f"## {ph}: {PT / 1e3:.1f} ms of kernel time; {gaps[ph][0] / 1e3:.1f} ms idle in "
                  f"{gaps[ph][1]} gaps under 100 us between consecutive kernels", "",
                  "| kernel | launches | total ms | us per launch | share of phase |", "|---|---|---|---|---|"]
        for k, v in phase_tot[ph].most_common(20):
            c = phase_cnt[ph][k]
            lines.append(f"| {k[:90]} | {c} | {v / 1e3:.2f} | {v / c:.2f} | {100 * v / PT:.1f}% |")
        lg = sorted(long_gaps[ph], reverse=True)
        lines += ["", f"{len(lg)} gaps of 100 us or more (the device idle while the host works): "
                  f"{sum(g for g, _, _ in lg) / 1e3:.1f} ms in total; the longest:", "",
                  "| gap us | after kernel | before kernel |", "|---|---|---|"]
        for g, a, b in lg[:15]:
            lines.append(f"| {g:.0f} | {a[:60]} | {b[:60]} |")
        pairs = Counter()
        for g, a, b in lg:
            pairs[(a[:50], b[:50])] += g
        lines += ["", "Long gaps summed by the kernels on either side:", "", "| ms | after | before |",
                  "|---|---|---|"]
        for (a, b), g in pairs.most_common(10):
            lines.append(f"| {g / 1e3:.1f} | {a} | {b} |")
    Path(path).parent.mkdir(parents=True, exist_ok=True)
    Path(path).write_text("\n".join(lines) + "\n")


def run_decode_only(batch):
    import torch

    from qwen3_naive_inference_b200 import ops
    dev = torch.device("cuda", 0)
    ms, nbytes, _ = decode_microbench(torch, ops, dev, n_iter=3, batch=batch)
    print(json.dumps({"kernel": "paged_decode_kernel", "case": f"config 3 shapes, batch {batch}",
                      "ms_per_launch": ms, "algorithmic_bytes": nbytes,
                      "achieved_gbs": nbytes / (ms / 1000) / 1e9, "cpu_baseline": config3_cpu_baseline()}),
          flush=True)


def config3_cpu_baseline(n_seqs=8):
    """The oracle's paged decode attention (gather K/V through the page table, GQA, fp32 softmax;
    flash_attn_with_kvcache semantics, qwen3_naive.py:672-680) on the host cores, on a bounded
    sample of config 3: n_seqs sequences with context U[1k, 8k] in randomly permuted 256-token
    pages.  Returns GB/s of algorithmic bytes (K/V of every context token, q and out)."""
    import torch

    from oracle import ref_ops as R
    torch.set_num_threads(os.cpu_count())
    g = torch.Generator().manual_seed(3)
    hq, hkv, Dh = 16, 8, 128
    ctx = torch.randint(1024, 8193, (n_seqs,), generator=g)
    pages = [(int(c) + 255) // 256 for c in ctx]
    pool = sum(pages)
    perm = torch.randperm(pool, generator=g)
    bt = torch.full((n_seqs, max(pages)), -1, dtype=torch.int32)
    o = 0
    for i, n in enumerate(pages):
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    kc = torch.randn(pool, 256, hkv, Dh, generator=g).to(torch.bfloat16)
    vc = torch.randn(pool, 256, hkv, Dh, generator=g).to(torch.bfloat16)
    q = torch.randn(n_seqs, hq, Dh, generator=g).to(torch.bfloat16)
    R.paged_decode(q[:1], kc, vc, bt[:1], ctx[:1], Dh ** -0.5)
    t0 = time.perf_counter()
    R.paged_decode(q, kc, vc, bt, ctx, Dh ** -0.5)
    sec = time.perf_counter() - t0
    nbytes = int(ctx.sum()) * hkv * Dh * 2 * 2 + n_seqs * hq * Dh * 2 * 2
    return {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n_seqs} sequences of config 3 (ctx U[1k,8k], 16q/8kv, d128), oracle paged decode"}


def rollout_attn_case(torch, ops, dev):
    """Decode attention mid-rollout (config 4 shapes): 64 groups x 8 completions, prompt U[64,512],
    256 generated tokens each.  Builds the K/V pool twice over the same values: the reference's
    layout (every completion holds its own copy of the prompt K/V; plain paged decode) and the
    grouped layout (prompt pages shared, own tokens on fresh pages; grouped decode).  Returns the
    launch closures and the K/V bytes each layout needs per launch."""
    g = torch.Generator().manual_seed(5)
    G, n_groups, gen, hq, hkv, D = 8, 64, 256, 16, 8, 128
    B = G * n_groups
    plens = torch.randint(64, 513, (n_groups,), generator=g).tolist()
    grouped_pages = sum(-(-L // 256) + G * (-(-gen // 256)) for L in plens)
    plain_pages = sum(G * (-(-(L % 256 + gen) // 256)) for L in plens)
    n_pages = grouped_pages + plain_pages
    kc = torch.randn(n_pages, 256, hkv, D, device=dev, dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    free = list(range(n_pages))[::-1]
    tables, ptables, lens, members, shared, kv_start = [], [], [], [], [], []
    src, dst = [], []  # token rows copied into the plain layout
    for L in plens:
        sh = [free.pop() for _ in range(-(-L // 256))]
        n_full = L // 256
        row = []
        for _ in range(G):
            own = [free.pop() for _ in range(-(-gen // 256))]
            row.append(len(tables))
            tables.append(sh + own)
            P = len(sh) * 256
            lens.append(P + gen)
            kv_start.append(P)
            tail = [free.pop() for _ in range(-(-(L - n_full * 256 + gen) // 256))]
            ptables.append(sh[:n_full] + tail)
            for t in range(n_full * 256, L + gen):
                s_slot = sh[t // 256] * 256 + t % 256 if t < L else own[(t - L) // 256] * 256 + (t - L) % 256
                src.append(s_slot)
                dst.append(ptables[-1][t // 256] * 256 + t % 256)
        members.append(row)
        shared.append(L)
    src_t, dst_t = torch.tensor(src, device=dev), torch.tensor(dst, device=dev)
    for c in (kc, vc):
        flat = c.view(-1, hkv, D)
        flat[dst_t] = flat[src_t]

    def table(rows):
        W = max(len(t) for t in rows)
        bt = torch.full((len(rows), W), -1, dtype=torch.int32)
        for i, t in enumerate(rows):
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        return bt.to(dev)

    bt, bt_plain = table(tables), table(ptables)
    plain_lens = [L for L in plens for _ in range(G)]
    cl = (torch.tensor(lens, dtype=torch.int32) - 1).to(dev)
    cl_plain = (torch.tensor(plain_lens, dtype=torch.int32) + gen - 1).to(dev)
    q = torch.randn(B, hq, D, device=dev, dtype=torch.bfloat16)
    mem_d = torch.tensor(members, dtype=torch.int32, device=dev)
    sl_d = torch.tensor(shared, dtype=torch.int32, device=dev)
    ks_d = torch.tensor(kv_start, dtype=torch.int32, device=dev)
    split, ms = ops.decode_split_plan(B, hkv, max(plain_lens) + gen)
    # the rollout's decode graphs plan with the captured context bound (prompt + 512 new + a page)
    ctx_bound = 512 + 512 + 256
    plan = ops.grouped_decode_plan(B, hkv, ctx_bound, ctx_bound)
    ws_p = torch.empty(max(1, ops.lib().qb_paged_decode_workspace_bytes(B, hq, D, ms) // 4), device=dev)
    ws_g = ops.grouped_workspace(B, hq, D, plan, dev)
    # the grouped decode on the plain layout (every sequence its own group, nothing shared)
    mem_1 = torch.full((B, 8), -1, dtype=torch.int32, device=dev)
    mem_1[:, 0] = torch.arange(B, dtype=torch.int32, device=dev)
    zeros_b = torch.zeros(B, dtype=torch.int32, device=dev)
    plan_1 = ops.grouped_decode_plan(B, hkv, 64, ctx_bound)
    ws_1 = ops.grouped_workspace(B, hq, D, plan_1, dev)
    runs = {
        "plain": lambda: ops.paged_decode_attention(q, kc, vc, bt_plain, cl_plain, D ** -0.5, split_tokens=split,
                                                    max_splits=ms, workspace=ws_p),
        "grouped": lambda: ops.paged_decode_attention_grouped(q, kc, vc, bt, cl, D ** -0.5, mem_d, sl_d, ks_d, plan,
                                                              workspace=ws_g),
        "grouped_unshared": lambda: ops.paged_decode_attention_grouped(q, kc, vc, bt_plain, cl_plain, D ** -0.5, mem_1,
                                                                       zeros_b, zeros_b, plan_1, workspace=ws_1),
    }
    kv_plain = (sum(plain_lens) + B * gen) * hkv * D * 4
    kv_grouped = (sum(shared) + B * gen) * hkv * D * 4
    small = 2 * B * hq * D * 2 + bt.numel() * 4 + B * 4 * 2 + mem_d.numel() * 4  # q, out, tables
    return {"runs": runs, "kv_plain": kv_plain, "kv_grouped": kv_grouped, "alg_grouped": kv_grouped + small,
            "plan": {"plain": [split, ms], "grouped": list(plan)}, "own_tokens": B * gen,
            "shared_tokens": sum(shared)}


def time_launches(torch, fn, n=20):
    """Mean ms of ``fn`` over n back-to-back launches between two events on the launching stream
    (after 3 untimed ones).  The K/V read per launch is several times the 126 MB L2."""
    for _ in range(3):
        fn()
    st = torch.cuda.current_stream()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(n):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / n


def run_rollout_attn():
    """Plain paged decode (reference layout) vs the grouped decode (grouped layout) vs the grouped
    decode with nothing shared, on the mid-rollout case; prints ms and K/V bytes read."""
    import torch

    from qwen3_naive_inference_b200 import ops
    dev = torch.device("cuda", 0)
    case = rollout_attn_case(torch, ops, dev)
    runs = case["runs"]
    out = {name: time_launches(torch, fn) for name, fn in runs.items()}
    ref = runs["plain"]().float()
    err = max((runs[k]().float() - ref).abs().max().item() for k in ("grouped", "grouped_unshared"))
    ops.check_device_errors()
    kv_plain, kv_grouped = case["kv_plain"], case["kv_grouped"]
    print(json.dumps({"rollout_attn": {"ms": out, "kv_bytes": {"plain": kv_plain, "grouped": kv_grouped},
                                       "gbs": {"plain": kv_plain / out["plain"] / 1e6,
                                               "grouped_unshared": kv_plain / out["grouped_unshared"] / 1e6,
                                               "grouped_effective": kv_plain / out["grouped"] / 1e6,
                                               "grouped_actual": kv_grouped / out["grouped"] / 1e6},
                                       "plan": case["plan"], "max_abs_diff": err}}), flush=True)

def run_loss_only():
    """Config 1 on one GPU: log-prob -> GRPO loss -> logit gradient over 1024 rows of bf16 logits
    ~N(0,1) (2 prompts x G=4 x 128 tokens, vocab 151936; targets U[0,151643), rewards
    Bernoulli(0.5), old/ref log-probs = current + N(0, 0.05), beta 0.04, clip 0.2, random tail
    masks).  The timed pass is qb_grpo_logit_loss: each row read once into the shared memory of
    a 4-CTA cluster and its gradient written once (the algorithmic minimum); the two-pass chain
    of the training step's chunks (qb_logprob_fwd, qb_grpo_loss, qb_logprob_bwd) is timed beside
    it.  The backward overwrites the logits, so each pass starts from a fresh copy, followed by
    an L2 flush, both outside the timed events."""
    import torch

    from qwen3_naive_inference_b200 import ops
    dev = torch.device("cuda", 0)
    N, S, V = 8, 128, 151936
    g = torch.Generator(device=dev).manual_seed(1)
    logits0 = torch.randn(N * S, V, device=dev, generator=g).to(torch.bfloat16)
    work = torch.empty_like(logits0)
    flush = torch.empty(256 * 2**20, dtype=torch.uint8, device=dev)
    tgt = torch.randint(0, 151643, (N * S,), device=dev, generator=g)
    dest = torch.arange(N * S, dtype=torch.int64, device=dev)
    lens = torch.randint(1, S + 1, (N,), device=dev, generator=g)
    mask = (torch.arange(S, device=dev)[None, :] < lens[:, None]).float()
    rewards = torch.bernoulli(torch.full((N,), 0.5, device=dev), generator=g)
    gids = torch.arange(N, device=dev) // 4
    new_lp = torch.zeros(N, S, device=dev)
    lse = torch.empty(N * S, device=dev)
    grad = torch.zeros(N, S, device=dev)
    loss = torch.zeros(3, device=dev)
    L, err = ops.lib(), ops.err_flag(dev)
    mask_total = ops.mask_sum(mask)

    def fwd(x):
        ops.check(L.qb_logprob_fwd(x.data_ptr(), N * S, V, x.stride(0), tgt.data_ptr(), dest.data_ptr(),
                                   new_lp.data_ptr(), lse.data_ptr(), err.data_ptr(), ops.stream_ptr()),
                  "qb_logprob_fwd")

    work.copy_(logits0)
    fwd(work)
    old = new_lp + 0.05 * torch.randn(N, S, device=dev, generator=g)
    ref = new_lp + 0.05 * torch.randn(N, S, device=dev, generator=g)

    def step():
        fwd(work)
        ops.grpo_loss_raw(rewards, gids, new_lp, old, mask, ref_lp=ref, mask_total=mask_total, clip_eps=0.2,
                          beta=0.04, row_begin=0, row_end=N, grad_new=grad, loss_out=loss)
        ops.check(L.qb_logprob_bwd(work.data_ptr(), N * S, V, work.stride(0), tgt.data_ptr(), dest.data_ptr(),
                                   lse.data_ptr(), grad.data_ptr(), err.data_ptr(), ops.stream_ptr()),
                  "qb_logprob_bwd")

    def single_pass():  # qb_grpo_logit_loss: one read and one write of the logits
        ops.grpo_logit_loss(work, tgt, rewards, gids, old, mask, ref_lp=ref, mask_total=mask_total, clip_eps=0.2,
                            beta=0.04, loss_out=loss)

    st = torch.cuda.current_stream()

    def time_pass(fn, n=10, warm=3):
        total = 0.0
        for i in range(warm + n):
            work.copy_(logits0)
            loss.zero_()
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            fn()
            e1.record(st)
            torch.cuda.synchronize()
            if i >= warm:
                total += e0.elapsed_time(e1)
        ops.check_device_errors()
        return total / n

    ms_two = time_pass(step)
    ms = time_pass(single_pass)
    alg = 2 * N * S * V * 2     # read the logits + write their gradient, once each
    moved = 2 * N * S * V * 2   # the single-pass kernel moves exactly that
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    cpu = config1_cpu_baseline()
    print(json.dumps({"loss_only": {"rows": N * S, "vocab": V, "ms": ms, "algorithmic_bytes": alg,
                                    "achieved_gbs": alg / (ms / 1000) / 1e9, "frac_of_hbm": alg / (ms / 1000) / 1e9 / hbm,
                                    "bytes_moved": moved, "moved_gbs": moved / (ms / 1000) / 1e9,
                                    "tokens_per_s": N * S / (ms / 1000), "loss": loss.tolist(),
                                    "kernel": "logit_loss_kernel (4-CTA clusters, one read + one write)",
                                    "two_pass_ms": ms_two, "two_pass_kernels": "logprob_fwd + grpo_loss + logprob_bwd",
                                    "cpu_baseline": cpu}}), flush=True)


def config1_cpu_baseline(reps=3):
    """Config 1 exactly on the host cores with the oracle (the reference's pure-PyTorch path:
    fp32 log_softmax + gather of [1024, 151936] bf16 logits, compute_grpo_advantage, the clipped
    surrogate + 0.04 k3 KL masked token mean, backward to the logits;
    qwen3_grpo_train.py:46-53, :162-199).  Returns tokens (rows) per second and ms per pass."""
    import torch

    from oracle import ref_ops as R
    torch.set_num_threads(os.cpu_count())
    N, S, V = 8, 128, 151936
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(N * S, V, generator=g).to(torch.bfloat16)
    tgt = torch.randint(0, 151643, (N * S,), generator=g)
    lens = torch.randint(1, S + 1, (N,), generator=g)
    mask = (torch.arange(S)[None, :] < lens[:, None]).float()
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    gids = torch.arange(N) // 4
    with torch.no_grad():
        base = R.log_probs(logits, tgt).view(N, S)
    old = base + 0.05 * torch.randn(N, S, generator=g)
    ref = base + 0.05 * torch.randn(N, S, generator=g)
    times = []
    for i in range(reps + 1):
        t0 = time.perf_counter()
        x = logits.float().requires_grad_(True)
        lp = torch.log_softmax(x, dim=-1).gather(-1, tgt[:, None]).squeeze(-1).view(N, S)
        adv = R.grpo_advantage(rewards, gids)
        loss = R.ppo_loss(old, lp, adv[:, None] * mask, mask, 0.2, ref, 0.04)
        loss.backward()
        if i:
            times.append(time.perf_counter() - t0)
    ms = 1000 * sum(times) / len(times)
    return {"value": N * S / (ms / 1000), "unit": "tokens/s", "ms_per_pass": ms, "cores": torch.get_num_threads(),
            "kind": "port", "sample": "config 1 exactly: 1024 rows x 151936 bf16 logits, fp32 log-softmax + gather, "
                                      "advantages, clipped + KL loss, backward to the logits (oracle, all host threads)"}


GEMM_SHAPES = {  # (M, N, K): tokens x out x in of the model's projections
    "qkv_proj": (8192, 4096, 1024), "o_proj": (8192, 1024, 2048), "gate_up_proj": (8192, 6144, 1024),
    "down_proj": (8192, 1024, 3072), "lm_head": (4096, 151936, 1024), "qkv_decode512": (512, 4096, 1024),
    "lm_head_decode512": (512, 151936, 1024), "o_decode512": (512, 1024, 2048), "down_decode512": (512, 1024, 3072),
    "gate_up_decode512": (512, 6144, 1024),
}


def run_gemm_only(shape=None):
    """Each projection shape on the tcgen05 GEMM and on cuBLAS (torch.mm).  A launch sequence
    cycles through enough copies of the weight to exceed L2 twice (weights come from HBM, as in
    the step, where a layer's weights are read once per decode step) and is captured in a CUDA
    graph, so the time per launch is GPU time, not host launch overhead."""
    import torch

    from qwen3_naive_inference_b200 import ops
    dev = torch.device("cuda", 0)
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("bf16_tflops", 1590.0)
    out = {}
    # a custom shape "M,N,K[,1]": the optional 1 stores B [K, N] (MN-major, as the backward reads a weight)
    shapes = GEMM_SHAPES if shape is None else {"custom": tuple(int(x) for x in shape.split(","))}
    for name, dims in shapes.items():
        M, N, K = dims[:3]
        b_mn = len(dims) > 3 and dims[3] == 1
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        b = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        if b_mn:
            b = b.t().contiguous()
        copies = max(1, min(64, -(-2 * 126 * 2**20 // (N * K * 2))))
        bs = [b] + [b.clone() for _ in range(copies - 1)]
        c = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        res = {}
        ours = (lambda w: ops.gemm_ex(a, False, w, True, out=c)) if b_mn else (lambda w: ops.gemm(a, w, out=c))
        theirs = (lambda w: torch.mm(a, w, out=c)) if b_mn else (lambda w: torch.mm(a, w.t(), out=c))
        for impl, fn in [("tcgen05", ours), ("cublas", theirs)]:
            for w in bs[:3]:
                fn(w)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for w in bs:
                    fn(w)
            st = torch.cuda.current_stream()
            for _ in range(2):
                graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = 5
            e0.record(st)
            for _ in range(reps):
                graph.replay()
            e1.record(st)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / (reps * len(bs))
            from torch.profiler import ProfilerActivity, profile
            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                fn(bs[0])
                torch.cuda.synchronize()
            names = sorted({e.name.split("(")[0][:120] for e in prof.events()
                            if str(getattr(e, "device_type", "")).endswith("CUDA")})
            res[impl] = {"ms": ms, "tflops": 2 * M * N * K / (ms / 1000) / 1e12, "kernels": names}
            del graph
        ref = (a.float() @ (b.float() if b_mn else b.float().t()))
        ours(b)
        res["max_rel_err"] = ((c.float() - ref).abs().max() / ref.abs().max()).item()
        res["frac_of_peak"] = res["tcgen05"]["tflops"] / peak
        res["weight_copies"] = len(bs)
        out[name] = res
        del bs
    print(json.dumps({"gemm": out, "peak_tflops": peak}), flush=True)


def _event_time(torch, fn, reps=20, warm=3):
    """Mean ms per call of fn() over `reps` back-to-back calls, CUDA events on the current stream."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(reps):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_gemm_qk():
    """The qkv projection with QK-norm + RoPE in the GEMM epilogue against the plain GEMM followed
    by the standalone QK-norm + RoPE kernel: T = 512 (decode step: rotated q out, K/V into the paged
    cache) and T = 4096 (training layout: raw projection + rotated copy + rstd)."""
    import torch

    from oracle import ref_ops as R  # the rotation table only
    from qwen3_naive_inference_b200 import ops
    dev = torch.device("cuda", 0)
    bf = torch.bfloat16
    hq, hkv, K = 16, 8, 1024
    N = (hq + 2 * hkv) * 128
    cs = R.rope_cache(128, 4096, 1e6).to(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.03).to(bf)
    qw = torch.ones(128, dtype=bf, device=dev)
    kw = torch.ones(128, dtype=bf, device=dev)
    res = {}
    for T, train in ((512, False), (4096, True)):
        x = torch.randn(T, K, device=dev, generator=g).to(bf)
        pos = torch.randint(0, 4000, (T,), device=dev, generator=g)
        out, raw = torch.empty(T, N, dtype=bf, device=dev), torch.empty(T, N, dtype=bf, device=dev)
        qr, kr = torch.empty(T, hq, device=dev), torch.empty(T, hkv, device=dev)
        kc = torch.zeros(4096, hkv, 128, dtype=bf, device=dev)
        vc = torch.zeros_like(kc)
        slots = torch.arange(T, dtype=torch.int32, device=dev)
        if train:
            fused = lambda: ops.gemm_qk_norm_rope(x, w, pos, cs, qw, kw, 1e-6, hq, hkv, out=out, raw=raw,  # noqa: E731
                                                  q_rstd=qr, k_rstd=kr)
            unfused = lambda: ops._qk_norm_rope_fwd(ops.gemm(x, w, out=raw), pos, cs, qw, kw, 1e-6, hq, hkv)  # noqa: E731
        else:
            fused = lambda: ops.qkv_norm_rope_store(x, w, pos, cs, qw, kw, 1e-6, hq, hkv, kc, vc, slots)  # noqa: E731
            unfused = lambda: ops.qk_norm_rope_store(ops.gemm(x, w, out=raw), pos, cs, qw, kw, 1e-6, hq, hkv,  # noqa: E731
                                                     kc, vc, slots)
        res[f"T{T}"] = {"fused_ms": _event_time(torch, fused), "gemm_then_kernel_ms": _event_time(torch, unfused)}
    ops.check_device_errors()
    print(json.dumps({"gemm_qk_norm_rope": res}), flush=True)


def run_elementwise():
    """The HBM-bound row kernels on one training microbatch (T = 32768 tokens): mean time per call
    (CUDA events) and algorithmic bytes / time."""
    import torch

    from oracle import ref_ops as R  # the rotation table only
    from qwen3_naive_inference_b200 import ops
    dev = torch.device("cuda", 0)
    bf = torch.bfloat16
    T, hq, hkv, H, I = 32768, 16, 8, 1024, 3072
    N = (hq + 2 * hkv) * 128
    g = torch.Generator(device=dev).manual_seed(0)
    cs = R.rope_cache(128, 4096, 1e6).to(dev)
    qkv = torch.randn(T, N, device=dev, generator=g).to(bf)
    pos = torch.randint(0, 4000, (T,), device=dev, generator=g)
    qw = torch.ones(128, dtype=bf, device=dev)
    kw = torch.ones(128, dtype=bf, device=dev)
    rot, q_rstd, k_rstd = ops._qk_norm_rope_fwd(qkv, pos, cs, qw, kw, 1e-6, hq, hkv)
    d = torch.randn(T, N, device=dev, generator=g).to(bf)
    gu = torch.randn(T, 2 * I, device=dev, generator=g).to(bf)
    dh = torch.randn(T, I, device=dev, generator=g).to(bf)
    dgu = torch.empty_like(gu)
    x = torch.randn(T, H, device=dev, generator=g).to(bf)
    dy = torch.randn(T, H, device=dev, generator=g).to(bf)
    nw = torch.ones(H, dtype=bf, device=dev)
    rstd = torch.ones(T, device=dev)
    dx = torch.empty_like(x)
    dnw = torch.zeros(H, device=dev)
    lib = ops.lib()
    cases = {
        # rotated q, k and the copied v: read + write of the row
        "qk_norm_rope_fwd8": (lambda: ops._qk_norm_rope_fwd(qkv, pos, cs, qw, kw, 1e-6, hq, hkv), 2 * T * N * 2),
        # in place in the attention gradient: read dq/dk and raw q/k, write dq/dk (v untouched)
        "qk_norm_rope_bwd8": (lambda: ops._qk_norm_rope_bwd(d, d, qkv, pos, cs, qw, kw, q_rstd, k_rstd, hq, hkv,
                                                            True), 3 * T * (hq + hkv) * 128 * 2),
        "silu_mul_fwd": (lambda: ops.silu_mul(gu), T * 3 * I * 2),
        "silu_mul_bwd": (lambda: ops.check(lib.qb_silu_mul_bwd(ops._p(dh), ops._p(gu), T, I, ops._p(dgu),
                                                               ops.stream_ptr()), "qb_silu_mul_bwd"), T * 5 * I * 2),
        "rmsnorm_bwd": (lambda: ops.check(lib.qb_rmsnorm_bwd(ops._p(dy), ops._p(x), ops._p(nw), ops._p(rstd), ops._p(dx),
                                                             ops._p(dnw), T, H, ops.stream_ptr()), "qb_rmsnorm_bwd"),
                        3 * T * H * 2),
    }
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    hbm = peaks.get("hbm_gbs", 6650.0)
    res = {}
    for name, (fn, nbytes) in cases.items():
        ms = _event_time(torch, fn)
        res[name] = {"ms": ms, "algorithmic_bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9,
                     "frac_of_measured_copy": nbytes / (ms * 1e-3) / 1e9 / hbm}
    ops.check_device_errors()
    print(json.dumps({"elementwise": res, "tokens": T}), flush=True)


def run_attn_only():
    """Packed causal attention of the training step (16 q / 8 kv heads, d128) on one 32k-token
    microbatch of bench-shaped sequences (prompt U[64,512] + 512 completion tokens): forward and
    backward timed with events, TFLOP/s from the causal FLOP count (fwd 4*H*D per (query, key)
    pair, bwd 2.5x fwd)."""
    import torch

    from qwen3_naive_inference_b200 import ops
    from qwen3_naive_inference_b200.qwen3_naive import packed_meta
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(7)
    lens = []
    while sum(lens) < 32768 - 1024:
        lens.append(int(torch.randint(64, 513, (1,), generator=g)) + 512)
    hq, hkv, D = 16, 8, 128
    T = sum(lens)
    pos, cu, tiles = packed_meta(lens, dev)
    qkv = (torch.randn(T, (hq + 2 * hkv) * D, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(True)
    pairs = sum(L * (L + 1) // 2 for L in lens)
    fwd_flop = 4 * hq * D * pairs

    def fwd():
        return ops.attention_packed(qkv, cu, tiles, hq, hkv, D ** -0.5)

    out = fwd()
    dout = torch.randn_like(out)
    ms_f = time_launches(torch, fwd, n=10)
    o = fwd()
    ms_fb = time_launches(torch, lambda: torch.autograd.grad(o, qkv, dout, retain_graph=True), n=10)
    ops.check_device_errors()
    print(json.dumps({"attn": {"tokens": T, "sequences": len(lens), "fwd_ms": ms_f, "bwd_ms": ms_fb,
                               "fwd_tflops": fwd_flop / (ms_f / 1e3) / 1e12,
                               "bwd_tflops": 2.5 * fwd_flop / (ms_fb / 1e3) / 1e12}}), flush=True)


def main():
    args = parse()
    if args.no_pdl and args.impl == "ours":
        from qwen3_naive_inference_b200._lib import load
        load().qb_set_pdl(0)
    args.total_prompts = 512
    if args.workload == "cfg5" and args.prompt_max == 512:
        args.prompt_max = 1024
    if args.rollout_attn:
        run_rollout_attn()
    elif args.attn_only:
        run_attn_only()
    elif args.gemm_qk:
        run_gemm_qk()
    elif args.elementwise:
        run_elementwise()
    elif args.gemm_only:
        run_gemm_only(args.gemm_shape)
    elif args.loss_only:
        run_loss_only()
    elif args.decode_only:
        run_decode_only(args.decode_batch)
    elif args.rollout_only:
        run_rollout_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
