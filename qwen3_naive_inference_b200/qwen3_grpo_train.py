"""GRPO on B200 kernels; drop-in for the reference's ``qwen3_grpo_train.py``.

Reference functions kept with their signatures and semantics:
  forward_logprob, forward_token_log_prob_my_own   (qwen3_grpo_train.py:46-59)
  compute_grpo_advantage                           (:162-173)
  ppo_clipped_loss                                 (:184-199)
  grpo_train_step                                  (:261-286)
  rollout_single, rollout_batch, compute_reward    (:69-151, :212-258, on the paged generator)

Extensions (off by default, so defaults equal the reference):
  * ``ref_log_probs`` / ``beta``: k3 KL to a frozen reference policy;
  * ``shift``: score token t+1 from position t (the reference scores token t at
    position t, qwen3_grpo_train.py:48-52, while its rollout stores each token's
    log-prob from the previous position, :111-116);
  * microbatching with a global token-mean denominator, so a batch too large
    for one pass gives the gradient of the whole batch;
  * ``process_group``: data parallelism -- the mask count and the gradients are
    summed over ranks (NCCL), so every rank steps on the global loss.

:func:`grpo_step` runs the whole north-star step: paged rollout -> rewards ->
reference-policy log-probs -> fused log-prob/loss/backward -> all-reduce -> AdamW.
"""
from __future__ import annotations

import copy
import math
import time

import numpy as np
import torch
import torch.distributed as dist

from . import ops
from .qwen3_naive import Qwen3ForCausalLM, packed_meta

# ---------------------------------------------------------------- hyper-parameters (qwen3_grpo_train.py:22-35)
N_ROLLOUT = 4
PPO_EPOCHS = 1
CLIP_EPSILON = 0.2
MAX_RESPONSE_LEN = 256
TEMPERATURE = 0.8
TOP_K = 20
LEARNING_RATE = 5e-6
EOS_TOKEN_ID = 151645
BOS_TOKEN_ID = 151643


# ---------------------------------------------------------------- log-probs
def forward_logprob(model: Qwen3ForCausalLM, input_ids: torch.Tensor, *, shift: bool = False,
                    chunk_rows: int = 4096) -> torch.Tensor:
    """Per-position token log-probs [batch, seq] fp32, differentiable (qwen3_grpo_train.py:46-53).

    shift=False scores input_ids[:, t] under the logits of position t, as the reference;
    shift=True scores input_ids[:, t] under position t-1 (column 0 is 0).  The
    [batch, seq, vocab] logits are never materialised: lm_head and the log-softmax run
    in row chunks inside :func:`ops.logprob`.
    """
    B, S = input_ids.shape
    h = model.model(input_ids)
    H = h.shape[-1]
    if not shift:
        return ops.logprob(h.reshape(B * S, H), model.lm_head.weight, input_ids.reshape(-1), chunk_rows).view(B, S)
    lp = ops.logprob(h[:, :-1].reshape(B * (S - 1), H), model.lm_head.weight, input_ids[:, 1:].reshape(-1),
                     chunk_rows).view(B, S - 1)
    return torch.cat([torch.zeros(B, 1, dtype=lp.dtype, device=lp.device), lp], dim=1)


forward_token_log_prob_my_own = forward_logprob


# ---------------------------------------------------------------- advantage and loss
def compute_grpo_advantage(rewards: torch.Tensor, prompt_ids: torch.Tensor) -> torch.Tensor:
    """(r - group mean) / (unbiased group std + 1e-8) per prompt group (qwen3_grpo_train.py:162-173)."""
    return ops.grpo_advantage(rewards, prompt_ids)


class _PPOLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, old, new, adv, mask, ref, clip_eps, beta):
        N, S = new.shape
        grad = torch.empty_like(new)
        loss = torch.zeros(3, dtype=torch.float32, device=new.device)
        ws = ops.grpo_workspace(N, new.device)
        ops.check(ops.lib().qb_ppo_clipped_loss(old.data_ptr(), new.data_ptr(), adv.data_ptr(), mask.data_ptr(),
                                                0 if ref is None else ref.data_ptr(), N, S, 0, float(clip_eps),
                                                float(beta), 0, grad.data_ptr(), loss.data_ptr(), ws.data_ptr(),
                                                ops.stream_ptr()), "qb_ppo_clipped_loss")
        ctx.save_for_backward(grad)
        return loss[0]

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return None, grad * g, None, None, None, None, None


def ppo_clipped_loss(old_log_probs, new_log_probs, advantages, response_mask, *, ref_log_probs=None,
                     beta: float = 0.0, clip_epsilon: float = CLIP_EPSILON) -> torch.Tensor:
    """-min(r A, clip(r, 1-eps, 1+eps) A) (+ beta * k3 KL) masked token mean over the whole batch
    (qwen3_grpo_train.py:184-199); one fused CUDA kernel computes the loss and its gradient."""
    f = lambda t: None if t is None else t.float().contiguous()
    return _PPOLoss.apply(f(old_log_probs), f(new_log_probs), f(advantages), f(response_mask), f(ref_log_probs),
                          clip_epsilon, beta if ref_log_probs is not None else 0.0)


# ---------------------------------------------------------------- packed batch
class PackedBatch:
    """Rollout results laid out for the recompute: padded [N, S] fp32 tensors for the loss
    plus per-row token lists for the packed (unpadded) transformer passes."""

    def __init__(self, seq_tokens, prompt_lens, old_log_probs, rewards, group_ids, device, *, shift=True):
        self.N = len(seq_tokens)
        self.lengths = np.array([len(t) for t in seq_tokens], dtype=np.int64)
        self.S = int(self.lengths.max())
        self.prompt_lens = np.asarray(prompt_lens, dtype=np.int64)
        self.tokens = seq_tokens
        self.shift = shift
        N, S = self.N, self.S
        old = np.zeros((N, S), dtype=np.float32)
        mask = np.zeros((N, S), dtype=np.float32)
        for i, (lp, pl) in enumerate(zip(old_log_probs, prompt_lens)):
            old[i, pl:pl + len(lp)] = lp
            mask[i, pl:pl + len(lp)] = 1.0
        self.device = device
        self.old_lp = torch.from_numpy(old).to(device)
        self.mask = torch.from_numpy(mask).to(device)
        self.mask_np = mask
        self.rewards = torch.as_tensor(rewards, dtype=torch.float32).to(device)
        self.group_ids = torch.as_tensor(group_ids, dtype=torch.int64).to(device)
        self.n_tokens = int(self.lengths.sum())

    def microbatches(self, max_tokens: int):
        """Consecutive row ranges [r0, r1) whose packed length stays within ``max_tokens``."""
        out, r0, acc = [], 0, 0
        for r, L in enumerate(self.lengths):
            if r > r0 and acc + L > max_tokens:
                out.append((r0, r))
                r0, acc = r, 0
            acc += int(L)
        out.append((r0, self.N))
        return out

    def rows_meta(self, r0, r1):
        """Device tensors for rows [r0, r1): ids, positions, cu_seqlens, tiles, and for the
        scored positions: packed index ``sel``, ``targets`` and padded destination ``dest``.
        ``row_tok`` (host) is the number of scored positions of each row."""
        lens = self.lengths[r0:r1]
        ids = np.concatenate([np.asarray(self.tokens[r], dtype=np.int64) for r in range(r0, r1)])
        starts = np.concatenate([[0], np.cumsum(lens)[:-1]])
        sel, tgt, dest, row_tok = [], [], [], []
        for k, r in enumerate(range(r0, r1)):
            L, pl = int(lens[k]), int(self.prompt_lens[r])
            if self.shift:   # token p (p >= prompt_len) scored from position p-1
                p = np.arange(pl, L)
                sel.append(starts[k] + p - 1)
                tgt.append(ids[starts[k] + p])
                dest.append(r * self.S + p)
            else:            # token p scored from position p (reference alignment)
                p = np.arange(pl, L)
                sel.append(starts[k] + p)
                tgt.append(ids[starts[k] + p])
                dest.append(r * self.S + p)
            row_tok.append(len(p))
        pos, cu, tiles = packed_meta(lens, self.device)
        cat = lambda xs: torch.from_numpy(np.concatenate(xs).astype(np.int64)).to(self.device, non_blocking=True)
        return (torch.from_numpy(ids).to(self.device, non_blocking=True), pos, cu, tiles, cat(sel), cat(tgt),
                cat(dest), np.asarray(row_tok))


def _row_chunks(row_tok, max_rows_tokens):
    """Split rows (by their scored-token counts) into chunks of at most ``max_rows_tokens``."""
    out, a, acc = [], 0, 0
    for i, n in enumerate(row_tok):
        if i > a and acc + n > max_rows_tokens:
            out.append((a, i))
            a, acc = i, 0
        acc += int(n)
    out.append((a, len(row_tok)))
    return out


@torch.no_grad()
def batch_log_probs(model: Qwen3ForCausalLM, batch: PackedBatch, microbatch_tokens=65536, chunk_rows=4096):
    """Scored-position log-probs of ``model`` for every row, padded [N, S] (no grad)."""
    out = torch.zeros(batch.N, batch.S, dtype=torch.float32, device=batch.device)
    for r0, r1 in batch.microbatches(microbatch_tokens):
        ids, pos, cu, tiles, sel, tgt, dest, _ = batch.rows_meta(r0, r1)
        h = model.model.forward_packed(ids, pos, cu, tiles)
        ops.logprob_forward(h.index_select(0, sel), model.lm_head.weight, tgt, dest=dest, out=out,
                            chunk_rows=chunk_rows)
    return out


def policy_loss_backward(model: Qwen3ForCausalLM, batch: PackedBatch, *, ref_lp=None, beta=0.0,
                         clip_epsilon=CLIP_EPSILON, mask_total=None, microbatch_tokens=32768, chunk_rows=4096,
                         process_group=None):
    """Fused recompute + GRPO loss + backward over microbatches; grads land in ``.grad``.

    Gradients accumulate in fp32 (the model's GradBuffer); with ``process_group`` (or an
    initialised default group) they are summed over ranks in fp32 before the bf16 ``.grad``
    tensors are written.

    For each chunk of rows the lm_head logits are produced once: log-softmax+gather
    (qb_logprob_fwd) -> fused loss and d loss/d logp for those rows (qb_grpo_loss,
    token-local given the global denominator) -> d loss/d logits in place
    (qb_logprob_bwd) -> dh and dW_lm_head.  Returns the loss tensor [3] (total,
    surrogate, kl) on the device.
    """
    dev = batch.device
    N, S = batch.N, batch.S
    if mask_total is None:
        mask_total = ops.mask_sum(batch.mask)
    new_lp = torch.zeros(N, S, dtype=torch.float32, device=dev)
    grad_new = torch.zeros(N, S, dtype=torch.float32, device=dev)
    loss = torch.zeros(3, dtype=torch.float32, device=dev)
    W = model.lm_head.weight
    V = W.shape[0]
    L = ops.lib()
    err = ops.err_flag(dev)
    buf = grad_buffer(model)
    buf.zero()
    buf.fold()  # gradients already present (none after zero_grad) join the fp32 sum
    buf.attach()
    dW = ops.grad32_target(W)
    try:
        _policy_microbatches(model, batch, buf, new_lp, grad_new, loss, W, V, L, err, dW, ref_lp, beta, clip_epsilon,
                             mask_total, microbatch_tokens, chunk_rows)
    finally:
        buf.detach()
    if process_group is not None or (dist.is_available() and dist.is_initialized()):
        buf.allreduce(process_group)
    buf.to_grads()
    return loss, new_lp


def _policy_microbatches(model, batch, buf, new_lp, grad_new, loss, W, V, L, err, dW, ref_lp, beta, clip_epsilon,
                         mask_total, microbatch_tokens, chunk_rows):
    dev = batch.device
    for r0, r1 in batch.microbatches(microbatch_tokens):
        ids, pos, cu, tiles, sel, tgt, dest, row_tok = batch.rows_meta(r0, r1)
        h = model.model.forward_packed(ids, pos, cu, tiles)
        hs_all = h.index_select(0, sel)
        hs = hs_all.detach()
        dhs = torch.empty_like(hs)
        lse = torch.empty(hs.shape[0], dtype=torch.float32, device=dev)
        tok_off = np.concatenate([[0], np.cumsum(row_tok)])
        with torch.no_grad():
            _lm_head_chunks(L, err, W, V, hs, dhs, lse, tgt, dest, new_lp, grad_new, loss, dW, batch, ref_lp,
                            beta, clip_epsilon, mask_total, r0, row_tok, tok_off, chunk_rows)
        hs_all.backward(dhs)
        buf.fold()
        del h, hs_all


def _lm_head_chunks(L, err, W, V, hs, dhs, lse, tgt, dest, new_lp, grad_new, loss, dW, batch, ref_lp, beta,
                    clip_epsilon, mask_total, r0, row_tok, tok_off, chunk_rows):
    """Per row chunk: logits once (GEMM with the log-softmax + gather in its epilogue) -> fused
    loss/grad -> d logits in place -> dh, and dW added into the fp32 accumulator ``dW``."""
    for a, b in _row_chunks(row_tok, chunk_rows):
        t0, t1 = int(tok_off[a]), int(tok_off[b])
        if t1 == t0:
            continue
        hc = hs[t0:t1]
        # one GEMM: bf16 logits for the backward, and the log-softmax + gather from the fp32
        # accumulators in its epilogue
        logits = torch.empty(t1 - t0, V, dtype=torch.bfloat16, device=hs.device)
        ops.lm_head_logprob(hc, W, tgt[t0:t1], dest=dest[t0:t1], out=new_lp.view(-1), lse=lse[t0:t1],
                            logits=logits)
        ops.grpo_loss_raw(batch.rewards, batch.group_ids, new_lp, batch.old_lp, batch.mask, ref_lp=ref_lp,
                          mask_total=mask_total, clip_eps=clip_epsilon, beta=beta, row_begin=r0 + a,
                          row_end=r0 + b, grad_new=grad_new, loss_out=loss)
        ops.check(L.qb_logprob_bwd(logits.data_ptr(), t1 - t0, V, logits.stride(0), tgt.data_ptr() + 8 * t0,
                                   dest.data_ptr() + 8 * t0, lse.data_ptr() + 4 * t0, grad_new.data_ptr(),
                                   err.data_ptr(), ops.stream_ptr()), "qb_logprob_bwd")
        ops.gemm_ex(logits, False, W, True, out=dhs[t0:t1])  # dh = dlogits . W
        ops.gemm_ex(logits, True, hc, True, out=dW, mode=2)   # dW += dlogits^T . h (fp32)
        del logits


def grpo_train_step(model, optimizer, input_ids, old_log_probs, response_mask, rewards, prompt_ids, *,
                    ref_log_probs=None, beta: float = 0.0, clip_epsilon: float = CLIP_EPSILON,
                    ppo_epochs: int = PPO_EPOCHS, shift: bool = False):
    """Advantages -> PPO epochs of {log-prob recompute, clipped loss, zero_grad, backward, AdamW}
    (qwen3_grpo_train.py:261-286); returns the mean loss as a float.

    Inputs are the reference's padded [batch, seq] tensors.  The forward runs on the
    full padded rows, as the reference does; :func:`grpo_step` is the packed,
    microbatched fast path.
    """
    advantages = compute_grpo_advantage(rewards, prompt_ids)
    token_adv = advantages.unsqueeze(-1) * response_mask.float()
    total = 0.0
    for _ in range(ppo_epochs):
        new_lp = forward_logprob(model, input_ids, shift=shift)
        loss = ppo_clipped_loss(old_log_probs, new_lp, token_adv, response_mask, ref_log_probs=ref_log_probs,
                                beta=beta, clip_epsilon=clip_epsilon)
        optimizer.zero_grad()
        loss.backward()
        optimizer.step()
        total += loss.item()
    return total / ppo_epochs


# ---------------------------------------------------------------- rollout
def compute_reward(response_text: str) -> float:
    """The reference's placeholder reward (qwen3_grpo_train.py:141-151): 1.0 when the decoded
    response has more than 5 non-blank characters, else 0.0."""
    return 1.0 if len(response_text.strip()) > 5 else 0.0


def _reward(tokenizer, completion, reward_fn):
    if reward_fn is not None:
        return float(reward_fn(completion))
    if tokenizer is None:  # no tokenizer: the same rule on the completion's token count
        return 1.0 if len(completion) > 5 else 0.0
    return compute_reward(tokenizer.decode(completion, skip_special_tokens=True))


@torch.no_grad()
def rollout_single(model, prompt_ids, tokenizer=None, *, max_new_tokens=MAX_RESPONSE_LEN,
                   temperature=TEMPERATURE, top_k=TOP_K, eos_token_ids=(EOS_TOKEN_ID, BOS_TOKEN_ID)):
    """One completion of ``prompt_ids`` [1, L] with each sampled token's log-prob
    (qwen3_grpo_train.py:69-120): returns input_ids [1, T] (prompt + response, the stop token
    included), old_log_probs [T] (0 on the prompt, the token's sampling log-prob at its own
    position) and response_mask [T].  Runs on the paged generator; ``tokenizer`` is accepted
    for signature compatibility (the reference does not use it here either)."""
    dev = model.lm_head.weight.device
    seq_tokens, _gen, lps, plens = model.generate_continuous_with_logprobs(
        [prompt_ids], max_new_tokens=max_new_tokens, temperature=temperature, top_k=top_k,
        eos_token_ids=list(eos_token_ids) if eos_token_ids else None)
    toks, lp, pl = seq_tokens[0], lps[0], plens[0]
    T = len(toks)
    old = torch.zeros(T)
    mask = torch.zeros(T)
    old[pl:pl + len(lp)] = torch.tensor(lp)
    mask[pl:pl + len(lp)] = 1.0
    return torch.tensor([toks], dtype=torch.long).to(dev), old.to(dev), mask.to(dev)


@torch.no_grad()
def rollout_batch(model, tokenizer, prompts, *, n_rollout=N_ROLLOUT, max_new_tokens=MAX_RESPONSE_LEN,
                  temperature=TEMPERATURE, top_k=TOP_K, eos_token_ids=(EOS_TOKEN_ID, BOS_TOKEN_ID),
                  reward_fn=None):
    """``n_rollout`` completions per prompt, padded like the reference's rollout_batch
    (qwen3_grpo_train.py:212-258): input_ids [B, L] (0-padded), old_log_probs and
    response_mask [B, L] with each response token's sampling log-prob at its own position,
    rewards [B] and prompt_ids [B].  All completions run in one batch on the paged generator
    instead of one reference rollout_single call each.  Rewards: ``compute_reward`` of the
    completion decoded by ``tokenizer`` (special tokens skipped), as the reference; with
    ``tokenizer=None`` the same rule on the completion's token count; ``reward_fn(completion
    token ids) -> float`` overrides both."""
    expanded, pid = [], []
    for i, p in enumerate(prompts):
        for _ in range(n_rollout):
            expanded.append(p)
            pid.append(i)
    seq_tokens, gen, lps, plens = model.generate_continuous_with_logprobs(
        expanded, max_new_tokens=max_new_tokens, temperature=temperature, top_k=top_k,
        eos_token_ids=list(eos_token_ids) if eos_token_ids else None)
    dev = model.lm_head.weight.device
    B, Lmax = len(seq_tokens), max(len(t) for t in seq_tokens)
    ids = torch.zeros(B, Lmax, dtype=torch.long)
    old = torch.zeros(B, Lmax)
    mask = torch.zeros(B, Lmax)
    for i, (t, lp, pl) in enumerate(zip(seq_tokens, lps, plens)):
        ids[i, :len(t)] = torch.tensor(t)
        old[i, pl:pl + len(lp)] = torch.tensor(lp)
        mask[i, pl:pl + len(lp)] = 1.0
    rewards = torch.tensor([_reward(tokenizer, g, reward_fn) for g in gen])
    return ids.to(dev), old.to(dev), mask.to(dev), rewards.to(dev), torch.tensor(pid, device=dev)


# ---------------------------------------------------------------- the full step
def make_reference_copy(model: Qwen3ForCausalLM) -> Qwen3ForCausalLM:
    """Frozen copy of the policy's weights (the KL anchor); shares no storage with it and
    carries none of the policy's KV cache or captured graphs."""
    from .qwen3_naive import build_model
    w = model.lm_head.weight
    ref = build_model(model.config, device=w.device, dtype=w.dtype, seed=None)
    with torch.no_grad():
        src = dict(model.named_parameters())
        for name, p in ref.named_parameters():
            p.copy_(src[name])
            p.requires_grad_(False)
    return ref


class GradBuffer:
    """One flat fp32 buffer holding the gradient of every trainable parameter of a model.

    During a fused training pass (:func:`policy_loss_backward`) each parameter carries a view of
    it as ``_qb_grad32``: the projection, lm_head and embedding backward kernels add their
    products straight into that view (GEMM mode 2, fp32), so microbatches accumulate in fp32;
    the few small gradients autograd still returns in bf16 (norm weights) are folded in after each
    microbatch.  For data parallelism the buffer is all-reduced in place, in flat buckets, in fp32
    (no per-hop bf16 rounding, no concatenation or copy-back), and only then converted to the bf16
    ``.grad`` tensors the optimizer reads.  The tied lm_head and embedding are two Parameters with
    two gradients (the reference steps both, qwen3_naive.py:830-831), so both are reduced."""

    def __init__(self, model):
        self.params = [p for p in model.parameters() if p.requires_grad]
        n = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(n, dtype=torch.float32, device=self.params[0].device)
        self.views, off = [], 0
        for p in self.params:
            self.views.append(self.flat[off:off + p.numel()].view(p.shape))
            off += p.numel()

    def zero(self):
        self.flat.zero_()

    def attach(self):
        for p, v in zip(self.params, self.views):
            p._qb_grad32 = v

    def detach(self):
        for p in self.params:
            if hasattr(p, "_qb_grad32"):
                del p._qb_grad32

    def fold(self):
        """Adds gradients autograd returned in bf16 into the fp32 views and clears them."""
        for p, v in zip(self.params, self.views):
            if p.grad is not None:
                v.add_(p.grad)
                p.grad = None

    def allreduce(self, group=None, bucket_bytes=512 << 20):
        """Sums the buffer over the ranks of ``group`` in place, bucket by bucket."""
        step = max(1, bucket_bytes // 4)
        for a in range(0, self.flat.numel(), step):
            dist.all_reduce(self.flat[a:a + step], group=group)

    def to_grads(self):
        """bf16 ``.grad`` of every parameter from its fp32 view (the optimizer's input)."""
        for p, v in zip(self.params, self.views):
            p.grad = ops._to_bf16(v) if v.is_cuda else v.to(p.dtype)


def grad_buffer(model) -> GradBuffer:
    buf = getattr(model, "_qb_grad_buffer", None)
    if buf is None:
        buf = GradBuffer(model)
        model._qb_grad_buffer = buf
    return buf


def allreduce_grads(model, group=None, bucket_bytes=512 << 20):
    """Sums every parameter's ``.grad`` over ranks through the model's fp32 GradBuffer (for callers
    that ran their own backward; :func:`grpo_step` reduces the fp32 accumulators directly)."""
    if group is None and not (dist.is_available() and dist.is_initialized()):
        return
    buf = grad_buffer(model)
    buf.zero()
    buf.fold()
    buf.allreduce(group, bucket_bytes)
    buf.to_grads()


def grpo_step(policy: Qwen3ForCausalLM, optimizer, prompts, *, ref_model=None, group_size=8, max_new_tokens=512,
              temperature=1.0, top_k=None, eos_token_ids=None, rewards=None, reward_gen=None, beta=0.04,
              clip_epsilon=CLIP_EPSILON, shift=True, microbatch_tokens=32768, chunk_rows=4096,
              process_group=None, return_batch=False, share_prefix=True):
    """One GRPO step (the north-star path) on this rank's prompt groups.

    prompts: list of [1, L] int64 tensors (this rank's share); each is sampled
    ``group_size`` times.  rewards: optional [n_prompts*group_size] tensor; otherwise
    Bernoulli(0.5) from ``reward_gen`` (a torch.Generator).  With ``process_group``
    (or an initialised default group) the response-token count and the gradients are
    summed across ranks before the optimizer step.  Returns a dict of metrics; all
    device work is complete on return (the loss is read back).
    """
    dev = policy.lm_head.weight.device
    t0 = time.perf_counter()
    expanded = [p for p in prompts for _ in range(group_size)]
    gids = [i for i in range(len(prompts)) for _ in range(group_size)]
    if share_prefix and group_size <= 8:
        # prompt prefilled once per group, its KV pages shared by the G completions
        seq_tokens, gen, lps, plens = policy.generate_grouped_with_logprobs(
            prompts, group_size, max_new_tokens=max_new_tokens, temperature=temperature, top_k=top_k,
            eos_token_ids=eos_token_ids)
    else:  # the reference's scheduler: every completion prefilled and stored separately
        seq_tokens, gen, lps, plens = policy.generate_continuous_with_logprobs(
            expanded, max_new_tokens=max_new_tokens, temperature=temperature, top_k=top_k,
            eos_token_ids=eos_token_ids)
    t_roll = time.perf_counter()
    if rewards is None:
        rewards = torch.bernoulli(torch.full((len(expanded),), 0.5), generator=reward_gen)
    batch = PackedBatch(seq_tokens, plens, lps, rewards, gids, dev, shift=shift)
    use_dist = process_group is not None or (dist.is_available() and dist.is_initialized())
    mask_total = ops.mask_sum(batch.mask)
    if use_dist:
        dist.all_reduce(mask_total, group=process_group)
    ref_lp = None
    if ref_model is not None and beta != 0.0:
        ref_lp = batch_log_probs(ref_model, batch, microbatch_tokens=2 * microbatch_tokens, chunk_rows=chunk_rows)
    t_ref = time.perf_counter()
    optimizer.zero_grad(set_to_none=True)
    loss, _ = policy_loss_backward(policy, batch, ref_lp=ref_lp, beta=beta if ref_lp is not None else 0.0,
                                   clip_epsilon=clip_epsilon, mask_total=mask_total,
                                   microbatch_tokens=microbatch_tokens, chunk_rows=chunk_rows,
                                   process_group=process_group)
    optimizer.step()
    loss_host = loss.cpu()  # the step's one device->host read of the result
    t_end = time.perf_counter()
    out = {"loss": float(loss_host[0]), "surrogate": float(loss_host[1]), "kl": float(loss_host[2]),
           "tokens": batch.n_tokens, "completion_tokens": int(sum(len(g) for g in gen)),
           "prompt_tokens": int(sum(plens)), "mean_reward": float(torch.as_tensor(rewards).float().mean()),
           "t_rollout": t_roll - t0, "t_ref": t_ref - t_roll, "t_train": t_end - t_ref,
           "rollout_stats": dict(policy.rollout_stats)}
    if return_batch:
        out["batch"] = batch
    return out
