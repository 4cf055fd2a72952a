"""The allocation-free GRPO loss entry point (qb_grpo_loss_noalloc).

It exists for callers that cannot give the library device memory: hosts whose GPU
memory belongs to another allocator, or FFI bindings that only pass tensors they
already own.  Its scratch is a fixed array inside the library, so it must give the
same results as qb_grpo_loss with a caller-provided workspace, call after call.
This file is collected last so a failure here never hides the other GPU tests.
"""
import ctypes

import pytest
import torch

from qwen3_naive_inference_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _case(seed, N, S, cuda):
    g = torch.Generator().manual_seed(seed)
    G = 4
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    gids = torch.arange(N // G).repeat_interleave(G)
    new = -torch.rand(N, S, generator=g) * 5
    old = new + 0.05 * torch.randn(N, S, generator=g)
    ref = new + 0.05 * torch.randn(N, S, generator=g)
    mask = (torch.rand(N, S, generator=g) > 0.3).float()
    return [t.to(cuda).contiguous() for t in (rewards, gids, new, old, ref, mask)]


def _launch(fn_name, args, N, S, *, rows=None, mask_total=None, sync=True):
    """One call through the C ABI; with_ws entry points get a fresh zeroed workspace.  Returns
    (loss[3], grad, adv) device tensors; with sync=False the call is only enqueued."""
    lib = _lib.load()
    rewards, gids, new, old, ref, mask = args
    r0, r1 = rows if rows is not None else (0, N)
    grad = torch.zeros_like(new)
    loss = torch.zeros(3, dtype=torch.float32, device=new.device)
    adv = torch.zeros(N, dtype=torch.float32, device=new.device)
    p = lambda t: None if t is None else t.data_ptr()
    common = [p(rewards), p(gids), N, S, r0, r1, p(new), p(old), p(ref), p(mask), p(mask_total), 0.2, 0.04, None,
              p(grad), p(loss), p(adv)]
    if fn_name == "qb_grpo_loss":
        ws = torch.zeros(lib.qb_grpo_workspace_bytes(N) // 4 + 1, dtype=torch.float32, device=new.device)
        status = lib.qb_grpo_loss(*common, p(ws), ops.stream_ptr())
    else:
        status = lib.qb_grpo_loss_noalloc(*common, ops.stream_ptr())
    assert status == 0, lib.qb_status_string(status)
    if sync:
        torch.cuda.synchronize()
    return loss, grad, adv


def _same(a, b):
    (l1, g1, a1), (l0, g0, a0) = a, b
    assert torch.allclose(l1, l0, rtol=2e-3, atol=1e-6)
    assert torch.allclose(g1, g0, rtol=1e-4, atol=1e-7)
    assert torch.allclose(a1, a0, rtol=1e-6, atol=1e-6)


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    for seed, (N, S) in enumerate([(24, 40), (64, 130)]):  # two calls in a row, different sizes
        args = _case(seed, N, S, cuda)
        _same(_launch("qb_grpo_loss_noalloc", args, N, S), _launch("qb_grpo_loss", args, N, S))


def test_noalloc_back_to_back_calls_on_one_stream(cuda):
    """Two calls enqueued before one synchronize: the second call's header clear runs after the
    first call's kernels on the stream, so both match the workspace entry point."""
    a, b = _case(10, 32, 70, cuda), _case(11, 48, 33, cuda)
    ra = _launch("qb_grpo_loss_noalloc", a, 32, 70, sync=False)
    rb = _launch("qb_grpo_loss_noalloc", b, 48, 33, sync=False)
    torch.cuda.synchronize()
    _same(ra, _launch("qb_grpo_loss", a, 32, 70))
    _same(rb, _launch("qb_grpo_loss", b, 48, 33))


def test_noalloc_row_range_and_given_denominator(cuda):
    """A microbatch's rows [8, 20) of 24 with the caller's precomputed mask total (the global
    token count), as a microbatched training step calls it."""
    N, S = 24, 50
    args = _case(12, N, S, cuda)
    total = args[5].sum().reshape(1)
    for rows, mt in (((8, 20), total), ((0, 24), total), ((5, 9), None)):
        _same(_launch("qb_grpo_loss_noalloc", args, N, S, rows=rows, mask_total=mt),
              _launch("qb_grpo_loss", args, N, S, rows=rows, mask_total=mt))


def test_noalloc_rejects_bad_arguments_before_any_work(cuda):
    lib = _lib.load()
    status = lib.qb_grpo_loss_noalloc(None, None, 16385, 8, 0, 16385, None, None, None, None, None, 0.2, 0.0,
                                      None, None, None, None, ops.stream_ptr())
    assert status == 1  # QB_ERR_INVALID: more rows than the fixed scratch holds, nothing launched
    args = _case(13, 8, 16, cuda)
    rewards, gids, new, old, ref, mask = args
    p = lambda t: t.data_ptr()
    # a null input is an argument error (not a CUDA error), an empty row range does nothing
    assert lib.qb_grpo_loss_noalloc(p(rewards), p(gids), 8, 16, 0, 8, None, p(old), None, p(mask), None, 0.2, 0.0,
                                    None, None, None, None, ops.stream_ptr()) == 1
    assert lib.qb_grpo_loss_noalloc(p(rewards), p(gids), 8, 16, 3, 2, p(new), p(old), None, p(mask), None, 0.2,
                                    0.0, None, None, None, None, ops.stream_ptr()) == 1
    assert lib.qb_grpo_loss_noalloc(None, None, 8, 16, 4, 4, None, None, None, None, None, 0.2, 0.0, None, None,
                                    None, None, ops.stream_ptr()) == 0
    torch.cuda.synchronize()
