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


def _run(fn_name, args, N, S, with_ws):
    lib = _lib.load()
    rewards, gids, new, old, ref, mask = args
    grad = torch.empty_like(new)
    loss = torch.zeros(3, dtype=torch.float32, device=new.device)
    adv = torch.empty(N, dtype=torch.float32, device=new.device)
    p = lambda t: t.data_ptr()
    common = [p(rewards), p(gids), N, S, 0, N, p(new), p(old), p(ref), p(mask), None, 0.2, 0.04, None, p(grad),
              p(loss), p(adv)]
    if with_ws:
        ws = torch.zeros(lib.qb_grpo_workspace_bytes(N) // 4 + 1, dtype=torch.float32, device=new.device)
        status = getattr(lib, fn_name)(*common, p(ws), ops.stream_ptr())
    else:
        status = getattr(lib, fn_name)(*common, ops.stream_ptr())
    assert status == 0, lib.qb_status_string(status)
    torch.cuda.synchronize()
    return loss, grad, adv


def test_noalloc_matches_workspace_entry_point_twice(cuda):
    for seed, (N, S) in enumerate([(24, 40), (64, 130)]):  # two calls in a row, different sizes
        args = _case(seed, N, S, cuda)
        l0, g0, a0 = _run("qb_grpo_loss", args, N, S, with_ws=True)
        l1, g1, a1 = _run("qb_grpo_loss_noalloc", args, N, S, with_ws=False)
        assert torch.allclose(l1, l0, rtol=2e-3, atol=1e-6)
        assert torch.allclose(g1, g0, rtol=1e-4, atol=1e-7)
        assert torch.allclose(a1, a0, rtol=1e-6, atol=1e-6)


def test_noalloc_rejects_rows_beyond_its_scratch(cuda):
    lib = _lib.load()
    status = lib.qb_grpo_loss_noalloc(None, None, 16385, 8, 0, 16385, None, None, None, None, None, 0.2, 0.0,
                                      None, None, None, None, ops.stream_ptr())
    assert status == 1  # QB_ERR_INVALID, nothing launched
