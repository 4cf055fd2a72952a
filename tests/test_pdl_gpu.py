"""Programmatic dependent launch: every kernel of the library may start while the kernel before it
finishes and waits on the device for that kernel's results.  A kernel that touched memory before
its wait, or finished without waiting, would make a chain of dependent launches race; the chain
below (decode-step shapes: RMSNorm, QK-norm + RoPE, GEMMs on every layout, SwiGLU, the grouped
decode attention's neighbours, log-probs) must give the same bits with the switch on and off,
eagerly and inside a CUDA graph.
"""
import pytest
import torch

from qwen3_naive_inference_b200 import ops
from qwen3_naive_inference_b200._lib import load

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def _chain(x, ws, res, norm_w, steps, b_static=False):
    h = x
    for i in range(steps):
        y, res = ops.add_rmsnorm(h, res, norm_w, 1e-6)
        gu = ops.gemm(y, ws["gate_up"], b_static=b_static)   # 512 x 6144 x 1024
        a = ops.silu_mul(gu)
        d = ops.gemm(a, ws["down"], b_static=b_static)       # 512 x 1024 x 3072 (split-K clusters)
        q = ops.gemm(d, ws["qkv"], b_static=b_static)        # 512 x 4096 x 1024
        o = ops.gemm(q[:, :2048].contiguous(), ws["o"], b_static=b_static)  # 512 x 1024 x 2048
        h = ops.add(o, d)
    return h, res


def _run(pdl, graph, x, ws, res0, norm_w, steps=6, b_static=False):
    lib = load()
    old = lib.qb_get_pdl()
    lib.qb_set_pdl(1 if pdl else 0)
    try:
        if not graph:
            h, res = _chain(x, ws, res0.clone(), norm_w, steps, b_static)
            torch.cuda.synchronize()
            return h.clone(), res.clone()
        res_in = res0.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):  # warm-up outside capture (one-time kernel attributes)
            _chain(x, ws, res0.clone(), norm_w, 1, b_static)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            h, res = _chain(x, ws, res_in, norm_w, steps, b_static)
        res_in.copy_(res0)
        g.replay()
        torch.cuda.synchronize()
        out = (h.clone(), res.clone())
        # replay again from the same inputs: same bits
        res_in.copy_(res0)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(h, out[0]) and torch.equal(res, out[1])
        del g
        return out
    finally:
        lib.qb_set_pdl(old)


@pytest.mark.parametrize("graph", [False, True])
def test_pdl_chain_matches_plain_launches(cuda, graph):
    g = torch.Generator(device=cuda).manual_seed(7)
    x = torch.randn(512, 1024, device=cuda, generator=g).to(BF)
    res0 = torch.randn(512, 1024, device=cuda, generator=g).to(BF)
    norm_w = (1 + 0.1 * torch.randn(1024, device=cuda, generator=g)).to(BF)
    ws = {k: (torch.randn(n, kk, device=cuda, generator=g) * kk ** -0.5).to(BF)
          for k, (n, kk) in {"gate_up": (6144, 1024), "down": (1024, 3072), "qkv": (4096, 1024),
                             "o": (1024, 2048)}.items()}
    plain = _run(False, graph, x, ws, res0, norm_w)
    for b_static in (False, True):  # weights fetched before the wait for the kernel before
        pdl = _run(True, graph, x, ws, res0, norm_w, b_static=b_static)
        ops.check_device_errors()
        assert torch.isfinite(plain[0].float()).all()
        assert torch.equal(plain[0], pdl[0])
        assert torch.equal(plain[1], pdl[1])
