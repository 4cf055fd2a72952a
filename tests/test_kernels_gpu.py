"""Kernel-level parity: every CUDA entry point against the CPU oracle on seeded inputs.

Tolerances: bf16 outputs within a few bf16 ulps (atol/rtol 1e-2 relative to unit-scale
data), fp32 reductions within 1e-5..2e-3 relative as stated per test.
"""
import math

import numpy as np
import pytest
import torch

from oracle import ref_ops as R
from qwen3_naive_inference_b200 import ops

pytestmark = pytest.mark.gpu
BF = torch.bfloat16


def gen(seed):
    return torch.Generator().manual_seed(seed)


def close_bf16(a, b, tol=2e-2):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-6
    assert err <= tol * scale, f"max abs err {err} vs scale {scale}"


def test_embedding(cuda):
    g = gen(0)
    W = torch.randn(1000, 256, generator=g).to(BF)
    ids = torch.randint(0, 1000, (77,), generator=g)
    out = ops.embedding(ids.to(cuda), W.to(cuda))
    assert torch.equal(out.cpu(), W[ids])
    Wd = W.to(cuda).requires_grad_(True)
    y = ops.embedding(ids.to(cuda), Wd)
    gy = torch.randn(77, 256, generator=g).to(BF)
    y.backward(gy.to(cuda))
    ref = torch.zeros(1000, 256).index_add_(0, ids, gy.float()).to(BF)
    close_bf16(Wd.grad, ref, 1e-2)
    ops.check_device_errors()


@pytest.mark.parametrize("rows,cols", [(1, 1024), (37, 1024), (300, 256), (64, 2048)])
def test_rmsnorm(cuda, rows, cols):
    g = gen(rows)
    x = torch.randn(rows, cols, generator=g).to(BF)
    w = (1 + 0.1 * torch.randn(cols, generator=g)).to(BF)
    y = ops.rmsnorm(x.to(cuda), w.to(cuda), 1e-6)
    close_bf16(y, R.rms_norm(x, w, 1e-6), 8e-3)
    r = torch.randn(rows, cols, generator=g).to(BF)
    y2, r2 = ops.add_rmsnorm(x.to(cuda), r.clone().to(cuda), w.to(cuda), 1e-6)
    ry, rr = R.add_rms_norm(x, r, w, 1e-6)
    assert torch.equal(r2.cpu(), rr)
    close_bf16(y2, ry, 8e-3)


def test_rmsnorm_backward(cuda):
    g = gen(3)
    x = torch.randn(129, 1024, generator=g).to(BF)
    w = (1 + 0.1 * torch.randn(1024, generator=g)).to(BF)
    dy = torch.randn(129, 1024, generator=g).to(BF)
    xr, wr = x.float().requires_grad_(True), w.float().requires_grad_(True)
    yr = (xr * torch.rsqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6)) * wr
    yr.backward(dy.float())
    xd, wd = x.to(cuda).requires_grad_(True), w.to(cuda).requires_grad_(True)
    ops.rmsnorm(xd, wd, 1e-6).backward(dy.to(cuda))
    close_bf16(xd.grad, xr.grad, 1e-2)
    close_bf16(wd.grad, wr.grad, 1e-2)


def _qkv_case(T, seed, hq=16, hkv=8):
    g = gen(seed)
    qkv = torch.randn(T, (hq + 2 * hkv) * 128, generator=g).to(BF)
    pos = torch.randint(0, 4000, (T,), generator=g)
    qw = (1 + 0.1 * torch.randn(128, generator=g)).to(BF)
    kw = (1 + 0.1 * torch.randn(128, generator=g)).to(BF)
    return qkv, pos, qw, kw


def test_qk_norm_rope_and_store(cuda):
    T, hq, hkv = 45, 16, 8
    qkv, pos, qw, kw = _qkv_case(T, 5)
    cs = R.rope_cache(128, 4096, 1e6)
    q_ref, k_ref, v_ref = R.qk_norm_rope(qkv, pos, cs, qw, kw, 1e-6, hq, hkv)
    out = ops.qk_norm_rope(qkv.to(cuda), pos.to(cuda), cs.to(cuda), qw.to(cuda), kw.to(cuda), 1e-6, hq, hkv)
    out = out.cpu()
    close_bf16(out[:, :hq * 128].reshape(T, hq, 128), q_ref, 1e-2)
    close_bf16(out[:, hq * 128:(hq + hkv) * 128].reshape(T, hkv, 128), k_ref, 1e-2)
    assert torch.equal(out[:, (hq + hkv) * 128:].reshape(T, hkv, 128), v_ref)
    # paged store: slots with a -1 hole
    nslots = 3 * 256
    slots = torch.randperm(nslots, generator=gen(6))[:T].to(torch.int32)
    slots[3] = -1
    kc = torch.zeros(3, 256, hkv, 128, dtype=BF)
    vc = torch.zeros_like(kc)
    kcd, vcd = kc.to(cuda), vc.to(cuda)
    q = ops.qk_norm_rope_store(qkv.to(cuda), pos.to(cuda), cs.to(cuda), qw.to(cuda), kw.to(cuda), 1e-6, hq, hkv,
                               kcd, vcd, slots.to(cuda))
    close_bf16(q.cpu(), q_ref, 1e-2)
    R.store_kvcache(k_ref, v_ref, kc.view(-1, hkv, 128), vc.view(-1, hkv, 128), slots)
    close_bf16(kcd.cpu(), kc, 1e-2)
    assert torch.equal(vcd.cpu(), vc)
    ops.check_device_errors()


@pytest.mark.parametrize("rope_grad", [True, False])
def test_qk_norm_rope_backward(cuda, rope_grad):
    T, hq, hkv = 33, 16, 8
    qkv, pos, qw, kw = _qkv_case(T, 9)
    cs = R.rope_cache(128, 4096, 1e6)
    dout = torch.randn(T, (hq + 2 * hkv) * 128, generator=gen(10)).to(BF)
    # fp32 autograd restatement of norm -> (bf16 round, straight-through) -> rope
    x = qkv.float().requires_grad_(True)
    qwf, kwf = qw.float().requires_grad_(True), kw.float().requires_grad_(True)
    q = x[:, :hq * 128].reshape(T, hq, 128)
    k = x[:, hq * 128:(hq + hkv) * 128].reshape(T, hkv, 128)
    v = x[:, (hq + hkv) * 128:]
    nq = (q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + 1e-6)) * qwf
    nk = (k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + 1e-6)) * kwf
    rq, rk = R.apply_rope(nq, pos, cs, torch.float32), R.apply_rope(nk, pos, cs, torch.float32)
    if not rope_grad:
        rq, rk = rq.detach(), rk.detach()
    y = torch.cat([rq.reshape(T, -1), rk.reshape(T, -1), v], dim=1)
    y.backward(dout.float())
    xd = qkv.to(cuda).requires_grad_(True)
    qwd, kwd = qw.to(cuda).requires_grad_(True), kw.to(cuda).requires_grad_(True)
    yd = ops.qk_norm_rope(xd, pos.to(cuda), cs.to(cuda), qwd, kwd, 1e-6, hq, hkv, rope_grad=rope_grad)
    yd.backward(dout.to(cuda))
    close_bf16(xd.grad, x.grad, 1e-2)
    if rope_grad:
        close_bf16(qwd.grad, qwf.grad, 1e-2)
        close_bf16(kwd.grad, kwf.grad, 1e-2)
    else:
        assert qwd.grad is None and kwd.grad is None
        assert xd.grad[:, :(hq + hkv) * 128].abs().max().item() == 0.0


@pytest.mark.parametrize("rope_grad", [True, False])
def test_qk_norm_rope_attention_fused_backward(cuda, rope_grad):
    """The fused node (QK-norm backward in place in the attention backward's buffer) against the
    two-node composition: same projection gradient bit for bit, same norm-weight gradients up to
    the order of the fp32 atomics.  1500 tokens: more than one wave of the backward's grid, so
    blocks walk several tokens."""
    hq, hkv = 16, 8
    lens = [700, 300, 500]
    T = sum(lens)
    qkv, pos, qw, kw = _qkv_case(T, 21)
    pos = torch.cat([torch.arange(n) for n in lens])
    cs = R.rope_cache(128, 4096, 1e6).to(cuda)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=cuda)
    tiles = torch.from_numpy(ops.build_tiles(lens)).to(cuda)
    dout = torch.randn(T, hq * 128, generator=gen(22)).to(BF).to(cuda)
    scale = 128 ** -0.5
    grads = []
    for fused in (False, True):
        x = qkv.to(cuda).requires_grad_(True)
        qwd, kwd = qw.to(cuda).requires_grad_(True), kw.to(cuda).requires_grad_(True)
        if fused:
            o = ops.qk_norm_rope_attention(x, pos.to(cuda), cs, qwd, kwd, 1e-6, cu, tiles, hq, hkv, scale,
                                           rope_grad=rope_grad)
        else:
            rot = ops.qk_norm_rope(x, pos.to(cuda), cs, qwd, kwd, 1e-6, hq, hkv, rope_grad=rope_grad)
            o = ops.attention_packed(rot, cu, tiles, hq, hkv, scale)
        o.backward(dout)
        grads.append((o.detach(), x.grad, qwd.grad, kwd.grad))
    ops.check_device_errors()
    (o0, dx0, dq0, dk0), (o1, dx1, dq1, dk1) = grads
    assert torch.equal(o0, o1)
    assert torch.equal(dx0, dx1)
    if rope_grad:
        torch.testing.assert_close(dq1.float(), dq0.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dk1.float(), dk0.float(), rtol=1e-2, atol=1e-2)
    else:
        assert dq1 is None and dk1 is None
        assert dx1[:, :(hq + hkv) * 128].abs().max().item() == 0.0
    with torch.no_grad():
        o2 = ops.qk_norm_rope_attention(qkv.to(cuda), pos.to(cuda), cs, qw.to(cuda), kw.to(cuda), 1e-6, cu, tiles,
                                        hq, hkv, scale)
    assert torch.equal(o2, o0)


@pytest.mark.parametrize("T", [512, 45, 2048])  # decode step (one head per tile), tails, CTA pairs
def test_gemm_qk_norm_rope_matches_unfused(cuda, T):
    """The qkv GEMM with QK-norm + RoPE (+ K/V store) in its epilogue gives the bits of the
    projection followed by the standalone QK-norm + RoPE kernel."""
    hq, hkv, K = 16, 8, 1024
    N = (hq + 2 * hkv) * 128
    g = torch.Generator(device=cuda).manual_seed(T)
    x = torch.randn(T, K, device=cuda, generator=g).to(BF)
    w = (torch.randn(N, K, device=cuda, generator=g) * K ** -0.5).to(BF)
    pos = torch.randint(0, 4000, (T,), device=cuda, generator=g)
    cs = R.rope_cache(128, 4096, 1e6).to(cuda)
    qw = (1 + 0.1 * torch.randn(128, device=cuda, generator=g)).to(BF)
    kw = (1 + 0.1 * torch.randn(128, device=cuda, generator=g)).to(BF)
    plain = ops.gemm(x, w)
    # training layout: rotated copy, raw projection, rstd
    out, raw = torch.empty_like(plain), torch.empty_like(plain)
    qr = torch.empty(T, hq, dtype=torch.float32, device=cuda)
    kr = torch.empty(T, hkv, dtype=torch.float32, device=cuda)
    ops.gemm_qk_norm_rope(x, w, pos, cs, qw, kw, 1e-6, hq, hkv, out=out, raw=raw, q_rstd=qr, k_rstd=kr)
    # the projection: the plain GEMM's bits where it picks the same (non split-K) layout, else
    # within its output rounding
    if ops.gemm_plan(T, N, K)[2] == 1:
        assert torch.equal(raw, plain)
    else:
        assert (raw.float() - plain.float()).abs().max().item() <= 1e-2 * plain.float().abs().max().item()
    qkv = raw
    ref_out, ref_qr, ref_kr = ops._qk_norm_rope_fwd(qkv, pos, cs, qw, kw, 1e-6, hq, hkv)
    assert torch.equal(out, ref_out)
    assert torch.equal(qr, ref_qr) and torch.equal(kr, ref_kr)
    # paged layout: rotated q, k/v rows into the cache (slot -1 skips the store)
    nslots = 3 * 4096
    slots = torch.randperm(nslots, device=cuda, generator=g)[:T].to(torch.int32)
    slots[T // 2] = -1
    kc0 = torch.zeros(nslots, hkv, 128, dtype=BF, device=cuda)
    kc, vc, kc_r, vc_r = kc0.clone(), kc0.clone(), kc0.clone(), kc0.clone()
    q_ref = ops.qk_norm_rope_store(qkv, pos, cs, qw, kw, 1e-6, hq, hkv, kc_r, vc_r, slots)
    q = ops.qkv_norm_rope_store(x, w, pos, cs, qw, kw, 1e-6, hq, hkv, kc, vc, slots)
    assert torch.equal(q, q_ref)
    assert torch.equal(kc, kc_r) and torch.equal(vc, vc_r)
    ops.check_device_errors()


@pytest.mark.parametrize("rope_grad", [True, False])
def test_qkv_attention_fused_matches_unfused(cuda, rope_grad):
    """Projection + QK-norm + RoPE + attention as one node: same output and gradients as
    linear followed by the QK-norm + attention node (norm-weight grads up to atomics order)."""
    hq, hkv, K = 16, 8, 1024
    lens = [700, 300, 500]
    T = sum(lens)
    g = torch.Generator().manual_seed(31)
    x0 = torch.randn(T, K, generator=g).to(BF).to(cuda)
    w0 = (torch.randn((hq + 2 * hkv) * 128, K, generator=g) * K ** -0.5).to(BF).to(cuda)
    qw0 = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    kw0 = (1 + 0.1 * torch.randn(128, generator=g)).to(BF).to(cuda)
    pos = torch.cat([torch.arange(n) for n in lens]).to(cuda)
    cs = R.rope_cache(128, 4096, 1e6).to(cuda)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32, device=cuda)
    tiles = torch.from_numpy(ops.build_tiles(lens)).to(cuda)
    dout = torch.randn(T, hq * 128, generator=g).to(BF).to(cuda)
    res = []
    for fused in (False, True):
        x, w = x0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
        qw, kw = qw0.clone().requires_grad_(True), kw0.clone().requires_grad_(True)
        if fused:
            o = ops.qkv_attention(x, w, pos, cs, qw, kw, 1e-6, cu, tiles, hq, hkv, 128 ** -0.5, rope_grad=rope_grad)
        else:
            o = ops.qk_norm_rope_attention(ops.linear(x, w), pos, cs, qw, kw, 1e-6, cu, tiles, hq, hkv, 128 ** -0.5,
                                           rope_grad=rope_grad)
        o.backward(dout)
        res.append((o.detach(), x.grad, w.grad, qw.grad, kw.grad))
    ops.check_device_errors()
    (o0, dx0, dw0, dq0, dk0), (o1, dx1, dw1, dq1, dk1) = res
    assert torch.equal(o0, o1) and torch.equal(dx0, dx1) and torch.equal(dw0, dw1)
    if rope_grad:
        torch.testing.assert_close(dq1.float(), dq0.float(), rtol=1e-2, atol=1e-2)
        torch.testing.assert_close(dk1.float(), dk0.float(), rtol=1e-2, atol=1e-2)
    else:
        assert dq1 is None and dk1 is None and dq0 is None and dk0 is None
    with torch.no_grad():
        o2 = ops.qkv_attention(x0, w0, pos, cs, qw0, kw0, 1e-6, cu, tiles, hq, hkv, 128 ** -0.5)
    assert torch.equal(o2, o0)


def test_silu_mul(cuda):
    g = gen(11)
    gu = torch.randn(19, 2 * 3072, generator=g).to(BF)
    close_bf16(ops.silu_mul(gu.to(cuda)), R.silu_mul(gu), 1e-2)
    d = torch.randn(19, 3072, generator=g).to(BF)
    x = gu.float().requires_grad_(True)
    (torch.nn.functional.silu(x[:, :3072]) * x[:, 3072:]).backward(d.float())
    xd = gu.to(cuda).requires_grad_(True)
    ops.silu_mul(xd).backward(d.to(cuda))
    close_bf16(xd.grad, x.grad, 1e-2)


def _paged_case(lens, seed, hkv=8, extra_pages=3):
    """Random caches with pages shuffled in a pool; block table per sequence."""
    g = gen(seed)
    pages_per = [math.ceil(L / 256) for L in lens]
    n_pages = sum(pages_per) + extra_pages
    perm = torch.randperm(n_pages, generator=g)
    kc = torch.randn(n_pages, 256, hkv, 128, generator=g).to(BF)
    vc = torch.randn(n_pages, 256, hkv, 128, generator=g).to(BF)
    width = max(pages_per)
    bt = torch.full((len(lens), width), -1, dtype=torch.int32)
    o = 0
    for i, n in enumerate(pages_per):
        bt[i, :n] = perm[o:o + n].to(torch.int32)
        o += n
    return kc, vc, bt


@pytest.mark.parametrize("lens", [[1, 2, 255, 256, 257, 1000], [64] * 3 + [4097], [1], [8192, 1024, 3000]])
def test_paged_decode(cuda, lens):
    B, hq, hkv = len(lens), 16, 8
    kc, vc, bt = _paged_case(lens, len(lens) + lens[-1])
    q = torch.randn(B, hq, 128, generator=gen(1)).to(BF)
    ctx = torch.tensor(lens, dtype=torch.int32) - 1  # context_lens; kernel adds 1
    ref = R.paged_decode(q, kc, vc, bt, ctx + 1, 128 ** -0.5)
    for plan in [None, (64, math.ceil(max(lens) / 64)), (8192, 1)]:
        kw = {} if plan is None else {"split_tokens": plan[0], "max_splits": plan[1]}
        out = ops.paged_decode_attention(q.to(cuda), kc.to(cuda), vc.to(cuda), bt.to(cuda), ctx.to(cuda),
                                         128 ** -0.5, **kw)
        close_bf16(out, ref, 2e-2)
    ops.check_device_errors()


def test_paged_decode_bad_page_sets_error(cuda):
    kc, vc, bt = _paged_case([300], 3)
    bt[0, 1] = 10_000  # out of range: kernel must skip and flag, not fault
    q = torch.randn(1, 16, 128).to(BF)
    ops.paged_decode_attention(q.to(cuda), kc.to(cuda), vc.to(cuda), bt.to(cuda),
                               torch.tensor([299], dtype=torch.int32).to(cuda), 128 ** -0.5)
    with pytest.raises(ops.NativeError):
        ops.check_device_errors()


@pytest.mark.parametrize("qk", [[(5, 5), (1, 300), (130, 700), (1, 1)], [(2048, 2048)], [(64, 64), (65, 320)]])
def test_paged_prefill(cuda, qk):
    hq, hkv = 16, 8
    lq = [a for a, _ in qk]
    lk = [b for _, b in qk]
    kc, vc, bt = _paged_case(lk, sum(lk))
    q = torch.randn(sum(lq), hq, 128, generator=gen(2)).to(BF)
    cu_q = torch.tensor([0] + list(np.cumsum(lq)), dtype=torch.int32)
    cu_k = torch.tensor([0] + list(np.cumsum(lk)), dtype=torch.int32)
    ref = R.paged_attention(q, kc, vc, cu_q, cu_k, bt, 128 ** -0.5)
    for tiles in [None, torch.from_numpy(ops.build_tiles(lq))]:
        out = ops.attention_paged_prefill(q.to(cuda), kc.to(cuda), vc.to(cuda), cu_q.to(cuda), cu_k.to(cuda),
                                          max(lq), bt.to(cuda), 128 ** -0.5,
                                          tiles=None if tiles is None else tiles.to(cuda))
        close_bf16(out, ref, 2e-2)


@pytest.mark.parametrize("lens,qscale", [([1, 63, 64, 65, 200], 1.0), ([513], 1.0), ([1100, 40, 129], 1.0),
                                         ([700, 300], 6.0)])
def test_attention_packed_fwd_bwd(cuda, lens, qscale):
    """Packed causal attention (the training path on tcgen05: forward with 64 query positions x
    2 heads per tile and 64-key tiles, dK/dV on 128-key tiles, dQ) against fp32 autograd; the
    forward per element within 2^-7 of sum_j p_j |v_j| plus one bf16 ulp (P and the output are
    rounded to bf16).  qscale 6 makes the scores wide enough that a row's running max jumps by
    more than 2^8 between key tiles for some rows of a warp and not others, the case in which
    the forward rescales O in TMEM."""
    hq, hkv = 16, 8
    T = sum(lens)
    g = gen(T)
    qkv = torch.randn(T, (hq + 2 * hkv) * 128, generator=g)
    qkv[:, :hq * 128] *= qscale
    qkv = qkv.to(BF)
    dout = torch.randn(T, hq * 128, generator=g).to(BF)
    cu = torch.tensor([0] + list(np.cumsum(lens)), dtype=torch.int32)
    tiles = torch.from_numpy(ops.build_tiles(lens))
    # fp32 autograd reference
    x = qkv.float().requires_grad_(True)
    outs = []
    for b in range(len(lens)):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        L = s1 - s0
        q = x[s0:s1, :hq * 128].reshape(L, hq, 128)
        k = x[s0:s1, hq * 128:(hq + hkv) * 128].reshape(L, hkv, 128).repeat_interleave(2, 1)
        v = x[s0:s1, (hq + hkv) * 128:].reshape(L, hkv, 128).repeat_interleave(2, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) * 128 ** -0.5
        s = s.masked_fill(torch.triu(torch.ones(L, L), 1).bool()[None], float("-inf"))
        outs.append(torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(L, -1))
    y = torch.cat(outs)
    y.backward(dout.float())
    with torch.no_grad():
        scale = []
        for b in range(len(lens)):
            s0, s1 = int(cu[b]), int(cu[b + 1])
            L = s1 - s0
            q = x[s0:s1, :hq * 128].reshape(L, hq, 128)
            k = x[s0:s1, hq * 128:(hq + hkv) * 128].reshape(L, hkv, 128).repeat_interleave(2, 1)
            v = x[s0:s1, (hq + hkv) * 128:].reshape(L, hkv, 128).repeat_interleave(2, 1)
            s = torch.einsum("qhd,khd->hqk", q, k) * 128 ** -0.5
            s = s.masked_fill(torch.triu(torch.ones(L, L), 1).bool()[None], float("-inf"))
            scale.append(torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v.abs()).reshape(L, -1))
        scale = torch.cat(scale)
    xd = qkv.to(cuda).requires_grad_(True)
    yd = ops.attention_packed(xd, cu.to(cuda), tiles.to(cuda), hq, hkv, 128 ** -0.5)
    close_bf16(yd, y.detach(), 2e-2)
    ym, yr = yd.detach().float().cpu(), y.detach()
    ulp = torch.exp2(torch.floor(torch.log2(torch.maximum(ym.abs(), yr.abs()).clamp_min(2.0 ** -126))) - 7)
    assert ((ym - yr).abs() <= 2 ** -7 * scale + ulp).all(), (ym - yr).abs().max().item()
    yd.backward(dout.to(cuda))
    close_bf16(xd.grad, x.grad, 3e-2)


def test_logprob_fwd_bwd(cuda):
    g = gen(21)
    n, H, V = 300, 256, 5000
    h = (torch.randn(n, H, generator=g)).to(BF)
    W = (torch.randn(V, H, generator=g) * 0.1).to(BF)
    t = torch.randint(0, V, (n,), generator=g)
    gl = torch.randn(n, generator=g)
    hr, Wr = h.float().requires_grad_(True), W.float().requires_grad_(True)
    lg = (hr @ Wr.t())
    lp = torch.log_softmax(lg, -1).gather(-1, t[:, None]).squeeze(-1)
    lp.backward(gl)
    hd, Wd = h.to(cuda).requires_grad_(True), W.to(cuda).requires_grad_(True)
    lpd = ops.logprob(hd, Wd, t.to(cuda), chunk_rows=128)
    assert lpd.dtype == torch.float32
    err = (lpd.cpu() - lp.detach()).abs().max().item()
    assert err < 2e-3 * lp.detach().abs().max().item() + 2e-2, err
    lpd.backward(gl.to(cuda))
    cos = lambda a, b: torch.nn.functional.cosine_similarity(a.float().cpu().reshape(-1), b.float().reshape(-1), 0)
    assert 1 - cos(hd.grad, hr.grad) < 1e-2
    assert 1 - cos(Wd.grad, Wr.grad) < 1e-2


def test_sample_greedy_exact(cuda):
    g = gen(31)
    logits = torch.randn(64, 4096, generator=g).to(BF)
    logits[5, 17] = logits[5, 99] = 50.0  # tie: lowest index wins
    rng = torch.tensor([0, 0], dtype=torch.int64, device=cuda)
    tok, lp = ops.sample(logits.to(cuda), 1.0, 1, 123, rng)
    exp = logits.float().argmax(-1)
    assert torch.equal(tok.cpu(), exp)
    assert tok[5].item() == 17
    assert torch.all(lp.cpu() == 0)


@pytest.mark.parametrize("top_k,temp", [(None, 1.0), (20, 0.8), (3, 1.3)])
def test_sample_distribution(cuda, top_k, temp):
    V, draws = 512, 6000
    base = torch.randn(V, generator=gen(41)).to(BF) * 2
    logits = base[None].repeat(draws, 1)
    rng = torch.tensor([7, 99], dtype=torch.int64, device=cuda)
    tok, lp = ops.sample(logits.to(cuda), temp, top_k, 2024, rng)
    probs, logps = R.sample_distribution(base[None], temp, top_k)
    probs, logps = probs[0], logps[0]
    tok = tok.cpu()
    # log-prob of each sampled token equals the oracle's log_softmax at that token
    assert torch.allclose(lp.cpu(), logps[tok], atol=2e-5, rtol=1e-5)
    assert torch.all(probs[tok] > 0)  # never outside the top-k set
    counts = torch.bincount(tok, minlength=V).float()
    exp = probs * draws
    keep = exp > 5
    chi2 = (((counts - exp) ** 2) / exp.clamp_min(1e-9))[keep].sum().item()
    dof = int(keep.sum().item()) - 1
    assert chi2 < dof + 6 * math.sqrt(2 * max(dof, 1)) + 10, (chi2, dof)


def test_grpo_advantage_and_loss(cuda):
    g = gen(51)
    G, n_groups, S = 4, 6, 40
    N = G * n_groups
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    rewards[:G] = 1.0  # a constant group: advantage 0
    gids = torch.arange(n_groups).repeat_interleave(G)
    new = -torch.rand(N, S, generator=g) * 5
    old = new + 0.05 * torch.randn(N, S, generator=g)
    ref = new + 0.05 * torch.randn(N, S, generator=g)
    mask = torch.zeros(N, S)
    for i in range(N):
        L = int(torch.randint(1, S + 1, (1,), generator=g))
        mask[i, S - L:] = 1
    adv = ops.grpo_advantage(rewards.to(cuda), gids.to(cuda)).cpu()
    adv_ref = R.grpo_advantage(rewards, gids)
    assert torch.allclose(adv, adv_ref, rtol=1e-6, atol=1e-6)
    for beta, rp in [(0.0, None), (0.04, ref)]:
        loss_ref, grad_ref, _ = R.grpo_loss_and_grad(rewards, gids, new, old, mask, ref=rp, beta=beta)
        nd = new.to(cuda).requires_grad_(True)
        loss = ops.grpo_loss(nd, old.to(cuda), mask.to(cuda), rewards.to(cuda), gids.to(cuda),
                             None if rp is None else rp.to(cuda), 0.2, beta)
        loss.backward()
        assert abs(loss.item() - loss_ref.item()) <= 2e-3 * abs(loss_ref.item()) + 1e-6
        assert torch.allclose(nd.grad.cpu(), grad_ref, rtol=1e-4, atol=1e-7)


@pytest.mark.parametrize("split", [False, True])
def test_paged_decode_keyless_rows(cuda, split):
    """Rows of length <= 0 (decode-graph batch padding) read no keys and get zero output, with
    and without split-K; page 0, which they point at, holds NaN and must not leak into them."""
    g = gen(31)
    hq, hkv = 16, 8
    kc = torch.randn(6, 256, hkv, 128, generator=g).to(BF)
    vc = torch.randn(6, 256, hkv, 128, generator=g).to(BF)
    kc[0] = float("nan")
    vc[0] = float("nan")
    bt = torch.tensor([[1, 2], [0, 0], [3, 4], [0, 0]], dtype=torch.int32)
    ctx = torch.tensor([300, -1, 40, -1], dtype=torch.int32)  # key counts ctx + 1: 301, 0, 41, 0
    q = torch.randn(4, hq, 128, generator=g).to(BF)
    kw = dict(split_tokens=64, max_splits=8) if split else dict(split_tokens=512, max_splits=1)
    out = ops.paged_decode_attention(q.to(cuda), kc.to(cuda), vc.to(cuda), bt.to(cuda), ctx.to(cuda), 128 ** -0.5,
                                     **kw).cpu()
    ops.check_device_errors()
    live = [0, 2]
    ref = R.paged_decode(q[live], kc, vc, bt[live], ctx[live] + 1, 128 ** -0.5)
    close_bf16(out[live], ref, 2e-2)
    assert torch.equal(out[[1, 3]].float(), torch.zeros(2, hq, 128))


def test_paged_decode_grouped_rollout_scale(cuda):
    """Rollout-sized grouped decode (64 groups x 8 completions, page-aligned prompts shared per
    group, 1-600 own keys each: 512 shared-prefix CTAs and 4096 own-key CTAs) equals the plain
    paged decode kernel over the same pages; four back-to-back launches on one workspace give
    identical bits."""
    g = torch.Generator(device=cuda).manual_seed(123)
    gc = torch.Generator().manual_seed(123)
    hq, hkv, G, n_groups = 16, 8, 8, 64
    plen = [256 * int(x) for x in torch.randint(0, 3, (n_groups,), generator=gc)]
    own = torch.randint(1, 601, (G * n_groups,), generator=gc).tolist()
    n_pages = sum(p // 256 for p in plen) + sum(-(-o // 256) for o in own)
    kc = torch.randn(n_pages, 256, hkv, 128, device=cuda, generator=g).to(BF)
    vc = torch.randn(n_pages, 256, hkv, 128, device=cuda, generator=g).to(BF)
    perm = torch.randperm(n_pages, generator=gc).tolist()
    tables, lens, members = [], [], []
    for gi in range(n_groups):
        sh = [perm.pop() for _ in range(plen[gi] // 256)]
        row = []
        for m in range(G):
            b = gi * G + m
            row.append(b)
            tables.append(sh + [perm.pop() for _ in range(-(-own[b] // 256))])
            lens.append(plen[gi] + own[b])
        members.append(row)
    B = len(tables)
    bt = torch.full((B, max(len(t) for t in tables)), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    q = torch.randn(B, hq, 128, device=cuda, generator=g).to(BF)
    ctx = (torch.tensor(lens, dtype=torch.int32) - 1).to(cuda)
    bt = bt.to(cuda)
    ref = ops.paged_decode_attention(q, kc, vc, bt, ctx, 128 ** -0.5)
    plan = ops.grouped_decode_plan(B, hkv, max(plen), max(own))
    ws = ops.grouped_workspace(B, hq, 128, plan, cuda)
    kv_start = torch.tensor([plen[b // G] for b in range(B)], dtype=torch.int32).to(cuda)
    args = (q, kc, vc, bt, ctx, 128 ** -0.5, torch.tensor(members, dtype=torch.int32).to(cuda),
            torch.tensor(plen, dtype=torch.int32).to(cuda), kv_start, plan)
    first = ops.paged_decode_attention_grouped(*args, workspace=ws)
    close_bf16(first.cpu(), ref.cpu(), 2e-2)
    for _ in range(3):
        assert torch.equal(ops.paged_decode_attention_grouped(*args, workspace=ws), first)
    ops.check_device_errors()


@pytest.mark.parametrize("split", [64, 256])
def test_paged_decode_grouped_shared_prefix(cuda, split):
    """Groups sharing prompt pages: the grouped decode (shared keys once per group + own keys
    per sequence, then the split-K merge) equals plain attention over the concatenation of the
    shared keys [0, shared_len) and the own keys [kv_start, len).  Groups whose prompt ends
    inside a page leave a hole [shared_len, kv_start) filled with large garbage that must never
    be read; page-aligned groups use kv_start == shared_len.  A second call on the same workspace
    gives identical bits."""
    g = gen(77 + split)
    hq, hkv = 16, 8
    # (members, shared keys, own keys start on a fresh page?)
    groups = [(8, 512, False), (3, 256, False), (1, 0, False), (5, 768, False), (8, 0, False),
              (8, 300, True), (2, 17, True), (4, 511, True), (1, 700, True)]
    n_pages = 300
    kc = torch.randn(n_pages, 256, hkv, 128, generator=g).to(BF)
    vc = torch.randn(n_pages, 256, hkv, 128, generator=g).to(BF)
    perm = torch.randperm(n_pages, generator=g).tolist()
    tables, lens, members, shared, kv_start, keys = [], [], [], [], [], []
    for G_, sl, fresh in groups:
        sh_pages = [perm.pop() for _ in range(-(-sl // 256))]
        ks = len(sh_pages) * 256 if fresh else sl
        for idx, p in enumerate(sh_pages):  # garbage in the hole after the shared keys (never read)
            start = max(0, sl - idx * 256)
            kc[p, start:] = 1e4
            vc[p, start:] = 1e4
        row = []
        for _ in range(G_):
            n_own = int(torch.randint(1, 700, (1,), generator=g))
            own = [perm.pop() for _ in range(-(-(ks % 256 + n_own) // 256))]
            tab = sh_pages[:ks // 256] + own
            row.append(len(tables))
            tables.append(tab)
            lens.append(ks + n_own)
            kv_start.append(ks)
            # the keys this sequence attends to, as (page, slot) pairs in order
            keys.append([(sh_pages[t // 256], t % 256) for t in range(sl)]
                        + [(tab[t // 256], t % 256) for t in range(ks, ks + n_own)])
        members.append(row + [-1] * (8 - len(row)))
        shared.append(sl)
    B = len(tables)
    width = max(len(t) for t in tables)
    bt = torch.full((B, width), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    q = torch.randn(B, hq, 128, generator=g).to(BF)
    # oracle: gather each sequence's keys into a contiguous paged copy, plain decode attention
    n_ref = sum(-(-len(k) // 256) for k in keys)
    rk = torch.zeros(n_ref, 256, hkv, 128, dtype=BF)
    rv = torch.zeros_like(rk)
    rbt = torch.full((B, max(-(-len(k) // 256) for k in keys)), -1, dtype=torch.int32)
    nxt_page = 0
    for b, kl in enumerate(keys):
        for t, (p, j) in enumerate(kl):
            if t % 256 == 0:
                rbt[b, t // 256] = nxt_page
                nxt_page += 1
            rk[rbt[b, t // 256], t % 256] = kc[p, j]
            rv[rbt[b, t // 256], t % 256] = vc[p, j]
    ref = R.paged_decode(q, rk, rv, rbt, torch.tensor([len(k) for k in keys]), 128 ** -0.5)
    ctx = torch.tensor(lens, dtype=torch.int32) - 1
    plan = (split, -(-max(shared) // split) if max(shared) else 1,
            -(-max(L - s for L, s in zip(lens, kv_start)) // split))
    ws = ops.grouped_workspace(B, hq, 128, plan, cuda)
    args = (q.to(cuda), kc.to(cuda), vc.to(cuda), bt.to(cuda), ctx.to(cuda), 128 ** -0.5,
            torch.tensor(members, dtype=torch.int32).to(cuda), torch.tensor(shared, dtype=torch.int32).to(cuda),
            torch.tensor(kv_start, dtype=torch.int32).to(cuda), plan)
    out = ops.paged_decode_attention_grouped(*args, workspace=ws)
    close_bf16(out, ref, 2e-2)
    assert torch.equal(ops.paged_decode_attention_grouped(*args, workspace=ws), out)
    ops.check_device_errors()


@pytest.mark.parametrize("n,V", [(300, 151936), (100, 151936), (77, 1000), (40, 200)])
def test_lm_head_logprob_fused(cuda, n, V):
    """qb_lm_head_logprob (tcgen05 GEMM with the log-softmax and the gather in its epilogue) on the
    CTA-pair, 128x256 and 128x128 tile paths, V with and without a partial last tile: log-probs
    and log-sum-exp per element against the fp32 log_softmax of the same bf16 operands; the
    optional bf16 logits within one bf16 ulp; dest scatter with a skipped row; a target outside
    the vocabulary sets the token error bit and gives 0."""
    g = gen(61 + n)
    K = 1024
    h = torch.randn(n, K, generator=g).to(BF)
    W = (torch.randn(V, K, generator=g) * 0.05).to(BF)
    t = torch.randint(0, V, (n,), generator=g)
    ref_logits = h.float() @ W.float().t()
    ref_lse = torch.logsumexp(ref_logits, -1)
    ref = ref_logits.gather(-1, t[:, None]).squeeze(-1) - ref_lse
    dest = torch.arange(n, dtype=torch.int64) * 2
    dest[3] = -1
    out = torch.full((2 * n,), 7.0, device=cuda)
    lse = torch.empty(n, device=cuda)
    logits = torch.empty(n, V, dtype=BF, device=cuda)
    ops.lm_head_logprob(h.to(cuda), W.to(cuda), t.to(cuda), dest=dest.to(cuda), out=out, lse=lse, logits=logits)
    ops.check_device_errors()
    out = out.cpu()
    keep = torch.ones(n, dtype=torch.bool)
    keep[3] = False
    assert out[7].item() == 7.0 and out[6].item() == 7.0  # row 3 skipped (dest -1), odd slots untouched
    got = out[dest[keep]]
    assert ((got - ref[keep]).abs() <= 1e-4 * ref[keep].abs() + 1e-5).all(), (got - ref[keep]).abs().max()
    assert ((lse.cpu() - ref_lse).abs() <= 1e-5 * ref_lse.abs() + 1e-5).all()
    rl = ref_logits.to(BF).float()
    ulp = torch.exp2(torch.floor(torch.log2(rl.abs().clamp_min(2.0 ** -126))) - 7)
    # fp32 accumulation order differs from the CPU GEMM: near-zero logits move by ~1e-6 absolute
    assert ((logits.float().cpu() - rl).abs() <= ulp + 2e-5).all()
    # without the logits output, and with a bad target
    t2 = t.clone()
    t2[1] = V + 5
    out2, _ = ops.lm_head_logprob(h.to(cuda), W.to(cuda), t2.to(cuda))
    with pytest.raises(ops.NativeError):
        ops.check_device_errors()
    out2 = out2.cpu()
    assert out2[1].item() == 0.0
    assert torch.equal(out2[keep & (torch.arange(n) != 1)], out[dest[keep & (torch.arange(n) != 1)]])


@pytest.mark.parametrize("V,with_ref,given_total", [(1000, True, False), (151936, True, True), (151936, False, False)])
def test_grpo_logit_loss_single_pass(cuda, V, with_ref, given_total):
    """qb_grpo_logit_loss (config 1's pass in one read and one write of the logits, rows split over
    4-CTA clusters) against the oracle's fp32 autograd of log_softmax + gather -> advantages ->
    clipped surrogate (+ 0.04 k3 KL): log-probs per element, advantages, loss, and d loss / d
    logits per element within one bf16 ulp."""
    g = gen(71 + V)
    N, S = 8, 24
    logits = (torch.randn(N * S, V, generator=g) * 1.5).to(BF)
    tgt = torch.randint(0, V, (N * S,), generator=g)
    rewards = torch.bernoulli(torch.full((N,), 0.5), generator=g)
    gids = torch.arange(N) // 4
    lens = torch.randint(1, S + 1, (N,), generator=g)
    mask = (torch.arange(S)[None, :] < lens[:, None]).float()
    x = logits.float().requires_grad_(True)
    lp = torch.log_softmax(x, -1).gather(-1, tgt[:, None]).squeeze(-1).view(N, S)
    old = lp.detach() + 0.05 * torch.randn(N, S, generator=g)
    ref = lp.detach() + 0.05 * torch.randn(N, S, generator=g) if with_ref else None
    adv = R.grpo_advantage(rewards, gids)
    loss = R.ppo_loss(old, lp, adv[:, None] * mask, mask, 0.2, ref, 0.04 if with_ref else 0.0)
    loss.backward()
    work = logits.to(cuda)
    new_lp, loss3, adv_d = ops.grpo_logit_loss(
        work, tgt.to(cuda), rewards.to(cuda), gids.to(cuda), old.to(cuda), mask.to(cuda),
        ref_lp=None if ref is None else ref.to(cuda), mask_total=mask.sum().reshape(1).to(cuda) if given_total else None,
        beta=0.04 if with_ref else 0.0)
    ops.check_device_errors()
    assert ((new_lp.cpu() - lp.detach()).abs() <= 2e-5 * lp.detach().abs() + 1e-6).all()
    assert torch.allclose(adv_d.cpu(), adv, rtol=1e-6, atol=1e-6)
    assert abs(loss3[0].item() - loss.item()) <= 1e-5 * (abs(loss.item()) + 1e-3)
    gr = x.grad
    ulp = torch.exp2(torch.floor(torch.log2(gr.abs().clamp_min(2.0 ** -126))) - 7)
    d = (work.float().cpu() - gr).abs()
    assert (d <= ulp + 1e-10).all(), d.max().item()
    # a target outside the vocabulary: error bit, log-prob 0, zero gradient row
    tgt[5] = V + 3
    work = logits.to(cuda)
    new_lp, _, _ = ops.grpo_logit_loss(work, tgt.to(cuda), rewards.to(cuda), gids.to(cuda), old.to(cuda),
                                       mask.to(cuda))
    with pytest.raises(ops.NativeError):
        ops.check_device_errors()
    assert new_lp.view(-1)[5].item() == 0.0 and work[5].float().abs().max().item() == 0.0
