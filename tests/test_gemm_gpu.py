"""tcgen05 GEMM parity against a plain PyTorch fp32 reference of the same product.

Tolerance: the kernel accumulates in fp32 like the reference; only the bf16 output
rounding differs (<= 1 bf16 ulp, relative 2^-8), checked as 1e-2 of the output scale.
"""
import pytest
import torch

from qwen3_naive_inference_b200 import ops

pytestmark = pytest.mark.gpu


def ref(a, b):
    return a.float() @ b.float().t()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1, 128, 64), (7, 300, 128), (300, 1000, 1024),
                                   (512, 4096, 1024), (257, 6144, 1024), (513, 1024, 3072), (64, 151936, 1024),
                                   (1000, 2048, 4096),
                                   # 256x256 tiles on CTA pairs (>= one tile per SM pair), with M/N/K tails
                                   (2048, 2560, 512), (2000, 2600, 648), (8192, 6144, 1024),
                                   # split-K clusters of 4 (decode-step o_proj / down_proj) and of 2
                                   (512, 1024, 2048), (512, 1024, 3072), (300, 1000, 1024), (4, 256, 512),
                                   (809, 256, 512),
                                   # 128x192 tiles (one wave where 128x128 would need two), N and K tails
                                   (512, 6144, 1024), (500, 5000, 1000),
                                   # decode-like shapes with M, N and K tails
                                   (480, 4096, 1024), (300, 4000, 1000), (257, 6100, 1000),
                                   # pairs below one tile per SM pair (long K), with tails
                                   (1000, 1000, 20000), (4096, 1024, 30000)])
def test_gemm_bf16_out(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    c = ops.gemm(a, b)
    r = ref(a, b)
    err = (c.float() - r).abs().max().item()
    assert err <= 1e-2 * r.abs().max().item() + 1e-3, err
    ops.check_device_errors()


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("M,N,K", [(200, 384, 512), (2000, 2600, 648), (513, 1024, 3072), (500, 5000, 1000),
                                   (512, 4096, 1024)])
def test_gemm_fp32_out_and_accumulate(cuda, mode, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(mode)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, device=cuda, generator=g).to(torch.bfloat16)
    c0 = torch.randn(M, N, device=cuda, generator=g)
    c = c0.clone()
    ops.gemm(a, b, out=c, mode=mode)
    r = ref(a, b) + (c0 if mode == 2 else 0)
    assert torch.allclose(c, r, rtol=1e-4, atol=1e-3)


def test_gemm_strided_operands(cuda):
    """Row pitch larger than K (views into wider buffers)."""
    g = torch.Generator(device=cuda).manual_seed(5)
    A = torch.randn(96, 2048, device=cuda, generator=g).to(torch.bfloat16)
    B = torch.randn(320, 1536, device=cuda, generator=g).to(torch.bfloat16)
    a, b = A[:, 512:1536], B[:, :1024]
    c = ops.gemm(a, b)
    r = ref(a, b)
    assert (c.float() - r).abs().max().item() <= 1e-2 * r.abs().max().item()


def test_gemm_split_k_deterministic(cuda):
    """Split-K partials are summed in a fixed order: repeated launches give identical bits."""
    g = torch.Generator(device=cuda).manual_seed(11)
    a = torch.randn(512, 3072, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(1024, 3072, device=cuda, generator=g).to(torch.bfloat16)
    first = ops.gemm(a, b)
    for _ in range(20):
        assert torch.equal(ops.gemm(a, b), first)
    ops.check_device_errors()


def test_gemm_repeated_calls_stable(cuda):
    """Persistent kernel reuse: many launches, same answer every time."""
    g = torch.Generator(device=cuda).manual_seed(9)
    a = torch.randn(700, 1024, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(3000, 1024, device=cuda, generator=g).to(torch.bfloat16)
    first = ops.gemm(a, b)
    for _ in range(20):
        assert torch.equal(ops.gemm(a, b), first)


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (296, 1024, 776), (1000, 384, 4096), (64, 151936, 200),
                                   (2048, 2560, 512), (2000, 2600, 648), (400, 6000, 200), (512, 4096, 1024),
                                   (304, 4000, 520)])
def test_gemm_mn_major_operands(cuda, a_mn, b_mn, M, N, K):
    """Backward layouts: A stored [K, M] and/or B stored [K, N]; K need not be a multiple of 64
    (row pitches stay multiples of 8 elements, the TMA rule)."""
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    a_st = a.t().contiguous() if a_mn else a
    b_st = b.t().contiguous() if b_mn else b
    c = ops.gemm_ex(a_st, a_mn, b_st, b_mn)
    r = ref(a, b)
    err = (c.float() - r).abs().max().item()
    assert err <= 1e-2 * r.abs().max().item() + 1e-3, err
    acc = torch.randn(M, N, device=cuda, generator=g)
    out = acc.clone()
    ops.gemm_ex(a_st, a_mn, b_st, b_mn, out=out, mode=2)
    assert torch.allclose(out, acc + r, rtol=1e-3, atol=2e-2)


@pytest.mark.parametrize("M,N,K,b_mn,want", [
    (8192, 6144, 1024, False, ("pair", 256, 1)),   # training shapes: 256 x 256 tiles fill the SM pairs
    (512, 4096, 1024, False, ("single", 128, 1)),  # decode qkv_proj: one wave of 128 x 128 tiles
    (512, 6144, 1024, False, ("single", 192, 1)),  # decode gate_up_proj: one wave of 128 x 192
    (512, 1024, 2048, False, ("single", 128, 4)),  # decode o_proj: split-K over 4-CTA clusters
    (512, 1024, 3072, False, ("single", 128, 4)),  # decode down_proj
    (7, 300, 128, False, ("single", 128, 1)),
    # long K, too few 256 x 256 tiles to fill the SM pairs: pairs anyway (half the operand bytes
    # per MMA cycle): the lm_head backward dh = dlogits . W and a layer's weight gradient
    (4096, 1024, 151936, True, ("pair", 256, 1)),
    (4096, 1024, 32768, True, ("pair", 256, 1)),
])
def test_gemm_plan(cuda, M, N, K, b_mn, want):
    """The layouts the cases above rely on are the ones the dispatcher picks."""
    assert ops.gemm_plan(M, N, K, b_mn) == want


@pytest.mark.parametrize("M,N,K,want", [
    (1024, 2048, 32768, ("pair", 256, 2)),  # o_proj weight gradient: 32 pair tiles, K split 2 ways
    (6144, 1024, 32768, ("pair", 256, 3)),  # gate_up: 96 tiles would take two waves of 74 pairs
    (1024, 3072, 32768, ("pair", 256, 3)),  # down_proj
    (4096, 1024, 32768, ("pair", 256, 1)),  # qkv: 64 tiles, no split saves a wave
    (151936, 1024, 4096, ("pair", 256, 1)),  # lm_head: a huge C, a 2% saving is not worth atomics
])
def test_gemm_plan_weight_gradients(cuda, M, N, K, want):
    """Mode 2 (C +=) may split K over pairs; the plain modes never do."""
    assert ops.gemm_plan(M, N, K, True, mode=2) == want
    assert ops.gemm_plan(M, N, K, True, mode=0)[2] == 1


@pytest.mark.parametrize("M,N,K", [(1024, 2048, 16384), (1000, 1000, 20000), (600, 3000, 9000)])
def test_gemm_accumulate_split_over_pairs(cuda, M, N, K):
    """C += A.B^T with K split over CTA pairs (atomic adds): backward layouts, M/N/K tails."""
    g = torch.Generator(device=cuda).manual_seed(M + N)
    a = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(N, K, device=cuda, generator=g) * 0.05).to(torch.bfloat16)
    assert ops.gemm_plan(M, N, K, True, mode=2)[2] > 1
    acc = torch.randn(M, N, device=cuda, generator=g)
    out = acc.clone()
    ops.gemm_ex(a.t().contiguous(), True, b.t().contiguous(), True, out=out, mode=2)
    ref = acc + a.float() @ b.float().t()
    assert torch.allclose(out, ref, rtol=1e-3, atol=2e-2)
    ops.check_device_errors()


def test_gemm_k_tail_k_major(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    a = torch.randn(200, 100, device=cuda, generator=g).to(torch.bfloat16)[:, :72]
    b = torch.randn(300, 100, device=cuda, generator=g).to(torch.bfloat16)[:, :72]
    c = ops.gemm_ex(a.contiguous(), False, b.contiguous(), False)
    r = ref(a, b)
    assert (c.float() - r).abs().max().item() <= 1e-2 * r.abs().max().item()


@pytest.mark.parametrize("M,I,K", [
    (512, 3072, 1024),   # decode step: single-CTA tiles of 96 gate + 96 up columns, one wave
    (300, 3000, 1000),   # M, I (not a multiple of the half tile) and K tails
    (2048, 3072, 1024),  # 256-row tiles on CTA pairs (128 gate + 128 up columns)
    (1000, 3072, 520),   # pairs with an M tail and a K tail
    (7, 200, 64),
])
def test_gemm_swiglu_matches_unfused(cuda, M, I, K):
    """The gate_up GEMM with SwiGLU in its epilogue gives the bits of the gate_up GEMM followed by
    the SwiGLU kernel, and its optional gate_up output the bits of the plain GEMM."""
    g = torch.Generator(device=cuda).manual_seed(M + I + K)
    x = torch.randn(M, K, device=cuda, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * I, K, device=cuda, generator=g) * K ** -0.5).to(torch.bfloat16)
    gu_ref = ops.gemm(x, w)
    h_ref = ops.silu_mul(gu_ref)
    h, gu = ops._gemm_swiglu(x, w, True, False)
    assert torch.equal(gu, gu_ref)
    assert torch.equal(h, h_ref)
    h2, none = ops._gemm_swiglu(x, w, False, True)
    assert none is None and torch.equal(h2, h_ref)
    ops.check_device_errors()


def test_swiglu_linear_autograd(cuda):
    """Forward and gradients of the fused op equal those of linear + silu_mul."""
    g = torch.Generator(device=cuda).manual_seed(3)
    x0 = torch.randn(600, 1024, device=cuda, generator=g).to(torch.bfloat16)
    w0 = (torch.randn(2 * 3072, 1024, device=cuda, generator=g) * 0.03).to(torch.bfloat16)
    d = torch.randn(600, 3072, device=cuda, generator=g).to(torch.bfloat16)
    outs = []
    for fused in (False, True):
        x = x0.clone().requires_grad_(True)
        w = w0.clone().requires_grad_(True)
        h = ops.swiglu_linear(x, w) if fused else ops.silu_mul(ops.linear(x, w))
        h.backward(d)
        outs.append((h.detach(), x.grad, w.grad))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
