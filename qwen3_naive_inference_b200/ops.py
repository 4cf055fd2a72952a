"""Torch-facing wrappers over the C ABI in ``include/qwen3b200.h``.

Each function validates dtype/shape/contiguity/device, then calls one
``qb_*`` entry point on the current CUDA stream with raw pointers.  Tensors
must live on a CUDA device: there is no CPU fallback, and a missing shared
library raises :class:`NativeError`.

Training-path ops are ``torch.autograd.Function``s whose backward is a CUDA
kernel of this library as well (RMSNorm, QK-Norm+RoPE, attention, SwiGLU,
embedding).  Dense projections go through :func:`linear`.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from . import _lib
from ._lib import NativeError, check

__all__ = [
    "NativeError", "lib", "stream_ptr", "err_flag", "check_device_errors", "embedding", "rmsnorm",
    "add_rmsnorm", "qk_norm_rope", "qk_norm_rope_store", "qk_norm_rope_attention", "qkv_norm_rope_store",
    "gemm_qk_norm_rope", "qkv_attention", "attention_packed", "attention_paged_prefill",
    "paged_decode_attention", "silu_mul", "add", "linear", "swiglu_linear", "logprob", "sample", "grpo_advantage",
    "grpo_loss", "mask_sum", "build_tiles", "decode_split_plan", "lm_head_logprob",
    "grpo_logit_loss",
]

BF16 = torch.bfloat16


def lib():
    return _lib.load()


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t) -> int:
    return 0 if t is None else t.data_ptr()


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise NativeError("qwen3_naive_inference_b200 ops need CUDA tensors (no CPU fallback)")


_ERR: dict[int, torch.Tensor] = {}


def err_flag(device=None) -> torch.Tensor:
    """Device int32 error word shared by all launches on ``device``."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    t = _ERR.get(dev.index)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=dev)
        _ERR[dev.index] = t
    return t


_DEVERR_NAMES = {1: "page id out of range", 2: "slot out of range", 4: "token id out of range",
                 8: "inconsistent sequence lengths / positions", 16: "bounded wait timed out"}


def check_device_errors(device=None) -> None:
    """Reads (synchronously) and clears the device error word; raises if set."""
    f = err_flag(device)
    v = int(f.item())
    if v:
        f.zero_()
        names = [n for b, n in _DEVERR_NAMES.items() if v & b]
        raise NativeError(f"device-side bounds check failed: {', '.join(names)} (bits {v:#x})")


# ---------------------------------------------------------------- embedding
class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight):
        n = ids.numel()
        out = torch.empty(n, weight.shape[1], dtype=weight.dtype, device=weight.device)
        check(lib().qb_embedding_fwd(_p(ids), n, _p(weight), weight.shape[0], weight.shape[1], _p(out),
                                     _p(err_flag()), stream_ptr()), "qb_embedding_fwd")
        ctx.save_for_backward(ids)
        ctx.shape = weight.shape
        ctx.grad32 = grad32_target(weight)
        return out

    @staticmethod
    def backward(ctx, g):
        (ids,) = ctx.saved_tensors
        g = g.contiguous()
        direct = ctx.grad32  # fp32 accumulator of the table's gradient (see grad32_target)
        acc = direct if direct is not None else torch.zeros(ctx.shape, dtype=torch.float32, device=g.device)
        check(lib().qb_embedding_bwd(_p(ids), ids.numel(), _p(g), ctx.shape[0], ctx.shape[1], _p(acc),
                                     _p(err_flag()), stream_ptr()), "qb_embedding_bwd")
        return None, (None if direct is not None else _to_bf16(acc))


def embedding(ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``weight[ids]`` for int64 ``ids`` (any shape, flattened) -> [n, hidden] bf16."""
    _cuda(ids, weight)
    ids = ids.reshape(-1)
    if ids.dtype != torch.long:
        ids = ids.long()
    return _Embedding.apply(ids.contiguous(), weight)


def grad32_target(param):
    """The fp32 buffer a parameter's gradient accumulates into during a fused training pass
    (attached by qwen3_grpo_train.GradBuffer), or None: backward kernels then add their products
    straight into it (GEMM mode 2) instead of returning a bf16 gradient to autograd."""
    return getattr(param, "_qb_grad32", None)


def _to_bf16(acc: torch.Tensor) -> torch.Tensor:
    out = torch.empty(acc.shape, dtype=BF16, device=acc.device)
    check(lib().qb_f32_to_bf16(_p(acc), _p(out), acc.numel(), stream_ptr()), "qb_f32_to_bf16")
    return out


# ---------------------------------------------------------------- RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        rows, cols = x.numel() // x.shape[-1], x.shape[-1]
        y = torch.empty_like(x)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        check(lib().qb_rmsnorm_fwd(_p(x), _p(w), _p(y), _p(rstd), rows, cols, eps, stream_ptr()),
              "qb_rmsnorm_fwd")
        ctx.save_for_backward(x, w, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        rows, cols = x.numel() // x.shape[-1], x.shape[-1]
        dx = torch.empty_like(x)
        dw = torch.zeros(cols, dtype=torch.float32, device=x.device)
        check(lib().qb_rmsnorm_bwd(_p(dy), _p(x), _p(w), _p(rstd), _p(dx), _p(dw), rows, cols, stream_ptr()),
              "qb_rmsnorm_bwd")
        return dx, _to_bf16(dw).to(w.dtype), None


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    _cuda(x, w)
    x = x.contiguous()
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        return _RMSNorm.apply(x, w, eps)
    rows, cols = x.numel() // x.shape[-1], x.shape[-1]
    y = torch.empty_like(x)
    check(lib().qb_rmsnorm_fwd(_p(x), _p(w), _p(y), 0, rows, cols, eps, stream_ptr()), "qb_rmsnorm_fwd")
    return y


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """Fused ``residual += x; y = rmsnorm(residual)`` (inference); returns (y, residual)."""
    _cuda(x, residual, w)
    x = x.contiguous()
    residual = residual.contiguous().clone() if not residual.is_contiguous() else residual
    rows, cols = x.numel() // x.shape[-1], x.shape[-1]
    y = torch.empty_like(x)
    check(lib().qb_add_rmsnorm_fwd(_p(x), _p(residual), _p(w), _p(y), rows, cols, eps, stream_ptr()),
          "qb_add_rmsnorm_fwd")
    return y, residual


# ---------------------------------------------------------------- QK-Norm + RoPE
def _qk_norm_rope_fwd(qkv, positions, cos_sin, qw, kw, eps, hq, hkv, save=True):
    """Rotated copy of ``qkv`` plus (with ``save``) the per-head rstd the backward needs."""
    T, ld = qkv.shape
    out = torch.empty_like(qkv)
    q_rstd = torch.empty(T, hq, dtype=torch.float32, device=qkv.device) if save else None
    k_rstd = torch.empty(T, hkv, dtype=torch.float32, device=qkv.device) if save else None
    check(lib().qb_qk_norm_rope_fwd(_p(qkv), T, ld, hq, hkv, 128, _p(positions), _p(cos_sin),
                                    cos_sin.shape[0], _p(qw), _p(kw), eps, _p(out), ld, 0, 0, 0, 0, 0,
                                    _p(q_rstd) if save else 0, _p(k_rstd) if save else 0, _p(err_flag()),
                                    stream_ptr()),
          "qb_qk_norm_rope_fwd")
    return out, q_rstd, k_rstd


def _qk_norm_rope_bwd(dout, dqkv, qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd, hq, hkv, rope_grad):
    """Writes the projection gradient into ``dqkv`` (which may be ``dout`` itself: the v columns
    then stay in place) and returns the norm-weight gradients (None without rope_grad)."""
    T, ld = qkv.shape
    dqw = torch.zeros(128, dtype=torch.float32, device=qkv.device)
    dkw = torch.zeros(128, dtype=torch.float32, device=qkv.device)
    check(lib().qb_qk_norm_rope_bwd(_p(dout), _p(qkv), T, ld, hq, hkv, 128, _p(positions), _p(cos_sin),
                                    cos_sin.shape[0], _p(qw), _p(kw), _p(q_rstd), _p(k_rstd),
                                    1 if rope_grad else 0, _p(dqkv), _p(dqw), _p(dkw), _p(err_flag()),
                                    stream_ptr()), "qb_qk_norm_rope_bwd")
    if not rope_grad:  # the reference's Triton RoPE leaves q_norm/k_norm without a grad
        return None, None
    return _to_bf16(dqw).to(qw.dtype), _to_bf16(dkw).to(kw.dtype)


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, positions, cos_sin, qw, kw, eps, hq, hkv, rope_grad):
        out, q_rstd, k_rstd = _qk_norm_rope_fwd(qkv, positions, cos_sin, qw, kw, eps, hq, hkv)
        ctx.save_for_backward(qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd)
        ctx.cfg = (hq, hkv, rope_grad)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd = ctx.saved_tensors
        hq, hkv, rope_grad = ctx.cfg
        dout = dout.contiguous()
        dqkv = torch.empty_like(qkv)  # the incoming gradient may be the caller's tensor: not in place
        dqw, dkw = _qk_norm_rope_bwd(dout, dqkv, qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd, hq, hkv,
                                     rope_grad)
        return dqkv, None, None, dqw, dkw, None, None, None, None


def qk_norm_rope(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, rope_grad=True):
    """[T, (hq+2hkv)*128] projection -> same layout with normed+rotated q, k and copied v."""
    _cuda(qkv, positions, cos_sin)
    qkv = qkv.contiguous()
    if torch.is_grad_enabled() and (qkv.requires_grad or q_norm_w.requires_grad):
        return _QKNormRope.apply(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, rope_grad)
    T, ld = qkv.shape
    out = torch.empty_like(qkv)
    check(lib().qb_qk_norm_rope_fwd(_p(qkv), T, ld, hq, hkv, 128, _p(positions), _p(cos_sin), cos_sin.shape[0],
                                    _p(q_norm_w), _p(k_norm_w), eps, _p(out), ld, 0, 0, 0, 0, 0, 0, 0,
                                    _p(err_flag()), stream_ptr()), "qb_qk_norm_rope_fwd")
    return out


def qk_norm_rope_store(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, k_cache, v_cache,
                       slot_mapping):
    """Paged path: returns rotated q [T, hq, 128]; rotated k and v go to the cache rows slot_mapping."""
    _cuda(qkv, positions, cos_sin, k_cache, v_cache, slot_mapping)
    T, ld = qkv.shape
    q = torch.empty(T, hq, 128, dtype=qkv.dtype, device=qkv.device)
    num_slots = k_cache.numel() // (hkv * 128)
    check(lib().qb_qk_norm_rope_fwd(_p(qkv), T, ld, hq, hkv, 128, _p(positions), _p(cos_sin), cos_sin.shape[0],
                                    _p(q_norm_w), _p(k_norm_w), eps, 0, 0, _p(q), _p(k_cache), _p(v_cache),
                                    _p(slot_mapping), num_slots, 0, 0, _p(err_flag()), stream_ptr()),
          "qb_qk_norm_rope_fwd")
    return q


def gemm_qk_norm_rope(x, w, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, *, out=None, raw=None,
                      q_out=None, k_cache=None, v_cache=None, slot_mapping=None, q_rstd=None, k_rstd=None,
                      b_static=False):
    """``qb_gemm_qk_norm_rope``: the qkv projection x [T, K] . w^T with QK-norm, RoPE and the paged
    K/V store in the GEMM's epilogue (same bits as linear + qk_norm_rope[_store]).  Writes the given
    outputs; returns nothing."""
    _cuda(x, w, positions, cos_sin)
    x2, w2 = _gemm_operand(x), _gemm_operand(w)
    T, K = x2.shape
    num_slots = 0 if k_cache is None else k_cache.numel() // (hkv * 128)
    opt = lambda t: 0 if t is None else _p(t)  # noqa: E731
    check(lib().qb_gemm_qk_norm_rope(_p(x2), x2.stride(0), _p(w2), w2.stride(0), T, hq, hkv, K, _p(positions),
                                     _p(cos_sin), cos_sin.shape[0], _p(q_norm_w), _p(k_norm_w), eps, opt(out),
                                     0 if out is None else out.stride(0), opt(raw), 0 if raw is None else raw.stride(0),
                                     opt(q_out), opt(k_cache), opt(v_cache), opt(slot_mapping), num_slots, opt(q_rstd),
                                     opt(k_rstd), QB_GEMM_B_STATIC if b_static else 0, _p(err_flag()), stream_ptr()),
          "qb_gemm_qk_norm_rope")


def qkv_norm_rope_store(x, w, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, k_cache, v_cache,
                        slot_mapping):
    """Paged path in one GEMM: ``qk_norm_rope_store(linear(x, w), ...)`` -- returns rotated q
    [T, hq, 128]; rotated k and v go to the cache rows slot_mapping (inference only)."""
    q = torch.empty(x.shape[0], hq, 128, dtype=BF16, device=x.device)
    gemm_qk_norm_rope(x, w, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, q_out=q, k_cache=k_cache,
                      v_cache=v_cache, slot_mapping=slot_mapping, b_static=isinstance(w, torch.nn.Parameter))
    return q


# ---------------------------------------------------------------- attention
def build_tiles(lengths, block: int = 64) -> np.ndarray:
    """Host list of (sequence, first row) pairs covering each sequence in 64-row tiles."""
    lens = np.asarray(lengths, dtype=np.int64)
    n = (lens + block - 1) // block
    seq = np.repeat(np.arange(len(lens), dtype=np.int32), n)
    start = (np.arange(int(n.sum()), dtype=np.int64) - np.repeat(np.cumsum(n) - n, n)) * block
    return np.stack([seq, start.astype(np.int32)], axis=1).astype(np.int32).reshape(-1)


def _attn_packed_fwd(qkv, cu, tiles, hq, hkv, scale):
    T, ld = qkv.shape
    out = torch.empty(T, hq * 128, dtype=qkv.dtype, device=qkv.device)
    lse = torch.empty(hq, T, dtype=torch.float32, device=qkv.device)
    base = qkv.data_ptr()
    k_ptr = base + hq * 128 * 2
    v_ptr = base + (hq + hkv) * 128 * 2
    check(lib().qb_attn_varlen_fwd(base, ld, k_ptr, v_ptr, ld, 0, 0, 0, 256, _p(cu), _p(cu), cu.numel() - 1,
                                   _p(tiles), tiles.numel() // 2, 0, hq, hkv, 128, scale, _p(out), hq * 128,
                                   _p(lse), T, _p(err_flag()), stream_ptr()), "qb_attn_varlen_fwd")
    return out, lse


def _attn_packed_bwd(dout, qkv, cu, tiles, out, lse, hq, hkv, scale):
    """Fresh [T, ld] gradient w.r.t. the packed (rotated) q | k | v columns."""
    T, ld = qkv.shape
    dqkv = torch.empty_like(qkv)
    delta = torch.empty(hq, T, dtype=torch.float32, device=qkv.device)
    b = qkv.data_ptr()
    db = dqkv.data_ptr()
    koff, voff = hq * 128 * 2, (hq + hkv) * 128 * 2
    check(lib().qb_attn_varlen_bwd(b, b + koff, b + voff, ld, _p(out), _p(dout), hq * 128, _p(lse), _p(cu),
                                   cu.numel() - 1, _p(tiles), tiles.numel() // 2, hq, hkv, 128, scale, T,
                                   _p(delta), db, db + koff, db + voff, _p(err_flag()), stream_ptr()),
          "qb_attn_varlen_bwd")
    return dqkv


class _AttnPacked(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, cu, tiles, hq, hkv, scale):
        out, lse = _attn_packed_fwd(qkv, cu, tiles, hq, hkv, scale)
        ctx.save_for_backward(qkv, cu, tiles, out, lse)
        ctx.cfg = (hq, hkv, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, cu, tiles, out, lse = ctx.saved_tensors
        hq, hkv, scale = ctx.cfg
        return _attn_packed_bwd(dout.contiguous(), qkv, cu, tiles, out, lse, hq, hkv, scale), \
            None, None, None, None, None


class _QKNormRopeAttn(torch.autograd.Function):
    """QK-norm + RoPE followed by packed causal attention as one autograd node, so the attention
    backward's fresh gradient buffer takes the QK-norm backward in place (its v columns are
    already final and are not copied)."""

    @staticmethod
    def forward(ctx, qkv, positions, cos_sin, qw, kw, eps, hq, hkv, rope_grad, cu, tiles, scale):
        rot, q_rstd, k_rstd = _qk_norm_rope_fwd(qkv, positions, cos_sin, qw, kw, eps, hq, hkv)
        out, lse = _attn_packed_fwd(rot, cu, tiles, hq, hkv, scale)
        ctx.save_for_backward(qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd, rot, cu, tiles, out, lse)
        ctx.cfg = (hq, hkv, rope_grad, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd, rot, cu, tiles, out, lse = ctx.saved_tensors
        hq, hkv, rope_grad, scale = ctx.cfg
        d = _attn_packed_bwd(dout.contiguous(), rot, cu, tiles, out, lse, hq, hkv, scale)
        dqw, dkw = _qk_norm_rope_bwd(d, d, qkv, positions, cos_sin, qw, kw, q_rstd, k_rstd, hq, hkv, rope_grad)
        return d, None, None, dqw, dkw, None, None, None, None, None, None, None


def qk_norm_rope_attention(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, cu_seqlens, tiles, hq, hkv, scale,
                           rope_grad=True):
    """``attention_packed(qk_norm_rope(qkv, ...), ...)`` with one fused backward (training path)."""
    _cuda(qkv, positions, cos_sin, cu_seqlens, tiles)
    qkv = qkv.contiguous()
    if torch.is_grad_enabled() and (qkv.requires_grad or q_norm_w.requires_grad):
        return _QKNormRopeAttn.apply(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, rope_grad,
                                     cu_seqlens, tiles, scale)
    rot, _, _ = _qk_norm_rope_fwd(qkv, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, save=False)
    return _attn_packed_fwd(rot, cu_seqlens, tiles, hq, hkv, scale)[0]


class _QkvNormRopeAttn(torch.autograd.Function):
    """qkv projection -> QK-norm + RoPE -> packed causal attention as one autograd node: the
    forward is one GEMM with QK-norm and RoPE in its epilogue (which also keeps the bf16 projection
    and the rstd for the backward) and the attention kernel; the backward is the attention
    backward, the QK-norm backward in place in its gradient buffer, then dX and dW of the
    projection."""

    @staticmethod
    def forward(ctx, x2, w, grad32, positions, cos_sin, qw, kw, eps, hq, hkv, rope_grad, cu, tiles, scale):
        T = x2.shape[0]
        N = (hq + 2 * hkv) * 128
        raw = torch.empty(T, N, dtype=BF16, device=x2.device)
        rot = torch.empty(T, N, dtype=BF16, device=x2.device)
        q_rstd = torch.empty(T, hq, dtype=torch.float32, device=x2.device)
        k_rstd = torch.empty(T, hkv, dtype=torch.float32, device=x2.device)
        gemm_qk_norm_rope(x2, w, positions, cos_sin, qw, kw, eps, hq, hkv, out=rot, raw=raw, q_rstd=q_rstd,
                          k_rstd=k_rstd)
        out, lse = _attn_packed_fwd(rot, cu, tiles, hq, hkv, scale)
        ctx.save_for_backward(x2, w, raw, positions, cos_sin, qw, kw, q_rstd, k_rstd, rot, cu, tiles, out, lse)
        ctx.cfg = (hq, hkv, rope_grad, scale)
        ctx.grad32 = grad32
        return out

    @staticmethod
    def backward(ctx, dout):
        x2, w, raw, positions, cos_sin, qw, kw, q_rstd, k_rstd, rot, cu, tiles, out, lse = ctx.saved_tensors
        hq, hkv, rope_grad, scale = ctx.cfg
        d = _attn_packed_bwd(dout.contiguous(), rot, cu, tiles, out, lse, hq, hkv, scale)
        dqw, dkw = _qk_norm_rope_bwd(d, d, raw, positions, cos_sin, qw, kw, q_rstd, k_rstd, hq, hkv, rope_grad)
        dx = gemm_ex(d, False, w, True) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            if ctx.grad32 is not None:
                gemm_ex(d, True, x2, True, out=ctx.grad32, mode=2)
            else:
                dw = gemm_ex(d, True, x2, True)
        return dx, dw, None, None, None, dqw, dkw, None, None, None, None, None, None, None


def qkv_attention(x, w, positions, cos_sin, q_norm_w, k_norm_w, eps, cu_seqlens, tiles, hq, hkv, scale,
                  rope_grad=True):
    """``attention_packed(qk_norm_rope(linear(x, w), ...), ...)`` with the projection, QK-norm and
    RoPE in one GEMM; returns [T, hq * 128].  Same bits as the unfused path; faster for small T
    only (measured at T = 4096: 75 us against 35 + 15 us for the GEMM and the standalone kernel,
    whose epilogue threads each own a token row), so the model's training path does not use it."""
    _cuda(x, w, positions, cos_sin, cu_seqlens, tiles)
    x2, w2 = _gemm_operand(x), _gemm_operand(w)
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad or q_norm_w.requires_grad):
        return _QkvNormRopeAttn.apply(x2, w2, grad32_target(w) if w.requires_grad else None, positions, cos_sin,
                                      q_norm_w, k_norm_w, eps, hq, hkv, rope_grad, cu_seqlens, tiles, scale)
    rot = torch.empty(x2.shape[0], (hq + 2 * hkv) * 128, dtype=BF16, device=x2.device)
    gemm_qk_norm_rope(x2, w2, positions, cos_sin, q_norm_w, k_norm_w, eps, hq, hkv, out=rot,
                      b_static=isinstance(w, torch.nn.Parameter))
    return _attn_packed_fwd(rot, cu_seqlens, tiles, hq, hkv, scale)[0]


def attention_packed(qkv_rot, cu_seqlens, tiles, hq, hkv, scale):
    """Causal attention over packed sequences (training path).

    qkv_rot: [T, (hq+2hkv)*128] with rotated q/k and v; cu_seqlens int32 [B+1];
    tiles: int32 from :func:`build_tiles` on the sequence lengths.  Returns [T, hq*128].
    """
    _cuda(qkv_rot, cu_seqlens, tiles)
    return _AttnPacked.apply(qkv_rot.contiguous(), cu_seqlens, tiles, hq, hkv, scale)


def attention_paged_prefill(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, block_tables,
                            scale, tiles=None, hkv=None, out=None):
    """flash_attn_varlen_func(q, k_cache, v_cache, ..., causal=True, block_table=) equivalent.

    q: [Tq, hq, 128]; caches [num_blocks, 256, hkv, 128]; returns [Tq, hq, 128] (``out`` if given).
    """
    _cuda(q, k_cache, v_cache, cu_seqlens_q, cu_seqlens_k, block_tables)
    Tq, hq, D = q.shape
    num_blocks, page, hkv_c, _ = k_cache.shape
    if out is None:
        out = torch.empty_like(q)
    batch = cu_seqlens_q.numel() - 1
    tps = (int(max_seqlen_q) + 63) // 64
    n_tiles = 0 if tiles is None else tiles.numel() // 2
    check(lib().qb_attn_varlen_fwd(_p(q), hq * D, _p(k_cache), _p(v_cache), 0, _p(block_tables),
                                   block_tables.stride(0), num_blocks, page, _p(cu_seqlens_q), _p(cu_seqlens_k),
                                   batch, _p(tiles), n_tiles, tps, hq, hkv_c, D, scale, _p(out), hq * D, 0, Tq,
                                   _p(err_flag()), stream_ptr()), "qb_attn_varlen_fwd")
    return out


def decode_split_plan(batch: int, hkv: int, max_ctx: int, sm_count: int = 148) -> tuple[int, int]:
    """(split_tokens, max_splits) for the paged decode kernel: enough CTAs to cover the GPU
    at least twice, at most one split per 64 tokens."""
    want = max(1, math.ceil(4 * sm_count / max(1, batch * hkv)))
    max_splits = max(1, min(want, math.ceil(max_ctx / 64)))
    split_tokens = math.ceil(math.ceil(max_ctx / max_splits) / 64) * 64
    max_splits = math.ceil(max_ctx / split_tokens)
    return split_tokens, max_splits


def paged_decode_attention(q, k_cache, v_cache, block_tables, seqlens, scale, seqlen_add=1,
                           split_tokens=None, max_splits=None, workspace=None, max_ctx=None):
    """flash_attn_with_kvcache(q[:,None], k_cache, v_cache, cache_seqlens=seqlens+seqlen_add,
    block_table=block_tables, causal=True) equivalent; q [B, hq, 128] -> [B, hq, 128]."""
    _cuda(q, k_cache, v_cache, block_tables, seqlens)
    B, hq, D = q.shape
    num_blocks, page, hkv, _ = k_cache.shape
    if split_tokens is None:
        if max_ctx is None:
            max_ctx = block_tables.shape[1] * page
        split_tokens, max_splits = decode_split_plan(B, hkv, max_ctx)
    out = torch.empty_like(q)
    if max_splits > 1 and workspace is None:
        nbytes = lib().qb_paged_decode_workspace_bytes(B, hq, D, max_splits)
        workspace = torch.empty(nbytes // 4, dtype=torch.float32, device=q.device)
    check(lib().qb_paged_decode_attn(_p(q), _p(k_cache), _p(v_cache), num_blocks, page, _p(block_tables),
                                     block_tables.stride(0), _p(seqlens), seqlen_add, B, hq, hkv, D, scale,
                                     split_tokens, max_splits, _p(workspace) if max_splits > 1 else 0, _p(out),
                                     _p(err_flag()), stream_ptr()), "qb_paged_decode_attn",
          kernels=2 if max_splits > 1 else 1)
    return out


def grouped_decode_plan(batch, hkv, max_shared, max_own, sm_count=148):
    """(split_tokens, shared_splits, own_splits) for qb_paged_decode_attn_grouped."""
    want = max(1, math.ceil(4 * sm_count / max(1, batch * hkv)))
    own_max = max(64, max_own)
    split = max(64, math.ceil(math.ceil(own_max / want) / 64) * 64)
    return split, max(1, math.ceil(max(1, max_shared) / split)), max(1, math.ceil(own_max / split))


def grouped_workspace(batch, hq, D, plan, device):
    """Workspace of :func:`paged_decode_attention_grouped` (split-K partials)."""
    nbytes = lib().qb_paged_decode_grouped_workspace_bytes(batch, hq, D, plan[1] + plan[2])
    return torch.empty(nbytes // 4, dtype=torch.float32, device=device)


def paged_decode_attention_grouped(q, k_cache, v_cache, block_tables, seqlens, scale, group_members, shared_len,
                                   kv_start, plan, workspace=None, seqlen_add=1, out=None):
    """Decode attention where groups of sequences share their first ``shared_len`` keys (the
    pages of the group's first member): sequence b attends to those and to its own keys
    [kv_start[b], seqlens[b] + seqlen_add) of its page table; keys in between are skipped.
    With kv_start == shared_len this equals :func:`paged_decode_attention`, the shared keys
    read once per group.  group_members int32 [n_groups, 8] (-1 padded), shared_len int32
    [n_groups], kv_start int32 [B] (multiples of 64)."""
    _cuda(q, k_cache, v_cache, block_tables, seqlens, group_members, shared_len, kv_start)
    B, hq, D = q.shape
    num_blocks, page, hkv, _ = k_cache.shape
    split_tokens, s_sh, s_own = plan
    if workspace is None:
        workspace = grouped_workspace(B, hq, D, plan, q.device)
    if out is None:
        out = torch.empty_like(q)
    check(lib().qb_paged_decode_attn_grouped(_p(q), _p(k_cache), _p(v_cache), num_blocks, page, _p(block_tables),
                                             block_tables.stride(0), _p(seqlens), seqlen_add, B, hq, hkv, D, scale,
                                             _p(group_members), _p(shared_len), group_members.shape[0],
                                             _p(kv_start), split_tokens, s_sh, s_own, _p(workspace), _p(out),
                                             _p(err_flag()), stream_ptr()), "qb_paged_decode_attn_grouped")
    return out


# ---------------------------------------------------------------- MLP / adds / linear
class _SiluMul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        T, two_i = gu.shape
        out = torch.empty(T, two_i // 2, dtype=gu.dtype, device=gu.device)
        check(lib().qb_silu_mul_fwd(_p(gu), T, two_i // 2, _p(out), stream_ptr()), "qb_silu_mul_fwd")
        ctx.save_for_backward(gu)
        return out

    @staticmethod
    def backward(ctx, d):
        (gu,) = ctx.saved_tensors
        d = d.contiguous()
        dgu = torch.empty_like(gu)
        check(lib().qb_silu_mul_bwd(_p(d), _p(gu), gu.shape[0], gu.shape[1] // 2, _p(dgu), stream_ptr()),
              "qb_silu_mul_bwd")
        return dgu


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    _cuda(gate_up)
    gate_up = gate_up.contiguous()
    if torch.is_grad_enabled() and gate_up.requires_grad:
        return _SiluMul.apply(gate_up)
    T, two_i = gate_up.shape
    out = torch.empty(T, two_i // 2, dtype=gate_up.dtype, device=gate_up.device)
    check(lib().qb_silu_mul_fwd(_p(gate_up), T, two_i // 2, _p(out), stream_ptr()), "qb_silu_mul_fwd")
    return out


class _Add(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b):
        out = torch.empty_like(a)
        check(lib().qb_add_bf16(_p(a), _p(b), _p(out), a.numel(), stream_ptr()), "qb_add_bf16")
        return out

    @staticmethod
    def backward(ctx, g):
        return g, g


def add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """bf16 ``a + b`` (the reference's residual adds)."""
    _cuda(a, b)
    a, b = a.contiguous(), b.contiguous()
    if torch.is_grad_enabled() and (a.requires_grad or b.requires_grad):
        return _Add.apply(a, b)
    out = torch.empty_like(a)
    check(lib().qb_add_bf16(_p(a), _p(b), _p(out), a.numel(), stream_ptr()), "qb_add_bf16")
    return out


QB_GEMM_B_STATIC = 0x100  # include/qwen3b200.h


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, mode: int = 0,
         b_static: bool = False) -> torch.Tensor:
    """tcgen05 GEMM: ``a @ b.T`` for bf16 a [M, K], b [N, K] (unit stride along K).

    mode 0 -> bf16 result, 1 -> fp32 result, 2 -> ``out += a @ b.T`` in fp32.  ``b_static``: no
    kernel still running on the stream writes ``b`` (weights), so the GEMM may fetch it before
    the kernel before it has finished."""
    _cuda(a, b)
    if a.dtype != BF16 or b.dtype != BF16 or a.stride(-1) != 1 or b.stride(-1) != 1:
        raise NativeError("gemm needs bf16 operands with unit stride along K")
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=BF16 if mode == 0 else torch.float32, device=a.device)
    flags = QB_GEMM_B_STATIC if b_static else 0
    check(lib().qb_gemm_bf16(_p(a), a.stride(0), _p(b), b.stride(0), _p(out), out.stride(0), M, N, K,
                             mode | flags, _p(err_flag()), stream_ptr()), "qb_gemm_bf16")
    return out


def gemm_plan(M: int, N: int, K: int, b_mn: bool = False, mode: int = 0) -> tuple[str, int, int]:
    """The layout the GEMM picks for an M x N x K product: ("pair" | "single", tile width, split)."""
    import ctypes
    pair, tile_n, split = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(lib().qb_gemm_plan(M, N, K, 1 if b_mn else 0, mode, ctypes.addressof(pair), ctypes.addressof(tile_n),
                             ctypes.addressof(split)), "qb_gemm_plan")
    return ("pair" if pair.value else "single", tile_n.value, split.value)


def gemm_ex(a: torch.Tensor, a_mn: bool, b: torch.Tensor, b_mn: bool, out: torch.Tensor | None = None,
            mode: int = 0) -> torch.Tensor:
    """C = op(a) @ op(b).T on the tcgen05 GEMM.  ``a`` is [M, K] (a_mn False) or stored [K, M]
    (a_mn True); ``b`` is [N, K] (b_mn False) or stored [K, N] (b_mn True).  Unit inner stride."""
    _cuda(a, b)
    a, b = _gemm_operand(a), _gemm_operand(b)
    if a.dtype != BF16 or b.dtype != BF16:
        raise NativeError("gemm_ex needs bf16 operands")
    M, K = (a.shape[1], a.shape[0]) if a_mn else (a.shape[0], a.shape[1])
    N = b.shape[1] if b_mn else b.shape[0]
    if (b.shape[0] if b_mn else b.shape[1]) != K:
        raise NativeError("gemm_ex: inner dimensions differ")
    if out is None:
        out = torch.empty(M, N, dtype=BF16 if mode == 0 else torch.float32, device=a.device)
    check(lib().qb_gemm_bf16_ex(_p(a), a.stride(0), int(a_mn), _p(b), b.stride(0), int(b_mn), _p(out),
                                out.stride(0), M, N, K, mode, _p(err_flag()), stream_ptr()), "qb_gemm_bf16_ex")
    return out


def _gemm_operand(t: torch.Tensor) -> torch.Tensor:
    """2-D view with unit stride along K and a 16-byte row pitch (the TMA operand rules)."""
    if t.stride(-1) != 1 or t.stride(0) % 8 != 0 or t.data_ptr() % 16 != 0:
        t = t.contiguous()
    return t


class _Linear(torch.autograd.Function):
    """y = x w^T on the tcgen05 GEMM; the backward products contract over the output
    dimension and read w and x MN-major: dX = g . w  (B stored [out, in] = [K, N]),
    dW = g^T . x (A stored [tokens, out] = [K, M], B stored [tokens, in] = [K, N])."""

    @staticmethod
    def forward(ctx, x2, w, grad32):
        ctx.save_for_backward(x2, w)
        ctx.grad32 = grad32
        return gemm(x2, w)

    @staticmethod
    def backward(ctx, g):
        x2, w = ctx.saved_tensors
        g = g.contiguous()
        dx = gemm_ex(g, False, w, True) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            if ctx.grad32 is not None:  # dW += g^T x straight into the fp32 accumulator
                gemm_ex(g, True, x2, True, out=ctx.grad32, mode=2)
            else:
                dw = gemm_ex(g, True, x2, True)
        return dx, dw, None


def linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w.T`` for nn.Linear weights [out, in] (bf16) on the tcgen05 GEMM."""
    _cuda(x, w)
    shape = x.shape
    x2 = _gemm_operand(x.reshape(-1, shape[-1]))
    w2 = _gemm_operand(w)
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        y = _Linear.apply(x2, w2, grad32_target(w) if w.requires_grad else None)
    else:
        # a Parameter is written only by the optimizer's kernels, finished before any forward
        y = gemm(x2, w2, b_static=isinstance(w, torch.nn.Parameter))
    return y.view(*shape[:-1], w.shape[0])


def _gemm_swiglu(x2, w, with_gu, b_static):
    M, K = x2.shape
    I = w.shape[0] // 2
    h = torch.empty(M, I, dtype=BF16, device=x2.device)
    gu = torch.empty(M, 2 * I, dtype=BF16, device=x2.device) if with_gu else None
    check(lib().qb_gemm_swiglu(_p(x2), x2.stride(0), _p(w), w.stride(0), _p(h), I, _p(gu) if with_gu else 0,
                               2 * I, M, I, K, QB_GEMM_B_STATIC if b_static else 0, _p(err_flag()),
                               stream_ptr()), "qb_gemm_swiglu")
    return h, gu


class _SwigluLinear(torch.autograd.Function):
    """h = silu(x W_gate^T) * (x W_up^T) in one GEMM (SwiGLU in its epilogue); the bf16 gate_up
    product is kept for the backward, which is the unfused one: SwiGLU backward, then dX and dW of
    the gate_up projection."""

    @staticmethod
    def forward(ctx, x2, w, grad32):
        h, gu = _gemm_swiglu(x2, w, True, False)
        ctx.save_for_backward(x2, w, gu)
        ctx.grad32 = grad32
        return h

    @staticmethod
    def backward(ctx, d):
        x2, w, gu = ctx.saved_tensors
        d = d.contiguous()
        dgu = torch.empty_like(gu)
        check(lib().qb_silu_mul_bwd(_p(d), _p(gu), gu.shape[0], gu.shape[1] // 2, _p(dgu), stream_ptr()),
              "qb_silu_mul_bwd")
        dx = gemm_ex(dgu, False, w, True) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            if ctx.grad32 is not None:
                gemm_ex(dgu, True, x2, True, out=ctx.grad32, mode=2)
            else:
                dw = gemm_ex(dgu, True, x2, True)
        return dx, dw, None


def swiglu_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``silu_mul(linear(x, w))`` for the [2I, in] gate_up weight (gate rows first) in one fused
    GEMM: the same bits as the two-kernel path."""
    _cuda(x, w)
    shape = x.shape
    x2 = _gemm_operand(x.reshape(-1, shape[-1]))
    w2 = _gemm_operand(w)
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        h = _SwigluLinear.apply(x2, w2, grad32_target(w) if w.requires_grad else None)
    else:
        h, _ = _gemm_swiglu(x2, w2, False, isinstance(w, torch.nn.Parameter))
    return h.view(*shape[:-1], w.shape[0] // 2)


# ---------------------------------------------------------------- log-prob / sampling
def _logits_chunk(h, w):
    return gemm(_gemm_operand(h), _gemm_operand(w))


_LSE_WS: dict[tuple, torch.Tensor] = {}


def lm_head_logprob(h, weight, targets, *, dest=None, out=None, lse=None, logits=None):
    """One pass of ``qb_lm_head_logprob``: log-probs of ``targets`` under ``h @ weight.T`` with the
    log-softmax folded into the tcgen05 GEMM's epilogue (fp32 logits, never stored unless
    ``logits`` [n, V] bf16 is given).  ``out`` receives row i at ``out[dest[i]]`` (or ``out[i]``),
    ``lse`` [n] the rows' log-sum-exp.  Returns (out, lse)."""
    _cuda(h, weight, targets)
    h, w = _gemm_operand(h), _gemm_operand(weight)
    n, K = h.shape
    V = w.shape[0]
    if out is None:
        out = torch.empty(n, dtype=torch.float32, device=h.device)
    if lse is None:
        lse = torch.empty(n, dtype=torch.float32, device=h.device)
    nbytes = lib().qb_lm_head_logprob_workspace_bytes(n, V)
    key = (h.device.index, torch.cuda.current_stream(h.device).cuda_stream)
    ws = _LSE_WS.get(key)
    if ws is None or ws.numel() * 4 < nbytes:
        ws = torch.empty((nbytes + 3) // 4, dtype=torch.float32, device=h.device)
        _LSE_WS[key] = ws
    check(lib().qb_lm_head_logprob(_p(h), h.stride(0), _p(w), w.stride(0), n, V, K, _p(targets), _p(dest),
                                   _p(out), _p(lse), _p(logits), 0 if logits is None else logits.stride(0), _p(ws),
                                   _p(err_flag()), stream_ptr()), "qb_lm_head_logprob")
    return out, lse


def logprob_forward(h, weight, targets, dest=None, out=None, out_size=None, chunk_rows=4096, save_lse=True):
    """Token log-probs of ``targets`` under ``lm_head(h)``; no logits are stored.

    Rows are processed ``chunk_rows`` at a time by :func:`lm_head_logprob` (GEMM with the
    log-sum-exp and the gather in its epilogue).  ``dest`` (int64) scatters row i to
    ``out[dest[i]]``; without it ``out`` is [n].  Returns (out, lse[n]).
    """
    _cuda(h, weight, targets)
    n = h.shape[0]
    if out is None:
        size = n if out_size is None else out_size
        out = (torch.zeros if dest is not None else torch.empty)(size, dtype=torch.float32, device=h.device)
    lse = torch.empty(n, dtype=torch.float32, device=h.device)
    for r0 in range(0, n, chunk_rows):
        r1 = min(n, r0 + chunk_rows)
        lm_head_logprob(h[r0:r1], weight, targets[r0:r1], dest=None if dest is None else dest[r0:r1],
                        out=out if dest is not None else out[r0:r1], lse=lse[r0:r1])
    return out, lse


def logprob_backward(h, weight, targets, lse, grad, dest=None, chunk_rows=4096, dweight=None):
    """Gradient of :func:`logprob_forward` w.r.t. ``h`` and ``weight`` (recomputes logits chunks).

    ``grad`` is indexed like the forward's ``out`` (through ``dest``).  Returns (dh, dweight)
    with dweight accumulated into the given fp32 tensor when provided.
    """
    n, V = h.shape[0], weight.shape[0]
    dh = torch.empty_like(h)
    if dweight is None:
        dweight = torch.zeros(weight.shape, dtype=torch.float32, device=h.device)
    L = lib()
    for r0 in range(0, n, chunk_rows):
        r1 = min(n, r0 + chunk_rows)
        hc = h[r0:r1]
        logits = _logits_chunk(hc, weight)
        grad_ptr = _p(grad) if dest is not None else _p(grad) + 4 * r0
        check(L.qb_logprob_bwd(_p(logits), r1 - r0, V, logits.stride(0), _p(targets) + 8 * r0,
                               0 if dest is None else _p(dest) + 8 * r0, _p(lse) + 4 * r0, grad_ptr,
                               _p(err_flag()), stream_ptr()), "qb_logprob_bwd")
        gemm_ex(logits, False, weight, True, out=dh[r0:r1])  # dh = dlogits . W
        gemm_ex(logits, True, hc, True, out=dweight, mode=2)  # dW += dlogits^T . h in fp32
    return dh, dweight


class _LogProb(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, weight, targets, chunk_rows):
        out, lse = logprob_forward(h, weight, targets, chunk_rows=chunk_rows)
        ctx.save_for_backward(h, weight, targets, lse)
        ctx.chunk_rows = chunk_rows
        return out

    @staticmethod
    def backward(ctx, g):
        h, weight, targets, lse = ctx.saved_tensors
        dh, dw = logprob_backward(h, weight, targets, lse, g.contiguous().float(), chunk_rows=ctx.chunk_rows)
        return dh, dw.to(weight.dtype), None, None


def logprob(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, chunk_rows: int = 4096):
    """log_softmax(h @ weight.T).gather(targets) in fp32, differentiable w.r.t. h and weight."""
    h = h.contiguous()
    targets = targets.reshape(-1).long().contiguous()
    if torch.is_grad_enabled() and (h.requires_grad or weight.requires_grad):
        return _LogProb.apply(h, weight, targets, chunk_rows)
    return logprob_forward(h, weight, targets, chunk_rows=chunk_rows)[0]


def sample(logits: torch.Tensor, temperature: float, top_k, seed: int, rng_state: torch.Tensor,
           tokens=None, logp=None):
    """Sample one token per row of bf16 ``logits`` [n, V]; returns (tokens int64, logp fp32).

    ``rng_state`` is a 2-element int64 device tensor {Philox counter, seed mix}, read at run
    time so the call can sit inside a CUDA graph.  ``top_k`` None keeps the full vocabulary.
    """
    offset = rng_state
    _cuda(logits, offset)
    if offset.numel() < 2:
        raise ValueError("rng_state must hold {counter, seed}")
    n, V = logits.shape
    if tokens is None:
        tokens = torch.empty(n, dtype=torch.long, device=logits.device)
    if logp is None:
        logp = torch.empty(n, dtype=torch.float32, device=logits.device)
    k = 0 if top_k is None else int(top_k)
    check(lib().qb_sample(_p(logits), n, V, logits.stride(0), float(temperature), k, int(seed) & (2**64 - 1),
                          _p(offset), _p(tokens), _p(logp), _p(err_flag()), stream_ptr()), "qb_sample")
    return tokens, logp


# ---------------------------------------------------------------- GRPO
def grpo_advantage(rewards: torch.Tensor, group_ids: torch.Tensor) -> torch.Tensor:
    _cuda(rewards, group_ids)
    rewards = rewards.float().contiguous()
    gids = group_ids.long().contiguous()
    adv = torch.empty_like(rewards)
    check(lib().qb_grpo_advantage(_p(rewards), _p(gids), rewards.numel(), _p(adv), stream_ptr()),
          "qb_grpo_advantage")
    return adv


_WS: dict[tuple, torch.Tensor] = {}


def grpo_workspace(n_rows: int, device) -> torch.Tensor:
    """Zero-initialised scratch for the deterministic GRPO reductions (kept zeroed by the kernels)."""
    nbytes = lib().qb_grpo_workspace_bytes(n_rows)
    key = (torch.device(device).index, nbytes)
    ws = _WS.get(key)
    if ws is None:
        ws = torch.zeros((nbytes + 3) // 4, dtype=torch.float32, device=device)
        _WS[key] = ws
    return ws


def grpo_logit_loss(logits, targets, rewards, group_ids, old_lp, mask, *, ref_lp=None, mask_total=None,
                    clip_eps=0.2, beta=0.0, grad_new=None, loss_out=None):
    """``qb_grpo_logit_loss``: log-probs, advantages, clipped + KL loss and d loss / d logits in one
    read and one write of the bf16 ``logits`` [N*S, V] (overwritten with the gradient).
    old_lp / mask / ref_lp are [N, S] fp32.  Returns (new_lp [N, S], loss[3], adv [N])."""
    _cuda(logits, targets, rewards, group_ids, old_lp, mask, ref_lp, mask_total)
    N, S = mask.shape
    V = logits.shape[1]
    if logits.dtype != BF16 or logits.stride(1) != 1 or logits.shape[0] != N * S:
        raise NativeError("grpo_logit_loss needs bf16 logits [N*S, V] with unit column stride")
    new_lp = torch.empty(N, S, dtype=torch.float32, device=logits.device)
    if loss_out is None:
        loss_out = torch.zeros(3, dtype=torch.float32, device=logits.device)
    adv = torch.empty(N, dtype=torch.float32, device=logits.device)
    ws = torch.empty((lib().qb_grpo_logit_loss_workspace_bytes(N, S) + 3) // 4, dtype=torch.float32,
                     device=logits.device)
    f = lambda t: None if t is None else t.float().contiguous()
    old_lp, mask, ref_lp = f(old_lp), f(mask), f(ref_lp)
    check(lib().qb_grpo_logit_loss(_p(logits), logits.stride(0), V, _p(targets.long().contiguous()),
                                   _p(rewards.float().contiguous()), _p(group_ids.long().contiguous()), N, S,
                                   _p(old_lp), _p(ref_lp), _p(mask), _p(mask_total), float(clip_eps), float(beta),
                                   _p(new_lp), _p(grad_new), _p(loss_out), _p(adv), _p(ws), _p(err_flag()),
                                   stream_ptr()), "qb_grpo_logit_loss")
    return new_lp, loss_out, adv


def mask_sum(mask: torch.Tensor, out=None) -> torch.Tensor:
    _cuda(mask)
    mask = mask.float().contiguous()
    if out is None:
        out = torch.empty(1, dtype=torch.float32, device=mask.device)
    ws = grpo_workspace(1, mask.device)
    check(lib().qb_mask_sum(_p(mask), mask.numel(), _p(out), _p(ws), stream_ptr()), "qb_mask_sum")
    return out


def grpo_loss_raw(rewards, group_ids, new_lp, old_lp, mask, *, ref_lp=None, mask_total=None, clip_eps=0.2,
                  beta=0.0, row_begin=0, row_end=None, grad_new=None, loss_out=None, adv_out=None,
                  grad_scale=None):
    """Direct call of ``qb_grpo_loss`` on [N, S] fp32 tensors; see the header for semantics."""
    _cuda(rewards, new_lp, old_lp, mask)
    N, S = new_lp.shape
    row_end = N if row_end is None else row_end
    ws = grpo_workspace(N, new_lp.device)
    check(lib().qb_grpo_loss(_p(rewards), _p(group_ids), N, S, row_begin, row_end, _p(new_lp), _p(old_lp),
                             _p(ref_lp), _p(mask), _p(mask_total), float(clip_eps), float(beta), _p(grad_scale),
                             _p(grad_new), _p(loss_out), _p(adv_out), _p(ws), stream_ptr()), "qb_grpo_loss",
          kernels=1 if mask_total is not None else 2)


class _GRPOLoss(torch.autograd.Function):
    @staticmethod
    def forward(ctx, new_lp, old_lp, mask, rewards, group_ids, ref_lp, clip_eps, beta):
        grad = torch.empty_like(new_lp)
        loss = torch.zeros(3, dtype=torch.float32, device=new_lp.device)
        grpo_loss_raw(rewards, group_ids, new_lp, old_lp, mask, ref_lp=ref_lp, clip_eps=clip_eps, beta=beta,
                      grad_new=grad, loss_out=loss)
        ctx.save_for_backward(grad)
        return loss[0]

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return grad * g, None, None, None, None, None, None, None


def grpo_loss(new_lp, old_lp, mask, rewards, group_ids, ref_lp=None, clip_eps=0.2, beta=0.0):
    """Fused advantage + clipped surrogate (+ beta * k3 KL) masked token-mean; differentiable in new_lp."""
    f = lambda t: None if t is None else t.float().contiguous()
    return _GRPOLoss.apply(f(new_lp), f(old_lp), f(mask), f(rewards), group_ids.long().contiguous(), f(ref_lp),
                           clip_eps, beta)
