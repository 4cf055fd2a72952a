"""ctypes binding of ``libqwen3b200.so`` (declared in ``include/qwen3b200.h``).

The library is loaded once per process.  Loading works without a GPU (the CPU
test suite checks every exported symbol); *calling* any compute entry point
requires CUDA tensors -- there is deliberately no CPU fallback.  If the shared
library is missing this module raises at import-use time with the build
command, so a GPU run can never silently route around the native code.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libqwen3b200.so"

P = c_void_p
I = c_int
L = c_int64
F = c_float

# name -> (restype, argtypes); mirrors include/qwen3b200.h one to one.
SIGNATURES: dict[str, tuple] = {
    "qb_abi_version": (I, []),
    "qb_status_string": (ctypes.c_char_p, [I]),
    "qb_embedding_fwd": (I, [P, L, P, L, L, P, P, P]),
    "qb_embedding_bwd": (I, [P, L, P, L, L, P, P, P]),
    "qb_rmsnorm_fwd": (I, [P, P, P, P, L, L, F, P]),
    "qb_add_rmsnorm_fwd": (I, [P, P, P, P, L, L, F, P]),
    "qb_rmsnorm_bwd": (I, [P, P, P, P, P, P, L, L, P]),
    "qb_qk_norm_rope_fwd": (I, [P, L, L, I, I, I, P, P, L, P, P, F, P, L, P, P, P, P, L, P, P, P, P]),
    "qb_qk_norm_rope_bwd": (I, [P, P, L, L, I, I, I, P, P, L, P, P, P, P, I, P, P, P, P, P]),
    "qb_silu_mul_fwd": (I, [P, L, L, P, P]),
    "qb_silu_mul_bwd": (I, [P, P, L, L, P, P]),
    "qb_add_bf16": (I, [P, P, P, L, P]),
    "qb_attn_varlen_fwd": (I, [P, L, P, P, L, P, L, L, I, P, P, I, P, I, I, I, I, I, F, P, L, P, L, P, P]),
    # (q, q_stride, k, v, kv_stride, block_tables, bt_stride, num_blocks, page_size, cu_q, cu_k,
    #  batch, tile_info, n_tiles, tiles_per_seq, hq, hkv, D, scale, out, o_stride, lse, total_q,
    #  err, stream)
    "qb_attn_varlen_bwd": (I, [P, P, P, L, P, P, L, P, P, I, P, I, I, I, I, F, L, P, P, P, P, P, P]),
    "qb_paged_decode_attn": (I, [P, P, P, L, I, P, L, P, I, I, I, I, I, F, I, I, P, P, P, P]),
    "qb_paged_decode_workspace_bytes": (c_size_t, [I, I, I, I]),
    "qb_paged_decode_attn_grouped": (I, [P, P, P, L, I, P, L, P, I, I, I, I, I, F, P, P, I, P, I, I, I, P, P, P,
                                         P]),
    "qb_paged_decode_grouped_workspace_bytes": (c_size_t, [I, I, I, I]),
    "qb_logprob_fwd": (I, [P, L, L, L, P, P, P, P, P, P]),
    "qb_logprob_bwd": (I, [P, L, L, L, P, P, P, P, P, P]),
    "qb_lm_head_logprob": (I, [P, L, P, L, L, L, L, P, P, P, P, P, L, P, P, P]),
    "qb_lm_head_logprob_workspace_bytes": (c_size_t, [L, L]),
    "qb_sample": (I, [P, L, L, L, F, I, c_uint64, P, P, P, P, P]),
    "qb_grpo_advantage": (I, [P, P, L, P, P]),
    "qb_grpo_loss": (I, [P, P, L, L, L, L, P, P, P, P, P, F, F, P, P, P, P, P, P]),
    "qb_grpo_workspace_bytes": (c_size_t, [L]),
    "qb_grpo_logit_loss": (I, [P, L, L, P, P, P, L, L, P, P, P, P, F, F, P, P, P, P, P, P, P]),
    "qb_grpo_logit_loss_workspace_bytes": (c_size_t, [L, L]),
    "qb_ppo_clipped_loss": (I, [P, P, P, P, P, L, L, P, F, F, P, P, P, P, P]),
    "qb_grpo_loss_noalloc": (I, [P, P, L, L, L, L, P, P, P, P, P, F, F, P, P, P, P, P]),
    "qb_mask_sum": (I, [P, L, P, P, P]),
    "qb_gemm_bf16": (I, [P, L, P, L, P, L, L, L, L, I, P, P]),
    "qb_gemm_bf16_ex": (I, [P, L, I, P, L, I, P, L, L, L, L, I, P, P]),
    "qb_set_pdl": (I, [I]),
    "qb_get_pdl": (I, []),
    "qb_gemm_swiglu": (I, [P, L, P, L, P, L, P, L, L, L, L, I, P, P]),
    "qb_gemm_qk_norm_rope": (I, [P, L, P, L, L, I, I, L, P, P, L, P, P, F, P, L, P, L, P, P, P, P, L, P, P, I, P,
                                 P]),
    "qb_gemm_plan": (I, [L, L, L, I, I, P, P, P]),
    "qb_f32_to_bf16": (I, [P, P, L, P]),
    "qb_accumulate_bf16": (I, [P, P, L, P]),
}

_LIB = None

# Kernels launched per successful call of each entry point (for launch accounting).
KERNELS_PER_CALL = {"qb_attn_varlen_bwd": 3, "qb_grpo_loss": 1, "qb_ppo_clipped_loss": 1}
LAUNCHES = [0]  # running count of this library's kernel launches issued from Python


class NativeError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load the shared library (once) and attach the declared signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise NativeError(
            f"{LIB_PATH.name} is not built; run `python -m qwen3_naive_inference_b200.build` "
            "(the CUDA path has no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def check(status: int, what: str, kernels: int | None = None) -> None:
    if status != 0:
        msg = load().qb_status_string(status).decode()
        raise NativeError(f"{what} failed with status {status}: {msg}")
    LAUNCHES[0] += KERNELS_PER_CALL.get(what, 1) if kernels is None else kernels
