"""B200-native GRPO step for Qwen3 (drop-in for qwen3-naive-inference's GRPO path).

Modules mirror the reference's:
  qwen3_naive        Qwen3Config, Sequence, BlockManager, Qwen3ForCausalLM (+ generate_continuous*)
  qwen3_grpo_train   forward_logprob, compute_grpo_advantage, ppo_clipped_loss, grpo_train_step,
                     rollout_batch, grpo_step (the full step, data-parallel aware)
Kernels live in ``libqwen3b200.so`` (C ABI: include/qwen3b200.h), bound in ``_lib``/``ops``.
"""
from .qwen3_naive import (BlockManager, Qwen3Config, Qwen3ForCausalLM, Sequence,  # noqa: F401
                          load_weights)

__all__ = ["BlockManager", "Qwen3Config", "Qwen3ForCausalLM", "Sequence", "load_weights"]
