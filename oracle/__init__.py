"""CPU oracle for the GRPO-step hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU (fp32 internals), the
algorithms of the reference ``qwen3-naive-inference`` on the GRPO path, each
function citing the reference file:line it follows.  It is the checker the
GPU parity tests compare the CUDA kernels against, and the timed CPU baseline
of ``bench.py --impl reference``.  Nothing in the product package imports it.

Pinning: ``tests/golden/make_golden.py`` imports the reference itself (in the
build container, where its source is present) and records golden vectors for
the host logic (BlockManager, metadata builders, scheduler traces), the GRPO
math and a small dense model forward/backward; ``tests/test_oracle_golden.py``
checks this oracle against those vectors.  Attention inside the reference is
flash-attn (third-party, not shipped with the reference); its restatement
here follows the flash-attn API semantics used at qwen3_naive.py:540,631,672
and is pinned through the reference's dense attention (qwen3_naive.py:553-593),
which the golden model forward exercises.
"""
