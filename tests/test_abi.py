"""The C-ABI library: loads without a GPU, exports every declared entry point, and
rejects bad arguments on the host before any launch (CPU only)."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

from qwen3_naive_inference_b200 import _lib, ops

HEADER = Path(__file__).resolve().parents[1] / "include" / "qwen3b200.h"


def declared():
    src = HEADER.read_text()
    return re.findall(r"\n(?:int|size_t|const char\*)\s+(qb_\w+)\(([^;]*?)\);", src, re.S)


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    protos = declared()
    assert len(protos) >= 20
    for name, args in protos:
        assert hasattr(lib, name), name
        n = 0 if args.strip() in ("void", "") else len(args.split(","))
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes table"
        assert len(_lib.SIGNATURES[name][1]) == n, f"{name}: {n} C args vs {len(_lib.SIGNATURES[name][1])}"
    assert set(_lib.SIGNATURES) == {n for n, _ in protos}


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.qb_abi_version() == 2
    assert lib.qb_status_string(0) == b"ok"
    assert b"invalid" in lib.qb_status_string(1)
    assert b"unsupported" in lib.qb_status_string(2)


def test_pdl_switch():
    """The library-wide launch switch (programmatic dependent launch) needs no GPU to set."""
    lib = _lib.load()
    old = lib.qb_get_pdl()
    assert old == 1  # on by default
    assert lib.qb_set_pdl(0) == 0 and lib.qb_get_pdl() == 0
    assert lib.qb_set_pdl(7) == 0 and lib.qb_get_pdl() == 1
    lib.qb_set_pdl(old)


def test_workspace_size_queries():
    lib = _lib.load()
    assert lib.qb_paged_decode_workspace_bytes(256, 16, 128, 1) == 0
    assert lib.qb_paged_decode_workspace_bytes(256, 16, 128, 4) == 256 * 4 * 16 * 132 * 4
    assert lib.qb_grpo_workspace_bytes(4096) >= 16 + 8 * 4096
    # grouped decode: split-K partials only (shared + own slots per sequence and head)
    assert lib.qb_paged_decode_grouped_workspace_bytes(512, 16, 128, 2) == 512 * 2 * 16 * 132 * 4


def test_host_side_argument_validation():
    lib = _lib.load()
    # null pointers with work to do -> QB_ERR_INVALID, no launch
    assert lib.qb_rmsnorm_fwd(None, None, None, None, 4, 1024, 1e-6, None) == 1
    assert lib.qb_rmsnorm_fwd(None, None, None, None, 4, 1000, 1e-6, None) == 1  # cols % 256
    assert lib.qb_embedding_fwd(None, 3, None, 10, 1024, None, None, None) == 1
    # unsupported head_dim / page size
    assert lib.qb_paged_decode_attn(None, None, None, 1, 256, None, 1, None, 1, 1, 16, 8, 64, 1.0, 64, 1, None,
                                    None, None, None) == 2
    assert lib.qb_attn_varlen_fwd(None, 0, None, None, 0, None, 0, 0, 256, None, None, 1, None, 1, 0, 16, 8, 96,
                                  1.0, None, 0, None, 0, None, None) == 2
    # empty work is a no-op success
    assert lib.qb_rmsnorm_fwd(None, None, None, None, 0, 1024, 1e-6, None) == 0
    assert lib.qb_sample(None, 0, 8, 8, 1.0, 0, 0, None, None, None, None, None) == 0
    # bad sampling arguments
    assert lib.qb_sample(None, 1, 8, 8, 0.0, 0, 0, None, None, None, None, None) == 1


def test_ops_refuse_cpu_tensors():
    x = torch.zeros(2, 1024, dtype=torch.bfloat16)
    w = torch.ones(1024, dtype=torch.bfloat16)
    with pytest.raises(ops.NativeError):
        ops.rmsnorm(x, w, 1e-6)
    with pytest.raises(ops.NativeError):
        ops.grpo_advantage(torch.zeros(4), torch.zeros(4, dtype=torch.long))


def test_build_tiles():
    t = ops.build_tiles([1, 64, 65, 0, 130]).reshape(-1, 2).tolist()
    assert t == [[0, 0], [1, 0], [2, 0], [2, 64], [4, 0], [4, 64], [4, 128]]


def test_decode_split_plan_covers_context():
    for B in (1, 8, 64, 256, 512):
        for ctx in (1, 64, 1000, 8192):
            st, ms = ops.decode_split_plan(B, 8, ctx)
            assert st % 64 == 0 and st * ms >= ctx and ms >= 1
            assert (ms - 1) * st < ctx
