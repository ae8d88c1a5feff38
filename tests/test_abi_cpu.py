"""The C-ABI library loads here (no GPU) and exports every symbol include/spd_b200.h
declares; without a CUDA tensor the ops refuse to run (no CPU fallback)."""
import re

import pytest
import torch

from speech_serving import _native as N
from speech_serving import ops


def _declared(repo):
    text = (repo / "include" / "spd_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|uint64_t)\s+(spd_\w+)\s*\(", text, re.M)))


def test_header_declares_the_bound_symbols(golden_dir):
    repo = golden_dir.parent.parent
    assert _declared(repo) == sorted(N.exported_symbols())


def test_library_loads_and_exports_every_declared_symbol(golden_dir):
    lib = N.load()
    for name in _declared(golden_dir.parent.parent):
        assert hasattr(lib, name), name
    assert lib.spd_version() >= 100


def test_last_error_text_roundtrip():
    lib = N.load()
    # invalid dtype is rejected on the host before touching the device
    rc = lib.spd_paged_decode_attn(None, None, None, None, None, None, 1, 1, 64, 16, 1, 1, 1.0, 99,
                                   None, None, None, 0, None)
    assert rc == N.SPD_ERR_UNSUPPORTED
    assert "dtype" in N.last_error()
    rc = lib.spd_block_gather(None, None, None, None, 1, 1, 64, 16, 1, 1, 1, 0, 1, N.SPD_F16, None, None)
    assert rc == N.SPD_ERR_INVALID_ARG


def test_ops_refuse_cpu_tensors():
    q = torch.zeros(2, 4, 64, dtype=torch.float16)
    pool = torch.zeros(8, 16, 4, 64, dtype=torch.float16)
    tab = torch.zeros(2, 1, dtype=torch.int32)
    ctx = torch.ones(2, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.paged_decode_attention(q, pool, pool, tab, ctx)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.cross_attention(q, pool.view(2, 4, 64, 64), pool.view(2, 4, 64, 64), ctx)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.block_gather(pool, tab, ctx, 16)
