"""The allocation-free paged attention entry point (spd_paged_decode_attn_noalloc).

It serves callers that cannot allocate GPU memory and so cannot hand the kernel a
workspace; its scratch is a fixed array inside the library.  These tests call it through
the C ABI and compare it with the workspace entry point (spd_paged_decode_attn) on two
calls in a row — the second with another batch size, which moves where the scratch
counters sit, and with the fused K/V append — at the fp16 tolerance of the other kernel
tests (2e-3 max-abs), and check that oversize calls are refused.  The file is named so
that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from speech_serving import _native as N
from speech_serving import ops

pytestmark = pytest.mark.gpu

ATOL = 2e-3


def _case(seed, B, H=12, D=64, bs=16, nb=2048, max_ctx=448):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, max_ctx + 1, (B,), generator=g, dtype=torch.int32)
    maxb = -(-max_ctx // bs)
    tables = torch.randperm(nb, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = (torch.randn(B, H, D, generator=g) * 0.5).half()
    kp = (torch.randn(nb, bs, H, D, generator=g) * 0.5).half()
    vp = (torch.randn(nb, bs, H, D, generator=g) * 0.5).half()
    kn = (torch.randn(B, H, D, generator=g) * 0.5).half()
    vn = (torch.randn(B, H, D, generator=g) * 0.5).half()
    return [t.cuda() for t in (q, kp, vp, tables, ctx, kn, vn)]


def _noalloc(q, kp, vp, tables, ctx, out, k_new=None, v_new=None, err=None):
    B, H, D = q.shape
    return N.load().spd_paged_decode_attn_noalloc(
        q.data_ptr(), kp.data_ptr(), vp.data_ptr(), tables.data_ptr(), ctx.data_ptr(), out.data_ptr(), B, H, D,
        kp.shape[1], tables.shape[1], kp.shape[0], 0.125, N.SPD_F16, None if k_new is None else k_new.data_ptr(),
        None if v_new is None else v_new.data_ptr(), None if err is None else err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # call 1: the BASELINE config-2 batch shape
    q, kp, vp, tab, ctx, _, _ = _case(1, B=64)
    ref = ops.paged_decode_attention(q, kp, vp, tab, ctx, scale=0.125)
    out = torch.full_like(q, float("nan"))
    assert _noalloc(q, kp, vp, tab, ctx, out, err=err) == N.SPD_OK, N.last_error()
    torch.cuda.synchronize()
    assert float((out.float() - ref.float()).abs().max()) <= ATOL
    assert int(err.item()) == 0

    # call 2, straight after: another batch size and the fused K/V append
    q, kp, vp, tab, ctx, kn, vn = _case(2, B=23)
    kp2, vp2 = kp.clone(), vp.clone()
    ref = ops.paged_decode_attention(q, kp, vp, tab, ctx, scale=0.125, k_new=kn, v_new=vn)
    out = torch.full_like(q, float("nan"))
    assert _noalloc(q, kp2, vp2, tab, ctx, out, k_new=kn, v_new=vn, err=err) == N.SPD_OK, N.last_error()
    torch.cuda.synchronize()
    assert float((out.float() - ref.float()).abs().max()) <= ATOL
    assert torch.equal(kp2, kp) and torch.equal(vp2, vp)  # identical appended rows
    assert int(err.item()) == 0


def test_noalloc_reports_device_errors_and_refuses_oversize():
    q, kp, vp, tab, ctx, _, _ = _case(3, B=8)
    tab[0, 0] = 10 ** 6  # a block id beyond the pool: clamped on the device and flagged
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    assert _noalloc(q, kp, vp, tab, ctx, out, err=err) == N.SPD_OK
    torch.cuda.synchronize()
    assert int(err.item()) & N.SPD_DEVERR_BLOCK_ID
    # a geometry whose scratch exceeds the fixed array is refused on the host
    big_q = torch.zeros(2048, 32, 128, dtype=torch.float16, device="cuda")
    rc = _noalloc(big_q, kp, vp, tab[:1].expand(2048, -1).contiguous(), ctx[:1].expand(2048).contiguous(),
                  torch.empty_like(big_q))
    assert rc == N.SPD_ERR_WORKSPACE
    assert "scratch" in N.last_error()
