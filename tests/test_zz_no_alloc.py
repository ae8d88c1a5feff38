"""The allocation-free paged attention entry point (spd_paged_decode_attn_noalloc).

It serves callers that cannot allocate GPU memory and so cannot hand the kernel a
workspace; its scratch is a fixed array inside the library.  These tests call it through
the C ABI and compare it with the workspace entry point (spd_paged_decode_attn) on calls
in a row: both run the same deterministic kernel on the same inputs, so the outputs must
be bit-identical.  The calls change geometry in both directions (a smaller batch with
the fused K/V append, then a larger B*H than the first call, which moves the scratch
counters to higher offsets) and dtype (fp16, bf16); one call is also checked against the
CPU oracle at the fp16 tolerance of the other kernel tests (2e-3 max-abs).  Oversize and
invalid calls are refused, and device error flags are OR-ed into the caller's word.  The
file is named so that pytest collects it last.
"""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from speech_serving import _native as N
from speech_serving import ops

pytestmark = pytest.mark.gpu

ATOL = 2e-3


def _case(seed, B, H=12, D=64, bs=16, nb=2048, max_ctx=448, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, max_ctx + 1, (B,), generator=g, dtype=torch.int32)
    maxb = -(-max_ctx // bs)
    tables = torch.randperm(nb, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = (torch.randn(B, H, D, generator=g) * 0.5).to(dtype)
    kp = (torch.randn(nb, bs, H, D, generator=g) * 0.5).to(dtype)
    vp = (torch.randn(nb, bs, H, D, generator=g) * 0.5).to(dtype)
    kn = (torch.randn(B, H, D, generator=g) * 0.5).to(dtype)
    vn = (torch.randn(B, H, D, generator=g) * 0.5).to(dtype)
    return [t.cuda() for t in (q, kp, vp, tables, ctx, kn, vn)]


def _noalloc(q, kp, vp, tables, ctx, out, k_new=None, v_new=None, err=None, scale=0.125):
    B, H, D = q.shape
    return N.load().spd_paged_decode_attn_noalloc(
        q.data_ptr(), kp.data_ptr(), vp.data_ptr(), tables.data_ptr(), ctx.data_ptr(), out.data_ptr(), B, H, D,
        kp.shape[1], tables.shape[1], kp.shape[0], scale, ops.dtype_code(q.dtype),
        None if k_new is None else k_new.data_ptr(), None if v_new is None else v_new.data_ptr(),
        None if err is None else err.data_ptr(), torch.cuda.current_stream().cuda_stream)


def _run_pair(case, append=False):
    """(no-alloc output, workspace output, pools after each) on one case."""
    q, kp, vp, tab, ctx, kn, vn = case
    kw = dict(k_new=kn, v_new=vn) if append else {}
    kp1, vp1 = kp.clone(), vp.clone()
    ref = ops.paged_decode_attention(q, kp1, vp1, tab, ctx, scale=0.125, **kw)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full_like(q, float("nan"))
    kp2, vp2 = kp.clone(), vp.clone()
    assert _noalloc(q, kp2, vp2, tab, ctx, out, err=err, **kw) == N.SPD_OK, N.last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out, ref, (kp1, vp1), (kp2, vp2)


def test_noalloc_is_bit_identical_to_workspace_entry_point_across_geometries():
    # call 1: the BASELINE config-2 batch shape, also checked against the CPU oracle
    c1 = _case(1, B=64)
    out, ref, _, _ = _run_pair(c1)
    assert torch.equal(out, ref)
    q, kp, vp, tab, ctx, _, _ = c1
    want = O.paged_decode_attention(q.float().cpu().numpy(), kp.float().cpu().numpy(), vp.float().cpu().numpy(),
                                    tab.cpu().numpy(), ctx.cpu().numpy(), 0.125)
    assert float(np.abs(out.float().cpu().numpy() - want).max()) <= ATOL

    # call 2, straight after: a smaller batch with the fused K/V append
    out, ref, pools_ws, pools_na = _run_pair(_case(2, B=23), append=True)
    assert torch.equal(out, ref)
    assert torch.equal(pools_ws[0], pools_na[0]) and torch.equal(pools_ws[1], pools_na[1])

    # call 3: a larger B*H than call 1 (counters and partials at higher offsets)
    out, ref, _, _ = _run_pair(_case(3, B=96, H=16, max_ctx=256))
    assert torch.equal(out, ref)

    # calls 4 and 5: bf16, twice in a row
    c4 = _case(4, B=40, dtype=torch.bfloat16)
    for _ in range(2):
        out, ref, _, _ = _run_pair(c4)
        assert torch.equal(out, ref)


def test_noalloc_reports_device_errors_and_refuses_bad_calls():
    q, kp, vp, tab, ctx, _, _ = _case(3, B=8)
    tab[0, 0] = 10 ** 6  # a block id beyond the pool: clamped on the device and flagged
    err = torch.full((1,), N.SPD_DEVERR_TIMEOUT, dtype=torch.int32, device="cuda")  # a flag set earlier
    out = torch.empty_like(q)
    assert _noalloc(q, kp, vp, tab, ctx, out, err=err) == N.SPD_OK
    torch.cuda.synchronize()
    assert int(err.item()) == N.SPD_DEVERR_BLOCK_ID | N.SPD_DEVERR_TIMEOUT  # OR-ed, not replaced
    # a geometry whose scratch exceeds the fixed array is refused on the host
    big_q = torch.zeros(2048, 32, 128, dtype=torch.float16, device="cuda")
    rc = _noalloc(big_q, kp, vp, tab[:1].expand(2048, -1).contiguous(), ctx[:1].expand(2048).contiguous(),
                  torch.empty_like(big_q))
    assert rc == N.SPD_ERR_WORKSPACE
    assert "scratch" in N.last_error()
    # invalid arguments are refused before the scratch is touched
    rc = N.load().spd_paged_decode_attn_noalloc(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), tab.data_ptr(),
                                                ctx.data_ptr(), out.data_ptr(), 8, 12, 64, 12, tab.shape[1],
                                                kp.shape[0], 0.125, N.SPD_F16, None, None, None,
                                                torch.cuda.current_stream().cuda_stream)
    assert rc == N.SPD_ERR_UNSUPPORTED and "block_size" in N.last_error()
