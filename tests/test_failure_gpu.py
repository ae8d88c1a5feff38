"""Failure detection on the GPU without faulting it.

Every wait in the attention kernels is bounded; a wait that runs out records
SPD_DEVERR_TIMEOUT in the launch's error word, the launch abandons its work, waits (with
the default bound) for its own copies still in flight and returns, so the context stays
usable.  The first test makes a wait run out on purpose: a barrier phase that nothing
completes, under a 1 ms bound.  The others give real launches a 1 ns bound: a wait
then gives up once 64 suspended tries on its barrier have come back empty (whether the
data beats that depends on the hardware's suspend interval), so each such launch either
completes exactly or stops with SPD_DEVERR_TIMEOUT — never faults — and the next launches
on the same context and workspace, under the default bound, are exact.  Nothing here
traps, faults or hangs: no launch is left with a copy in flight.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import c_oracle
from speech_serving import _native as N
from speech_serving import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture
def short_waits():
    """Restores the default bound after a test that shortened it."""
    lib = N.load()
    yield lib
    assert lib.spd_set_wait_timeout_ns(0) == N.SPD_OK
    assert lib.spd_get_wait_timeout_ns() == 2_000_000_000


def _paged_case(seed, B=64, H=12, D=64, bs=16, nb=4096, max_ctx=448):
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, max_ctx + 1, (B,), generator=g, dtype=torch.int32)
    maxb = max_ctx // bs
    tab = torch.randperm(nb, generator=g)[: B * maxb].view(B, maxb).to(torch.int32)
    q = (torch.randn(B, H, D, generator=g) * 0.5).half()
    kp = (torch.randn(nb, bs, H, D, generator=g) * 0.5).half()
    vp = (torch.randn(nb, bs, H, D, generator=g) * 0.5).half()
    return q, kp, vp, tab, ctx


def test_wait_that_nothing_completes_times_out(short_waits):
    lib = short_waits
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    assert lib.spd_selftest_wait_timeout(C.c_void_p(err.data_ptr()), 1_000_000,
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream)) == N.SPD_OK
    e.record()
    torch.cuda.synchronize()
    assert int(err.item()) == N.SPD_DEVERR_TIMEOUT
    assert s.elapsed_time(e) >= 0.9  # ms: the wait held on until its 1 ms bound
    assert lib.spd_selftest_wait_timeout(None, 1000, None) == N.SPD_ERR_INVALID_ARG


def test_paged_attention_under_tiny_bound_then_exact(short_waits):
    lib = short_waits
    q, kp, vp, tab, ctx = [t.to(DEV) for t in _paged_case(11)]
    ws = ops.paged_attn_workspace(64, 12, 64, tab.shape[1], torch.device(DEV))
    assert lib.spd_set_wait_timeout_ns(1) == N.SPD_OK and lib.spd_get_wait_timeout_ns() == 1
    ref = c_oracle.paged_decode_attention(q.cpu().numpy(), kp.cpu().numpy(), vp.cpu().numpy(), tab.cpu().numpy(),
                                          ctx.cpu().numpy(), 0.125)
    first = ops.paged_decode_attention(q, kp, vp, tab, ctx, scale=0.125, workspace=ws)
    torch.cuda.synchronize()
    word = ops.read_error_word(ws)
    print(f"paged attention under a 1 ns wait bound: error word {word}")
    assert word in (0, N.SPD_DEVERR_TIMEOUT)
    if word == 0:
        assert float(np.abs(first.float().cpu().numpy() - ref).max()) <= 2e-3
    # same context, same workspace (its counters were re-armed), default bound: exact
    assert lib.spd_set_wait_timeout_ns(0) == N.SPD_OK
    ws[:4].zero_()  # clear the sticky error word
    out = ops.paged_decode_attention(q, kp, vp, tab, ctx, scale=0.125, workspace=ws)
    torch.cuda.synchronize()
    assert ops.read_error_word(ws) == 0
    assert float(np.abs(out.float().cpu().numpy() - ref).max()) <= 2e-3
    again = ops.paged_decode_attention(q, kp, vp, tab, ctx, scale=0.125, workspace=ws)
    assert torch.equal(again, out)


def test_cross_attention_under_tiny_bound_then_exact(short_waits):
    lib = short_waits
    g = torch.Generator().manual_seed(5)
    B, H, T, D = 32, 12, 1500, 64
    q = (torch.randn(B, H, D, generator=g) * 0.5).half().to(DEV)
    k = (torch.randn(B, H, T, D, generator=g) * 0.5).half().to(DEV)
    v = (torch.randn(B, H, T, D, generator=g) * 0.5).half().to(DEV)
    valid = torch.randint(300, T + 1, (B,), generator=g, dtype=torch.int32).to(DEV)
    ws = ops.cross_attn_workspace(B, H, D, torch.device(DEV))
    fresh = ops.cross_attention(q, k, v, valid, scale=0.125)
    assert lib.spd_set_wait_timeout_ns(1) == N.SPD_OK
    first = ops.cross_attention(q, k, v, valid, scale=0.125, workspace=ws)
    torch.cuda.synchronize()
    word = ops.read_error_word(ws)
    print(f"cross attention under a 1 ns wait bound: error word {word}")
    assert word in (0, N.SPD_DEVERR_TIMEOUT)
    if word == 0:
        assert torch.equal(first, fresh)
    assert lib.spd_set_wait_timeout_ns(0) == N.SPD_OK
    ws[:4].zero_()
    out = ops.cross_attention(q, k, v, valid, scale=0.125, workspace=ws)
    torch.cuda.synchronize()
    assert ops.read_error_word(ws) == 0
    assert torch.equal(out, fresh)
