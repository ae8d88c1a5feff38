"""Parity of the sm_100a kernels (called through the C ABI) with the reference's
arithmetic: the golden fixtures made by running the reference, and the CPU oracle on
seeded inputs at BASELINE sizes.

Tolerances: fp16/bf16 attention outputs within 2e-3 max-abs of the
fp32 computation; fp32 within 2e-5; K/V writes and gathers bit-exact.
"""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from oracle import c_oracle
from speech_serving import _native as N
from speech_serving import ops

pytestmark = pytest.mark.gpu

ATOL_16 = 2e-3
ATOL_32 = 2e-5
DEV = "cuda"


def _case(npz, name):
    return {k.split("__", 1)[1]: npz[k] for k in npz.files if k.startswith(name + "__")}


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t if dtype is None else t.to(dtype)


def _tol(dtype):
    return ATOL_32 if dtype == torch.float32 else ATOL_16


def _np32(t):
    return t.float().cpu().numpy()


def _err(out: torch.Tensor, ref: np.ndarray) -> float:
    """Max-abs difference between a kernel output and the fp32 reference rounded to the
    output's dtype (the closest value that dtype can hold).  For fp16 the rounding is
    below 1e-3 at these magnitudes; for bf16 (8-bit mantissa) |out| ~ 1.5 alone carries
    a 4e-3 representation error, which no bf16 output can avoid."""
    ref_rounded = torch.from_numpy(np.asarray(ref, np.float32)).to(out.dtype).float().numpy()
    return float(np.abs(_np32(out) - ref_rounded).max())


# ----------------------------------------------------------------------------- op (1)
@pytest.mark.parametrize("case", ["small", "whisper"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_paged_attention_matches_reference_golden(golden_dir, case, dtype):
    g = _case(np.load(golden_dir / "paged_attn_ref.npz"), case)
    out = ops.paged_decode_attention(_t(g["q"], dtype), _t(g["k_pool"], dtype), _t(g["v_pool"], dtype),
                                     _t(g["block_tables"]), _t(g["context_lens"]))
    torch.cuda.synchronize()
    err = _err(out, g["out"])
    assert err <= _tol(dtype), err


def _random_paged(rng, B, H, D, bs, nb, ctx, dtype):
    max_blocks = max(1, max(-(-int(c) // bs) for c in ctx))
    perm = rng.permutation(nb)
    tables = np.zeros((B, max_blocks), np.int32)
    k = 0
    for b in range(B):
        n = -(-int(ctx[b]) // bs)
        tables[b, :n] = perm[k : k + n]
        k += n
    q = (rng.standard_normal((B, H, D)) * 0.5).astype(np.float32)
    kp = (rng.standard_normal((nb, bs, H, D)) * 0.5).astype(np.float32)
    vp = (rng.standard_normal((nb, bs, H, D)) * 0.5).astype(np.float32)
    tq, tk, tv = _t(q, dtype), _t(kp, dtype), _t(vp, dtype)
    # the oracle sees exactly the values the kernel sees
    return tq, tk, tv, _t(tables), _t(np.asarray(ctx, np.int32)), _np32(tq), _np32(tk), _np32(tv), tables


GEOMS = [  # (H, D, block_size)
    (12, 64, 16), (20, 64, 16), (4, 16, 8), (6, 64, 16), (8, 128, 16), (4, 32, 32), (2, 64, 8), (32, 64, 16),
]


@pytest.mark.parametrize("H,D,bs", GEOMS)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_paged_attention_matches_oracle(H, D, bs, dtype):
    if H * D * bs * (4 if dtype == torch.float32 else 2) * 2 > 220 * 1024:
        pytest.skip("one pool block of K and V exceeds shared memory (reported as SPD_ERR_UNSUPPORTED)")
    rng = np.random.default_rng(H * 100_000 + D * 100 + bs + 7 * [torch.float16, torch.bfloat16, torch.float32].index(dtype))
    B = 9
    ctx = np.array([1, bs, bs + 1, 0, 3 * bs - 1, 200, 448, 77, 2], np.int32)
    nb = int(sum(-(-c // bs) for c in ctx)) + 8
    tq, tk, tv, tt, tc, q, kp, vp, tables = _random_paged(rng, B, H, D, bs, nb, ctx, dtype)
    scale = 1.0 / math.sqrt(D)
    out = ops.paged_decode_attention(tq, tk, tv, tt, tc, scale=scale)
    ref = O.paged_decode_attention(q, kp, vp, tables, ctx, scale)
    err = _err(out, ref)
    assert err <= _tol(dtype), err
    assert not _np32(out)[3].any()  # context 0 -> zeros


@pytest.mark.parametrize("B,ctx_fn", [
    (1, lambda r, B: np.array([448])),                      # one sequence split over many CTAs
    (1, lambda r, B: np.array([1])),                        # fewer units than CTAs
    (3, lambda r, B: np.array([0, 0, 0])),                  # nothing to do
    (130, lambda r, B: r.integers(1, 449, B)),              # more sequences than SMs
    (700, lambda r, B: r.integers(0, 40, B)),               # many short / empty sequences
    (4, lambda r, B: np.array([4096, 1500, 37, 1030])),     # more than 32 items per sequence
    (3, lambda r, B: np.array([512, 513, 480])),            # 16 items (merged in registers), 17 (two passes)
])
def test_paged_attention_partitions(B, ctx_fn):
    rng = np.random.default_rng(B)
    H, D, bs = 12, 64, 16
    ctx = ctx_fn(rng, B).astype(np.int32)
    nb = int(sum(-(-int(c) // bs) for c in ctx)) + 4
    tq, tk, tv, tt, tc, q, kp, vp, tables = _random_paged(rng, B, H, D, bs, nb, ctx, torch.float16)
    out = ops.paged_decode_attention(tq, tk, tv, tt, tc, scale=0.125)
    ref = c_oracle.paged_decode_attention(q, kp, vp, tables, ctx, 0.125)
    assert _err(out, ref) <= ATOL_16


def test_paged_attention_config2_full_size():
    """B=64, H=12, D=64, bs=16, ctx ~ U[1,448], 4096-block pool
    (seeded permutation), q/K/V ~ N(0,1)*0.5, scale 1/8, fp16."""
    g = torch.Generator().manual_seed(2)
    B, H, D, bs, NB = 64, 12, 64, 16, 4096
    ctx = torch.randint(1, 449, (B,), generator=g, dtype=torch.int32)
    perm = torch.randperm(NB, generator=g).to(torch.int32)
    tables = perm[: B * 28].view(B, 28).contiguous()
    q = (torch.randn(B, H, D, generator=g) * 0.5).half()
    kp = (torch.randn(NB, bs, H, D, generator=g) * 0.5).half()
    vp = (torch.randn(NB, bs, H, D, generator=g) * 0.5).half()
    out = ops.paged_decode_attention(q.cuda(), kp.cuda(), vp.cuda(), tables.cuda(), ctx.cuda(), scale=0.125)
    ref = c_oracle.paged_decode_attention(q.numpy(), kp.numpy(), vp.numpy(), tables.numpy(), ctx.numpy(), 0.125)
    assert _err(out, ref) <= ATOL_16


@pytest.mark.parametrize("dtype,B", [(torch.float16, 5), (torch.bfloat16, 5), (torch.float16, 160)])
def test_fused_append_writes_row_and_attends_to_it(dtype, B):
    """B=160 runs the two-CTAs-per-SM form, whose stages take the new row by copy."""
    rng = np.random.default_rng(11)
    H, D, bs = 12, 64, 16
    ctx = np.array([1, 16, 17, 100, 33], np.int32) if B == 5 else rng.integers(1, 300, B).astype(np.int32)
    nb = int(sum(-(-int(c) // bs) for c in ctx)) + 8
    tq, tk, tv, tt, tc, q, kp, vp, tables = _random_paged(rng, B, H, D, bs, nb, ctx, dtype)
    k_new = (torch.randn(B, H, D) * 0.5).to(dtype).to(DEV)
    v_new = (torch.randn(B, H, D) * 0.5).to(dtype).to(DEV)
    before_k = tk.clone()
    out = ops.paged_decode_attention(tq, tk, tv, tt, tc, scale=0.125, k_new=k_new, v_new=v_new)
    # oracle: write the new rows with op (3) semantics, then attend
    kp2, vp2 = kp.copy(), vp.copy()
    O.kv_append(_np32(k_new)[:, :, None], _np32(v_new)[:, :, None], kp2, vp2, tables, ctx - 1)
    ref = O.paged_decode_attention(q, kp2, vp2, tables, ctx, 0.125)
    assert _err(out, ref) <= ATOL_16
    # the pool rows are bit-exact copies of k_new / v_new, and nothing else changed
    for b in range(B):
        pos = int(ctx[b]) - 1
        blk = int(tables[b, pos // bs])
        assert torch.equal(tk[blk, pos % bs], k_new[b])
        assert torch.equal(tv[blk, pos % bs], v_new[b])
        before_k[blk, pos % bs] = k_new[b]
    assert torch.equal(tk, before_k)


def test_paged_attention_repeat_calls_and_counters_reset():
    rng = np.random.default_rng(5)
    B, H, D, bs = 64, 12, 64, 16
    ctx = rng.integers(1, 449, B).astype(np.int32)
    nb = int(sum(-(-int(c) // bs) for c in ctx)) + 4
    tq, tk, tv, tt, tc, *_ = _random_paged(rng, B, H, D, bs, nb, ctx, torch.float16)
    ws = ops.paged_attn_workspace(B, H, D, tt.shape[1], tq.device)
    a = ops.paged_decode_attention(tq, tk, tv, tt, tc, workspace=ws)
    b = ops.paged_decode_attention(tq, tk, tv, tt, tc, workspace=ws)
    assert torch.equal(a, b)
    counters = ws[256 : 256 + 4 * B * H].view(torch.int32)  # per (sequence, head)
    assert not counters.any()
    work = ws[128:136].view(torch.int32)  # item counter and done-CTA counter
    assert not work.any()
    assert ops.read_error_word(ws) == 0


def test_paged_attention_poisoned_table_sets_error_word_without_fault():
    rng = np.random.default_rng(6)
    B, H, D, bs = 4, 4, 64, 16
    ctx = np.array([20, 5, 40, 1], np.int32)
    tq, tk, tv, tt, tc, *_ = _random_paged(rng, B, H, D, bs, 16, ctx, torch.float16)
    tt[2, 1] = 10_000  # block id beyond the pool
    ws = ops.paged_attn_workspace(B, H, D, tt.shape[1], tq.device)
    ops.paged_decode_attention(tq, tk, tv, tt, tc, workspace=ws)
    assert ops.read_error_word(ws) & N.SPD_DEVERR_BLOCK_ID
    ws.zero_()
    tt[2, 1] = 0
    tc[0] = 16 * tt.shape[1] + 1  # longer than the table covers
    ops.paged_decode_attention(tq, tk, tv, tt, tc, workspace=ws)
    assert ops.read_error_word(ws) & N.SPD_DEVERR_LENGTH
    torch.cuda.synchronize()  # the context is still healthy


def test_paged_attention_in_cuda_graph():
    rng = np.random.default_rng(8)
    B, H, D, bs = 16, 12, 64, 16
    ctx = rng.integers(1, 300, B).astype(np.int32)
    nb = int(sum(-(-int(c) // bs) for c in ctx)) + 4
    tq, tk, tv, tt, tc, *_ = _random_paged(rng, B, H, D, bs, nb, ctx, torch.float16)
    ws = ops.paged_attn_workspace(B, H, D, tt.shape[1], tq.device)
    out = torch.empty_like(tq)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.paged_decode_attention(tq, tk, tv, tt, tc, out=out, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ops.paged_decode_attention(tq, tk, tv, tt, tc, out=out, workspace=ws)
    eager = ops.paged_decode_attention(tq, tk, tv, tt, tc)
    out.zero_()
    tc += 1  # replay sees new lengths written in place
    eager = ops.paged_decode_attention(tq, tk, tv, tt, tc)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


# ----------------------------------------------------------------------------- op (2)
@pytest.mark.parametrize("case", ["small", "whisper"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_cross_attention_matches_reference_golden(golden_dir, case, dtype):
    g = _case(np.load(golden_dir / "cross_attn_ref.npz"), case)
    out = ops.cross_attention(_t(g["q"], dtype), _t(g["k"], dtype), _t(g["v"], dtype), _t(g["valid_lens"]))
    err = _err(out, g["out"])
    assert err <= _tol(dtype), err


@pytest.mark.parametrize("D", [16, 32, 64, 128])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_cross_attention_matches_oracle(D, dtype):
    rng = np.random.default_rng(D)
    B, H, T = 7, 5, 1500
    valid = np.array([1500, 1, 0, 300, 1499, 129, 2000], np.int32)  # 2000 > T: clamped + flagged
    q = _t((rng.standard_normal((B, H, D)) * 0.5).astype(np.float32), dtype)
    k = _t((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32), dtype)
    v = _t((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float32), dtype)
    ws = ops.cross_attn_workspace(B, H, D, q.device)
    out = ops.cross_attention(q, k, v, _t(valid), workspace=ws)
    ref = O.cross_attention(_np32(q), _np32(k), _np32(v), np.minimum(valid, T))
    assert _err(out, ref) <= _tol(dtype)
    assert ops.read_error_word(ws) & N.SPD_DEVERR_LENGTH


def test_cross_attention_graph_slot_layout():
    """K/V read straight out of the graph-slot layout [S, L, 2, H, T, D] for layer l."""
    rng = np.random.default_rng(12)
    S, L, H, T, D = 3, 4, 6, 1500, 64
    slots = _t((rng.standard_normal((S, L, 2, H, T, D)) * 0.5).astype(np.float16))
    q = _t((rng.standard_normal((S, H, D)) * 0.5).astype(np.float16))
    valid = np.array([1500, 700, 33], np.int32)
    for l in (0, 3):
        k, v = slots[:, l, 0], slots[:, l, 1]
        out = ops.cross_attention(q, k, v, _t(valid))
        ref = O.cross_attention(_np32(q), _np32(k), _np32(v), valid)
        assert _err(out, ref) <= ATOL_16


@pytest.mark.parametrize("B,H,T,valid_fn", [
    (3, 4, 6000, lambda r, B: np.array([6000, 5999, 2177])),    # long contexts: 6 items of 8 units
    (300, 2, 1500, lambda r, B: r.integers(0, 200, B)),         # many one-item pairs, some empty
    (2, 3, 1500, lambda r, B: np.array([0, 0])),                # nothing to attend to
])
def test_cross_attention_item_queue_edges(B, H, T, valid_fn):
    """The dynamic item queue and the split-pair merge: item counts at the per-pair cap,
    many tiny pairs, empty batches; three calls in a row on one workspace (the queue
    counter is re-armed by each launch), the last one replayed from a CUDA graph."""
    rng = np.random.default_rng(B * 7 + T)
    D = 64
    valid = valid_fn(rng, B).astype(np.int32)
    q = _t((rng.standard_normal((B, H, D)) * 0.5).astype(np.float16))
    k = _t((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float16))
    v = _t((rng.standard_normal((B, H, T, D)) * 0.5).astype(np.float16))
    ref = O.cross_attention(_np32(q), _np32(k), _np32(v), valid)
    ws = ops.cross_attn_workspace(B, H, D, q.device)
    tv = _t(valid)
    out = torch.full_like(q, float("nan"))
    for _ in range(2):
        ops.cross_attention(q, k, v, tv, out=out, workspace=ws)
        assert _err(out, ref) <= ATOL_16
    out.fill_(float("nan"))
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        ops.cross_attention(q, k, v, tv, out=out, workspace=ws)
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert _err(out, ref) <= ATOL_16
    assert ops.read_error_word(ws) == 0


def test_cross_attention_config3_full_size():
    """B=128, H=20, D=64, 1500 positions, valid ~ U[300,1500], bf16."""
    g = torch.Generator().manual_seed(3)
    B, H, T, D = 128, 20, 1500, 64
    valid = torch.randint(300, 1501, (B,), generator=g, dtype=torch.int32)
    q = (torch.randn(B, H, D, generator=g) * 0.5).bfloat16()
    k = (torch.randn(B, H, T, D, generator=g) * 0.5).bfloat16()
    v = (torch.randn(B, H, T, D, generator=g) * 0.5).bfloat16()
    out = ops.cross_attention(q.cuda(), k.cuda(), v.cuda(), valid.cuda())
    bits = lambda t: t.view(torch.int16).numpy().view(np.uint16)
    ref = c_oracle.cross_attention(bits(q), bits(k), bits(v), valid.numpy(), 0.125, bf16=True)
    assert _err(out, ref) <= ATOL_16


# ----------------------------------------------------------------------------- op (3)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_kv_append_reproduces_reference_pools(golden_dir, dtype):
    g = np.load(golden_dir / "kv_write_ref.npz")
    bs = int(g["block_size"])
    for l in range(g["k_pools"].shape[0]):
        kp = torch.zeros(g["k_pools"].shape[1:], dtype=dtype, device=DEV)
        vp = torch.zeros_like(kp)
        for b in range(len(g["lens"])):
            t = int(g["lens"][b])
            tab = _t(np.where(g["tables"][b : b + 1] < 0, 0, g["tables"][b : b + 1]).astype(np.int32))
            ops.kv_append(_t(g["k_rows"][b : b + 1, l, :, :t], dtype), _t(g["v_rows"][b : b + 1, l, :, :t], dtype),
                          kp, vp, tab, _t(np.array([0], np.int32)))
        ref_k = torch.from_numpy(g["k_pools"][l]).to(dtype)
        ref_v = torch.from_numpy(g["v_pools"][l]).to(dtype)
        for b in range(len(g["lens"])):
            for pos in range(int(g["lens"][b])):
                blk = int(g["tables"][b, pos // bs])
                assert torch.equal(kp[blk, pos % bs].cpu(), ref_k[blk, pos % bs])
                assert torch.equal(vp[blk, pos % bs].cpu(), ref_v[blk, pos % bs])


def test_kv_append_strided_sources_skip_and_errors():
    rng = np.random.default_rng(13)
    B, H, T, D, bs, nb = 4, 6, 5, 64, 16, 32
    src = _t(rng.standard_normal((B, T, H, D)).astype(np.float16)).permute(0, 2, 1, 3)  # [B,H,T,D] strided
    kp = torch.zeros(nb, bs, H, D, dtype=torch.float16, device=DEV)
    vp = torch.zeros_like(kp)
    tables = _t(rng.permutation(nb)[: B * 2].reshape(B, 2).astype(np.int32))
    pos = _t(np.array([0, 14, -1, 3], np.int32))
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.kv_append(src, src, kp, vp, tables, pos, error_word=err)
    kp_ref = np.zeros((nb, bs, H, D), np.float16)
    O.kv_append(_np32(src).astype(np.float16), None, kp_ref, None, tables.cpu().numpy(), pos.cpu().numpy())
    assert np.array_equal(kp.cpu().numpy(), kp_ref)
    assert int(err.item()) == 0
    tables[1, 1] = 999
    ops.kv_append(src, src, kp, vp, tables, pos, error_word=err)
    assert int(err.item()) & N.SPD_DEVERR_BLOCK_ID


# ----------------------------------------------------------------------------- op (5)
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_block_gather_reproduces_reference(golden_dir, dtype):
    g = np.load(golden_dir / "block_gather_ref.npz")
    Tm = g["gathered_k"].shape[3]
    tab = _t(np.where(g["tables"] < 0, 0, g["tables"]).astype(np.int32))
    for l in range(g["k_pools"].shape[0]):
        out = ops.block_gather(_t(g["k_pools"][l], dtype), tab, _t(g["lens"]), Tm)
        assert torch.equal(out.cpu(), torch.from_numpy(g["gathered_k"][:, l]).to(dtype))
        # store direction: writing the encoder's K/V through op (3) rebuilds the pool rows
        pool = torch.zeros(g["k_pools"].shape[1:], dtype=dtype, device=DEV)
        for b in range(len(g["lens"])):
            t = int(g["lens"][b])
            ops.kv_append(_t(g["src_k"][b : b + 1, l, :, :t], dtype), None, pool, None, tab[b : b + 1],
                          _t(np.array([0], np.int32)))
        again = ops.block_gather(pool, tab, _t(g["lens"]), Tm)
        assert torch.equal(again, out)


def test_block_gather_into_slot_layout_and_padding():
    rng = np.random.default_rng(14)
    nb, bs, H, D = 200, 16, 4, 64
    pool = _t(rng.standard_normal((nb, bs, H, D)).astype(np.float16))
    B, T = 3, 1500
    lens = np.array([1500, 1, 300], np.int32)
    tab = np.zeros((B, 94), np.int32)
    for b in range(B):
        tab[b] = rng.choice(nb, 94, replace=False)
    slots = torch.full((B, 2, 2, H, T, D), 7.0, dtype=torch.float16, device=DEV)  # [S, L, 2, H, T, D]
    view = slots[:, 1, 0]
    ops.block_gather(pool, _t(tab), _t(lens), T, out=view)
    ref = O.block_gather(pool.cpu().numpy(), tab, lens, T)
    assert np.array_equal(view.cpu().numpy(), ref)
    assert torch.all(slots[:, 0] == 7.0) and torch.all(slots[:, 1, 1] == 7.0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("cols", [384, 768, 1280])
def test_add_layernorm_matches_add_then_layernorm(dtype, cols):
    """The fused residual add + LayerNorm: x_out is exactly the rounded sum, y matches
    torch's LayerNorm of it (one output rounding apart)."""
    torch.manual_seed(cols)
    rows = 37
    ln = torch.nn.LayerNorm(cols).to(DEV, dtype)
    with torch.no_grad():
        ln.weight.uniform_(0.5, 1.5)
        ln.bias.uniform_(-0.5, 0.5)
    x = torch.randn(rows, cols, device=DEV).to(dtype)
    d = torch.randn(rows, cols, device=DEV).to(dtype)
    ref_x = x + d
    ref_y = torch.nn.functional.layer_norm(ref_x.float(), (cols,), ln.weight.float(), ln.bias.float(), ln.eps)
    xo, y = ops.add_layernorm(x.clone(), d, ln)
    assert torch.equal(xo, ref_x)
    tol = {torch.float32: 1e-5, torch.float16: 4e-3, torch.bfloat16: 2e-2}[dtype]
    torch.testing.assert_close(y.float(), ref_y, atol=tol, rtol=0)
    _, y2 = ops.add_layernorm(ref_x.clone(), None, ln)
    torch.testing.assert_close(y2.float(), ref_y, atol=tol, rtol=0)
    # y into the leading columns of a wider buffer (the q/k/v GEMM input): same values,
    # the columns beyond untouched
    wide = torch.full((rows, cols + 8), 7.0, device=DEV, dtype=dtype)
    ops.add_layernorm(x.clone(), d, ln, out_y=wide[:, :cols])
    assert torch.equal(wide[:, :cols], y)
    assert bool((wide[:, cols:] == 7).all())


# ----------------------------------------------------------------------------- greedy pick
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("cols,ld", [(51865, 51904), (51866, 51866), (1000, 1003), (7, 8)])
def test_argmax_rows_matches_masked_torch_argmax(dtype, cols, ld):
    """spd_argmax_rows == torch.argmax(x[:, :cols].masked_fill(mask, -inf), -1): ties to the
    first column (values drawn from a few levels), masked columns, a NaN row, an all -inf
    row, unaligned row strides."""
    g = torch.Generator(device="cpu").manual_seed(cols + ld)
    rows = 67
    x = (torch.randint(0, 6, (rows, ld), generator=g).float() - 3.0).to(dtype).to(DEV)
    x[5, 17 % cols] = float("nan")
    x[5, 3 % cols] = float("nan")
    x[9, :] = float("-inf")
    mask = torch.zeros(cols, dtype=torch.bool)
    mask[torch.randint(0, cols, (max(1, cols // 50),), generator=g)] = True
    mask = mask.to(DEV)
    for m in (None, mask):
        ref = x[:, :cols] if m is None else x[:, :cols].masked_fill(m, float("-inf"))
        want = torch.argmax(ref, dim=-1)
        got = ops.argmax_rows(x, cols, m)
        assert torch.equal(got, want), (got - want).nonzero()[:5]
