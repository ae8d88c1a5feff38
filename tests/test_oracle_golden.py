"""Pins the CPU oracle to golden vectors produced by the reference itself
(tests/golden/make_golden.py) and checks the C port of the oracle against it."""
import numpy as np
import pytest

from oracle import attention_oracle as O
from oracle import c_oracle


def _case(npz, name):
    return {k.split("__", 1)[1]: npz[k] for k in npz.files if k.startswith(name + "__")}


@pytest.mark.parametrize("case", ["small", "whisper"])
def test_paged_attention_oracle_matches_reference(golden_dir, case):
    g = _case(np.load(golden_dir / "paged_attn_ref.npz"), case)
    out = O.paged_decode_attention(g["q"], g["k_pool"], g["v_pool"], g["block_tables"], g["context_lens"])
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=1e-5)
    # context 0 rows are exactly zero, like the reference kernel's untouched output
    for b in np.flatnonzero(g["context_lens"] == 0):
        assert not out[b].any()


@pytest.mark.parametrize("case", ["small", "whisper"])
def test_cross_attention_oracle_matches_reference(golden_dir, case):
    g = _case(np.load(golden_dir / "cross_attn_ref.npz"), case)
    out = O.cross_attention(g["q"], g["k"], g["v"], g["valid_lens"])
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=1e-5)


def test_kv_write_oracle_reproduces_reference_pools(golden_dir):
    g = np.load(golden_dir / "kv_write_ref.npz")
    L = g["k_pools"].shape[0]
    for l in range(L):
        kp = np.zeros_like(g["k_pools"][l])
        vp = np.zeros_like(g["v_pools"][l])
        T = g["k_rows"].shape[3]
        for b in range(len(g["lens"])):
            t = int(g["lens"][b])
            O.kv_append(g["k_rows"][b : b + 1, l, :, :t], g["v_rows"][b : b + 1, l, :, :t], kp, vp,
                        g["tables"][b : b + 1], np.array([0], np.int32))
        used = sorted({int(x) for x in g["tables"].ravel() if x >= 0})
        # every written row is bit-identical to the reference's pool
        for b in range(len(g["lens"])):
            t = int(g["lens"][b])
            bs = int(g["block_size"])
            for pos in range(t):
                blk = int(g["tables"][b, pos // bs])
                assert np.array_equal(kp[blk, pos % bs], g["k_pools"][l][blk, pos % bs])
                assert np.array_equal(vp[blk, pos % bs], g["v_pools"][l][blk, pos % bs])
        assert used


def test_block_gather_oracle_reproduces_reference(golden_dir):
    g = np.load(golden_dir / "block_gather_ref.npz")
    L = g["k_pools"].shape[0]
    Tm = g["gathered_k"].shape[3]
    for l in range(L):
        gk = O.block_gather(g["k_pools"][l], g["tables"], g["lens"], Tm)
        gv = O.block_gather(g["v_pools"][l], g["tables"], g["lens"], Tm)
        assert np.array_equal(gk, g["gathered_k"][:, l])
        assert np.array_equal(gv, g["gathered_v"][:, l])
        # the gather of what the scheduler stored equals the encoder's own K/V
        assert np.array_equal(gk, g["src_k"][:, l])


def test_cross_kv_project_oracle_matches_reference(golden_dir):
    g = np.load(golden_dir / "cross_kv_project_ref.npz")
    L = len([k for k in g.files if k.startswith("wk")])
    res = O.cross_kv_project(g["enc_out"], [g[f"wk{l}"] for l in range(L)], [g[f"wv{l}"] for l in range(L)],
                             [g[f"bv{l}"] for l in range(L)], H=g["k0"].shape[1])
    for l in range(L):
        np.testing.assert_allclose(res[l][0], g[f"k{l}"], atol=1e-5, rtol=1e-5)
        np.testing.assert_allclose(res[l][1], g[f"v{l}"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_c_oracle_matches_numpy_oracle(dtype):
    rng = np.random.default_rng(3)
    B, H, D, bs, nb = 6, 3, 64, 16, 64
    q = (rng.standard_normal((B, H, D)) * 0.5).astype(dtype)
    kp = (rng.standard_normal((nb, bs, H, D)) * 0.5).astype(dtype)
    vp = (rng.standard_normal((nb, bs, H, D)) * 0.5).astype(dtype)
    tab = rng.permutation(nb)[: B * 10].reshape(B, 10).astype(np.int32)
    ctx = np.array([1, 16, 17, 0, 160, 99], np.int32)
    a = O.paged_decode_attention(q, kp, vp, tab, ctx, 0.125)
    b = c_oracle.paged_decode_attention(q, kp, vp, tab, ctx, 0.125, threads=2)
    np.testing.assert_allclose(a, b, atol=1e-6)
    k = (rng.standard_normal((B, H, 70, D))).astype(dtype)
    v = (rng.standard_normal((B, H, 70, D))).astype(dtype)
    val = np.array([70, 1, 0, 35, 200, 69], np.int32)
    np.testing.assert_allclose(O.cross_attention(q, k, v, val, 0.125),
                               c_oracle.cross_attention(q, k, v, val, 0.125, threads=2), atol=1e-6)


def test_oracle_flags_planted_mistake():
    """A wrong block table in the oracle changes its answer: the parity tests can fail."""
    rng = np.random.default_rng(4)
    q = rng.standard_normal((1, 2, 16)).astype(np.float32)
    kp = rng.standard_normal((4, 8, 2, 16)).astype(np.float32)
    vp = rng.standard_normal((4, 8, 2, 16)).astype(np.float32)
    good = O.paged_decode_attention(q, kp, vp, np.array([[0, 1]], np.int32), np.array([12], np.int32))
    bad = O.paged_decode_attention(q, kp, vp, np.array([[0, 2]], np.int32), np.array([12], np.int32))
    assert np.abs(good - bad).max() > 1e-3


def test_eager_decode_oracle_reproduces_reference_config1(golden_dir):
    """The CPU eager-decode oracle, given the seed-0 weights of the config-1 model,
    reproduces the reference scheduler's greedy tokens (tests/golden/config1_tokens.json)."""
    import json

    import torch

    from oracle import eager_decode
    from speech_serving.models import WhisperClassSpeechEncoderDecoderModel

    g = json.loads((golden_dir / "config1_tokens.json").read_text())
    torch.manual_seed(0)
    sd = WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865).state_dict()
    gen = torch.Generator().manual_seed(1)
    mels = torch.stack([torch.randn(80, 3000, generator=gen).clamp(-1.5, 1.5) for _ in range(4)])
    got = eager_decode.greedy_decode(sd, mels, g["prompt"], g["max_new_tokens"], num_heads=6)
    n = sum(len(t) for t in g["tokens"])
    agree = sum(a == b for ga, gb in zip(got, g["tokens"]) for a, b in zip(ga, gb))
    assert agree / n >= 0.99
