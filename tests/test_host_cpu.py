"""Host-side logic on CPU: pools and their allocation order, the dual cache, scheduler
admission and back-pressure, and the model definition pinned to the reference
(parameter fingerprint and greedy tokens of BASELINE config 1 from the reference run,
tests/golden/config1_tokens.json)."""
import json

import pytest
import torch

from speech_serving.block_manager import BlockManager
from speech_serving.dual_cache_manager import DualCacheManager
from speech_serving.encoder_block_manager import EncoderBlockManager
from speech_serving.graph_decode_buffers import batch_buckets
from speech_serving.memory_guard import MemoryGuard
from speech_serving.models import WhisperClassSpeechEncoderDecoderModel
from speech_serving.phase_aware_scheduler import (WHISPER_DEFAULT_PREFIX_TOKENS, PhaseAwareSpeechScheduler,
                                                  RequestPhase)


def _pools(enc_blocks=16, dec_blocks=16, bs=8, L=2, H=4, D=16):
    enc = EncoderBlockManager(L, H, D, bs, enc_blocks, dtype=torch.float32, device="cpu")
    dec = BlockManager(L, H, D, bs, dec_blocks, dtype=torch.float32, device="cpu")
    return enc, dec


def _tiny_model(vocab=256):
    return WhisperClassSpeechEncoderDecoderModel(2, 2, 4, 64, 80, vocab).eval()


# ----------------------------------------------------------------------------- pools
def test_block_manager_lifo_order_and_leaks():
    _, dec = _pools(dec_blocks=8)
    got = [dec.allocate_block() for _ in range(3)]
    assert got == [7, 6, 5]  # pops the end of the free list (reference block_manager.py:148)
    dec.free_blocks([6])
    assert dec.allocate_block() == 6
    dec.free_blocks(got + [6, 6])  # double free ignored
    assert dec.check_no_leaks() and dec.num_free_blocks == 8
    for _ in range(8):
        dec.allocate_block()
    with pytest.raises(RuntimeError, match="pool exhausted"):
        dec.allocate_block()


def test_block_manager_layout_is_one_allocation():
    _, dec = _pools()
    assert dec.key_pool[1].data_ptr() == dec.pool[1, 0].data_ptr()
    assert dec.key_pool[0].shape == (16, 8, 4, 16) and dec.key_pool[0].is_contiguous()
    t = dec.block_tables([[3, 1], [], [2]], max_blocks=4, device="cpu")
    assert t.dtype == torch.int32 and t.tolist() == [[3, 1, 0, 0], [0, 0, 0, 0], [2, 0, 0, 0]]
    with pytest.raises(ValueError):
        dec.block_tables([[1, 2, 3]], max_blocks=2, device="cpu")


def test_encoder_pool_fifo_refcounts_and_prefix_hits():
    enc, _ = _pools(enc_blocks=4)
    a, hit = enc.allocate_block("h0")
    assert (a, hit) == (0, False)
    b, hit = enc.allocate_block("h0")
    assert (b, hit) == (0, True) and enc.ref_counts[0] == 2
    c, _ = enc.allocate_block(None)
    assert c == 1  # FIFO from the front
    assert not enc.release_block(0) and enc.release_block(0)  # frees at count 0
    assert "h0" not in enc.prefix_hash_table
    assert enc.free_block_list[-1] == 0
    assert enc.hit_rate == pytest.approx(100 / 3, abs=0.01)


def test_dual_cache_rolls_back_partial_encoder_allocation():
    enc, dec = _pools(enc_blocks=3)
    dual = DualCacheManager(enc, dec)
    with pytest.raises(RuntimeError):
        dual.allocate_encoder_blocks(seq_len=8 * 4)  # 4 blocks from a pool of 3
    assert enc.allocated_block_count == 0
    table, hits = dual.allocate_encoder_blocks(seq_len=10)
    d = dual.allocate_decoder_block()
    out = dual.release_request_resources(table, [d])
    assert out == {"freed_encoder_blocks": 2, "freed_decoder_blocks": 1}
    assert enc.allocated_block_count == 0 and dec.allocated_block_count == 0


# ----------------------------------------------------------------------------- admission
def test_empty_pool_admission():
    """A request into an empty pool is always admitted (reference test_speech_engine.py:222)."""
    enc, dec = _pools()
    s = PhaseAwareSpeechScheduler(_tiny_model(), DualCacheManager(enc, dec), MemoryGuard(75.0), device="cpu")
    assert s.submit(torch.randn(80, 48), max_new_tokens=10) == 0
    req = s.queue[0]
    assert req.prompt_token_ids.tolist() == [[1]]  # small vocab: the generic start token
    assert req.phase == RequestPhase.QUEUED


def test_backpressure_counts_queued_demand_and_rejects():
    enc, dec = _pools(enc_blocks=16, dec_blocks=16)
    s = PhaseAwareSpeechScheduler(_tiny_model(), DualCacheManager(enc, dec), MemoryGuard(90.0), device="cpu")
    # each request: 24 encoder positions -> 3 blocks, 16 new tokens -> 2 decoder blocks
    ids = [s.submit(torch.randn(80, 48), max_new_tokens=16) for _ in range(6)]
    assert ids[:4] == [0, 1, 2, 3]  # 4 x 3 = 12 blocks = 75 %; the 5th would reach 93.75 %
    assert ids[4] is None and ids[5] is None
    assert s.rejected_requests_count == 2


def test_backpressure_evicts_retained_encoder_cache_first():
    enc, dec = _pools(enc_blocks=16, dec_blocks=64)
    guard = MemoryGuard(90.0, enable_periodic_gc=False)
    s = PhaseAwareSpeechScheduler(_tiny_model(), DualCacheManager(enc, dec), guard, device="cpu",
                                  retain_encoder_cache=True)
    # a retained cache entry holding 12 blocks, as left behind by a finished request
    table = [enc.allocate_block(None)[0] for _ in range(12)]
    s._full_input_enc_cache["x"] = {"block_table": table, "enc_seq_len": 96, "last_access_time": 0.0,
                                    "held_by_cache": True, "encode_time": 0.0}
    assert s.submit(torch.randn(80, 48), max_new_tokens=8) == 0
    assert enc.allocated_block_count == 0 and guard.eviction_events_count == 1
    assert s.get_encoder_telemetry()["full_input_cache_entries"] == 0


def test_full_input_hash_is_exact():
    a = torch.randn(1, 80, 40)
    b = a.clone()
    b[0, 0, 0] += 1e-6
    h = PhaseAwareSpeechScheduler._compute_full_input_hash
    assert h(a) == h(a.clone()) and h(a) != h(b)


def test_whisper_prompt_and_eos_defaults():
    enc, dec = _pools()
    m = WhisperClassSpeechEncoderDecoderModel(1, 1, 4, 64, 80, 51865).eval()
    s = PhaseAwareSpeechScheduler(m, DualCacheManager(enc, dec), device="cpu")
    s.submit(torch.randn(80, 16), max_new_tokens=4)
    assert s.queue[0].prompt_token_ids.tolist() == [WHISPER_DEFAULT_PREFIX_TOKENS]
    assert s.queue[0].eos_token_id == 50257


def test_graph_direct_encoder_kv_needs_graph_mode():
    enc, dec = _pools()
    with pytest.raises(ValueError):
        PhaseAwareSpeechScheduler(_tiny_model(), DualCacheManager(enc, dec), device="cpu",
                                  graph_direct_encoder_kv=True)


def test_batch_buckets():
    assert batch_buckets(4) == [1, 2, 4]
    assert batch_buckets(32) == [1, 2, 4, 8, 16, 32]
    assert batch_buckets(6) == [1, 2, 4, 6]


# ----------------------------------------------------------------------------- model pinned to the reference
def _config1():
    return json.loads((__import__("pathlib").Path(__file__).parent / "golden" / "config1_tokens.json").read_text())


def test_model_parameters_match_reference_init():
    """Same module order and shapes as the reference: seed 0 gives the same weights."""
    g = _config1()
    torch.manual_seed(0)
    m = WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865)
    sd = m.state_dict()
    assert list(sd) == list(g["param_fingerprint"])
    for name, (s, a) in g["param_fingerprint"].items():
        p = sd[name].double()
        assert float(p.sum()) == pytest.approx(s, rel=1e-9, abs=1e-9), name
        assert float(p.abs().sum()) == pytest.approx(a, rel=1e-9), name


def _config1_inputs():
    g = torch.Generator().manual_seed(1)
    return [torch.randn(80, 3000, generator=g).clamp(-1.5, 1.5) for _ in range(4)]


def test_eager_model_tokens_match_reference_config1():
    """The PyTorch model (encode + prompt prefill + incremental decode_step) reproduces the
    reference scheduler's greedy tokens for config 1 on CPU in fp32.  The GPU scheduler
    tests compare the kernels' tokens with the same golden."""
    g = _config1()
    torch.manual_seed(0)
    m = WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865).eval()
    mels = torch.stack(_config1_inputs())
    with torch.no_grad():
        _, enc_kv = m.encode(mels)  # batched, as the reference's batch_encoder run
        ids = torch.tensor([g["prompt"]] * 4)
        out = m.decode_step(ids, encoder_past_kv_list=enc_kv)
        toks = [out.logits[:, -1].argmax(-1)]
        kv = out.past_key_values
        for _ in range(g["max_new_tokens"] - 1):
            out = m.decode_step(toks[-1][:, None], past_key_values=kv, encoder_past_kv_list=enc_kv)
            kv = out.past_key_values
            toks.append(out.logits[:, -1].argmax(-1))
    got = torch.stack(toks, 1).tolist()
    agree = sum(a == b for ga, gb in zip(got, g["tokens"]) for a, b in zip(ga, gb))
    assert agree / (4 * g["max_new_tokens"]) >= 0.99, (got, g["tokens"])


def test_pretrained_whisper_prefill_matches_hf_decoder():
    """The HF wrapper's encode (fp32: per-layer projections) and multi-token decode_step
    reproduce the HF decoder's logits, including an incremental step from its cache."""
    from transformers import WhisperConfig

    from speech_serving.models import PretrainedWhisperModel

    cfg = WhisperConfig(vocab_size=51865, num_mel_bins=80, encoder_layers=2, decoder_layers=2, d_model=256,
                        encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=1024,
                        decoder_ffn_dim=1024, max_source_positions=100, max_target_positions=448,
                        pad_token_id=50257, bos_token_id=50257, eos_token_id=50257, decoder_start_token_id=50258)
    m = PretrainedWhisperModel(config=cfg, device="cpu", dtype=torch.float32, seed=0)
    hf = m.hf_model
    mel = torch.randn(1, 80, 200, generator=torch.Generator().manual_seed(2))
    ids = torch.tensor([WHISPER_DEFAULT_PREFIX_TOKENS])
    with torch.no_grad():
        e, kv = m.encode(mel)
        out = m.decode_step(ids, encoder_past_kv_list=kv)
        ref = hf.proj_out(hf.model.decoder(input_ids=ids, encoder_hidden_states=e).last_hidden_state)
        torch.testing.assert_close(out.logits, ref, atol=1e-5, rtol=1e-5)
        t = out.logits[:, -1].argmax(-1, keepdim=True)
        o2 = m.decode_step(t, past_key_values=out.past_key_values, encoder_past_kv_list=kv)
        ids2 = torch.cat([ids, t], 1)
        ref2 = hf.proj_out(hf.model.decoder(input_ids=ids2, encoder_hidden_states=e).last_hidden_state)
        torch.testing.assert_close(o2.logits[:, -1], ref2[:, -1], atol=1e-5, rtol=1e-5)
    assert [l.keys.shape[2] for l in o2.past_key_values.layers] == [5, 5]


def test_hf_attention_patch_swaps_and_restores_forwards():
    """patch_decoder replaces self_attn / encoder_attn forwards of every decoder layer and
    the handle puts the originals back (reference: scripts/evaluate_paging_variants.py:
    613-646 and its restore loop); a bad state is refused on the host."""
    from transformers import WhisperConfig, WhisperForConditionalGeneration

    from speech_serving.hf_attention import PagedDecodeState, patch_decoder

    cfg = WhisperConfig(vocab_size=100, num_mel_bins=80, encoder_layers=1, decoder_layers=2, d_model=64,
                        encoder_attention_heads=2, decoder_attention_heads=2, encoder_ffn_dim=128,
                        decoder_ffn_dim=128, max_source_positions=16, max_target_positions=32, pad_token_id=0,
                        bos_token_id=1, eos_token_id=1, decoder_start_token_id=2)
    dec = WhisperForConditionalGeneration(cfg).model.decoder
    pools = [torch.zeros(4, 16, 2, 32) for _ in range(2)]
    tables, lens = torch.zeros(3, 2, dtype=torch.int32), torch.zeros(3, dtype=torch.int32)
    ck = [torch.zeros(3, 2, 16, 32) for _ in range(2)]
    state = PagedDecodeState(pools, pools, tables, lens, cross_k=ck, cross_v=ck,
                             cross_lens=torch.full((3,), 16, dtype=torch.int32))
    before = [(lay.self_attn.forward, lay.encoder_attn.forward) for lay in dec.layers]
    handle = patch_decoder(dec, state)
    assert all(lay.self_attn.forward != b[0] and lay.encoder_attn.forward != b[1]
               for lay, b in zip(dec.layers, before))
    with pytest.raises(RuntimeError):  # one new token per sequence
        dec.layers[0].self_attn(torch.zeros(3, 2, 64))
    handle.restore()
    assert [(lay.self_attn.forward, lay.encoder_attn.forward) for lay in dec.layers] == before
    state.advance(2)
    assert state.context_lens.tolist() == [2, 2, 2]
    with pytest.raises(ValueError):
        PagedDecodeState(pools, pools, tables.long(), lens)
    with pytest.raises(ValueError):
        patch_decoder(dec, PagedDecodeState(pools[:1], pools[:1], tables, lens), cross=False)
    with pytest.raises(ValueError):
        patch_decoder(dec, PagedDecodeState(pools, pools, tables, lens), cross=True)


def test_qkv_bias_row_matches_separate_projections():
    """The decode step's q/k/v GEMM carries the biases as one more weight row against a
    ones column of its input: the same values as the three Linear layers (fp32, CPU)."""
    from speech_serving.models import _fused_qkv_aug, _qkv_input

    torch.manual_seed(5)
    d, hd, n = 64, 64, 5
    q, k, v = torch.nn.Linear(d, hd), torch.nn.Linear(d, hd, bias=False), torch.nn.Linear(d, hd)
    holder = torch.nn.Module()
    w = _fused_qkv_aug(holder, [(q, k, v)], q_scale=0.125)[0]
    assert w.shape == (3, d + 8, hd)
    h = torch.randn(n, d)
    buf = _qkv_input(holder, n, d, h)
    assert buf.shape == (n, d + 8) and bool((buf[:, d] == 1).all()) and bool((buf[:, d + 1:] == 0).all())
    buf[:, :d] = h
    got = torch.bmm(buf.unsqueeze(0).expand(3, n, d + 8), w)
    with torch.no_grad():
        want = torch.stack([q(h) * 0.125, k(h), v(h)])
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
    assert _qkv_input(holder, n, d, h) is buf  # one buffer per batch size


# ----------------------------------------------------------------------------- HF parity reference
def test_hf_greedy_reference_matches_plain_hf_decoding():
    """hf_greedy_tokens (cross K/V projected once, cached HF decoder steps) gives the same
    tokens as the HF decoder re-run over the whole prefix with the encoder states."""
    from transformers import WhisperConfig

    from speech_serving.hf_reference import hf_greedy_tokens, sequence_agreement
    from speech_serving.models import PretrainedWhisperModel

    cfg = WhisperConfig(vocab_size=320, num_mel_bins=16, encoder_layers=2, decoder_layers=2, d_model=64,
                        encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=128,
                        max_source_positions=20, max_target_positions=64, pad_token_id=300, bos_token_id=301,
                        eos_token_id=301, decoder_start_token_id=302, init_std=0.2)
    model = PretrainedWhisperModel(config=cfg, device="cpu", dtype=torch.float32, seed=0)
    torch.manual_seed(1)
    mels = torch.randn(3, 16, 40)
    prompt = [302, 303]
    got = hf_greedy_tokens(model, mels, prompt, [6, 4, 5], batch=2)
    hf = model.hf_model
    want = []
    with torch.no_grad():
        for m, n in zip(mels, [6, 4, 5]):
            e = hf.model.encoder(m[None]).last_hidden_state
            toks = []
            for _ in range(n):
                h = hf.model.decoder(input_ids=torch.tensor([prompt + toks]), encoder_hidden_states=e).last_hidden_state
                toks.append(int(hf.proj_out(h[0, -1]).argmax()))
            want.append(toks)
    assert got == want
    a = sequence_agreement(got, [want[0], want[1][:3] + [want[1][3] + 1], want[2]])
    assert a["identical"] == 2 and a["first_divergence"] == [3]


def test_hf_margins_and_near_tie_classification():
    """hf_top2_margins teacher-forces ragged sequences (right-padded in a batch) and gives
    each position's HF top-1 minus top-2 logit; on HF's own greedy sequences every top-1 is
    the sequence's token, so every margin is >= 0 and equals the one from an unbatched
    pass.  near_tie_divergences marks a divergence as a near-tie only within the given
    number of grid steps of the top-1 logit."""
    from transformers import WhisperConfig

    from speech_serving.hf_reference import grid_step, hf_greedy_tokens, hf_top2_margins, near_tie_divergences
    from speech_serving.models import PretrainedWhisperModel

    cfg = WhisperConfig(vocab_size=320, num_mel_bins=16, encoder_layers=2, decoder_layers=2, d_model=64,
                        encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=128,
                        max_source_positions=20, max_target_positions=64, pad_token_id=300, bos_token_id=301,
                        eos_token_id=301, decoder_start_token_id=302, init_std=0.2)
    model = PretrainedWhisperModel(config=cfg, device="cpu", dtype=torch.float32, seed=0)
    torch.manual_seed(2)
    mels = torch.randn(3, 16, 40)
    prompt = [302, 303]
    ref = hf_greedy_tokens(model, mels, prompt, [6, 3, 5], batch=3)
    m3 = hf_top2_margins(model, mels, prompt, ref, batch=3)
    m1 = hf_top2_margins(model, mels, prompt, ref, batch=1)
    assert [len(r) for r in m3] == [6, 3, 5]
    for ra, rb in zip(m3, m1):
        for (ma, ta), (mb, tb) in zip(ra, rb):
            assert ma >= 0 and abs(ma - mb) < 1e-4 and abs(ta - tb) < 1e-4
    assert grid_step(3.0, torch.bfloat16) == 2.0 ** -6 and grid_step(3.0, torch.float16) == 2.0 ** -9
    ours = [list(ref[0]), ref[1][:1] + [ref[1][1] + 1] + ref[1][2:], list(ref[2])]
    margin, top = m3[1][1]
    wide = near_tie_divergences(ours, ref, m3, torch.float32, steps=int(margin / grid_step(top, torch.float32)) + 2)
    assert wide["at_near_tie"] == 1 and wide["divergences"][0]["position"] == 1
    tight = near_tie_divergences(ours, ref, m3, torch.float32, steps=0)
    assert tight["at_near_tie"] == 0 and tight["requests_without_near_tie"] == 3
    assert tight["identical_without_near_tie"] == 2
