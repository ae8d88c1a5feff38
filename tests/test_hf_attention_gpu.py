"""The drop-in forwards for a Hugging Face Whisper decoder's attention modules
(speech_serving.hf_attention), which replace the reference benchmark's patched
``self_attn.forward`` (scripts/evaluate_paging_variants.py:615-646) with ops 1+3 and the
cross-attention with op 2.  Teacher-forced decoding through the patched decoder must
follow the unpatched HF decoder with its own DynamicCache, step by step."""
import pytest
import torch

from speech_serving.hf_attention import PagedDecodeState, patch_decoder

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _hf(dtype, layers=2):
    from transformers import WhisperConfig, WhisperForConditionalGeneration

    cfg = WhisperConfig(vocab_size=51865, num_mel_bins=80, encoder_layers=2, decoder_layers=layers, d_model=256,
                        encoder_attention_heads=4, decoder_attention_heads=4, encoder_ffn_dim=1024,
                        decoder_ffn_dim=1024, max_source_positions=100, max_target_positions=448)
    torch.manual_seed(0)
    return WhisperForConditionalGeneration(cfg).to(DEV, dtype).eval()


@pytest.mark.parametrize("dtype,bs", [(torch.float16, 16), (torch.bfloat16, 16), (torch.float16, 8)])
def test_patched_decoder_follows_hf_dynamic_cache(dtype, bs):
    hf = _hf(dtype)
    dec = hf.model.decoder
    L, H = len(dec.layers), dec.layers[0].self_attn.num_heads
    D = dec.layers[0].self_attn.head_dim
    B, steps = 3, 40
    torch.manual_seed(1)
    with torch.no_grad():
        enc = hf.model.encoder(torch.randn(B, 80, 200, device=DEV, dtype=dtype)).last_hidden_state
        T = enc.shape[1]
        cross_k = [lay.encoder_attn.k_proj(enc).view(B, T, H, D).transpose(1, 2).contiguous() for lay in dec.layers]
        cross_v = [lay.encoder_attn.v_proj(enc).view(B, T, H, D).transpose(1, 2).contiguous() for lay in dec.layers]
    tokens = torch.randint(0, 51865, (B, steps), generator=torch.Generator().manual_seed(2)).to(DEV)
    tokens[:, 0] = 50258

    # reference: the HF decoder with its own cache, one token per step
    from transformers import DynamicCache, EncoderDecoderCache

    ref = []
    cache = EncoderDecoderCache(DynamicCache(), DynamicCache())
    with torch.no_grad():
        for i in range(steps):
            o = dec(input_ids=tokens[:, i:i + 1], encoder_hidden_states=enc, past_key_values=cache, use_cache=True)
            cache = o.past_key_values
            ref.append(o.last_hidden_state[:, 0].float())

    # patched: paged pools behind a random block table, cross K/V with valid lengths
    nblk = 64
    pools_k = [torch.zeros(nblk, bs, H, D, device=DEV, dtype=dtype) for _ in range(L)]
    pools_v = [torch.zeros(nblk, bs, H, D, device=DEV, dtype=dtype) for _ in range(L)]
    max_blocks = (steps + bs - 1) // bs
    tables = torch.randperm(nblk, generator=torch.Generator().manual_seed(3))[:B * max_blocks].view(B, max_blocks)
    state = PagedDecodeState(pools_k, pools_v, tables.to(DEV, torch.int32), torch.zeros(B, dtype=torch.int32, device=DEV),
                             cross_k=cross_k, cross_v=cross_v,
                             cross_lens=torch.full((B,), T, dtype=torch.int32, device=DEV))
    originals = [(lay.self_attn.forward, lay.encoder_attn.forward) for lay in dec.layers]
    handle = patch_decoder(dec, state)
    got = []
    try:
        with torch.no_grad():
            for i in range(steps):
                pos = torch.full((B, 1), i, dtype=torch.long, device=DEV)
                o = dec(input_ids=tokens[:, i:i + 1], encoder_hidden_states=enc, position_ids=pos, use_cache=False)
                state.advance()
                got.append(o.last_hidden_state[:, 0].float())
    finally:
        handle.restore()
    assert [(lay.self_attn.forward, lay.encoder_attn.forward) for lay in dec.layers] == originals
    assert state.context_lens.tolist() == [steps] * B

    tol = 0.03 if dtype == torch.float16 else 0.15
    for i, (a, b) in enumerate(zip(got, ref)):
        err = float((a - b).abs().max())
        assert err <= tol * max(1.0, float(b.abs().max())), (i, err)
    # the pools hold the K/V rows the HF cache holds, at the table's blocks
    for l in range(L):
        kc = cache.self_attention_cache.layers[l].keys.float()  # [B, H, steps, D]
        for b in range(B):
            rows = torch.cat([pools_k[l][int(tables[b, j])] for j in range(max_blocks)])[:steps]  # [steps, H, D]
            err = float((rows.float().permute(1, 0, 2) - kc[b]).abs().max())
            assert err <= tol * max(1.0, float(kc[b].abs().max())), (l, b, err)
