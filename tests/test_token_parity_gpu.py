"""Request-level greedy-token parity of the serving path in 16-bit, at the serving
configurations' model dimensions.

The reference's serving gate (scripts/test_parity_graph.py:70-86, with the match counted
in scripts/evaluate_real_speech.py:723-725) requires >= 99 % of requests to produce
exactly the token list of the HF decoder.  Here 64 requests per configuration — synthetic
log-mels of audio U[2, 30] s zero-padded to 3000 frames, 64 new tokens, EOS disabled — go
through the repository's graph decode path with direct handoff (encoder + op-4
projection into the slots, the paged/cross kernels in CUDA graphs); the same requests are
decoded greedily by the unpatched HF decoder (speech_serving.hf_reference, the reference's
PretrainedWhisperModel arithmetic) on the same device, dtype and seeded random-init
weights, and whole sequences are compared.

Random-init weights (Whisper's init_std 0.02) make the first token's margin over the
runner-up large, so sequences are long runs of a few tokens; a divergence can only come
from a near-tie.  Every mismatch is reported with the HF margin at its first divergent
position."""
import pytest
import torch

from speech_serving.block_manager import BlockManager
from speech_serving.dual_cache_manager import DualCacheManager
from speech_serving.encoder_block_manager import EncoderBlockManager
from speech_serving.hf_reference import hf_greedy_tokens, sequence_agreement
from speech_serving.memory_guard import MemoryGuard
from speech_serving.models import PretrainedWhisperModel
from speech_serving.phase_aware_scheduler import WHISPER_DEFAULT_PREFIX_TOKENS, PhaseAwareSpeechScheduler
from speech_serving.serving import run_engine, synthetic_requests, whisper_config

pytestmark = pytest.mark.gpu
DEV = "cuda"
N_REQ, N_TOK = 64, 64


def _engine(model, dtype):
    L, H, D = model.num_decoder_layers, model.num_heads, model.head_dim
    enc = EncoderBlockManager(L, H, D, 16, 1, dtype=dtype, device=DEV)
    dec = BlockManager(L, H, D, 16, N_REQ * 6 + 16, dtype=dtype, device=DEV)
    return PhaseAwareSpeechScheduler(model, DualCacheManager(enc, dec), MemoryGuard(), max_batch_size=64, device=DEV,
                                     eos_token_id=-1, batch_encoder=True, graph_decode=True, graph_readback_k=4,
                                     graph_direct_encoder_kv=True), dec


def _margin_at(model, mel, prompt, prefix):
    """HF top-1 minus top-2 logit (and the top two ids) after prompt + prefix."""
    hf = model.hf_model
    with torch.no_grad():
        e = hf.model.encoder(mel[None].to(DEV, model.dtype)).last_hidden_state
        ids = torch.tensor([list(prompt) + list(prefix)], device=DEV)
        h = hf.model.decoder(input_ids=ids, encoder_hidden_states=e).last_hidden_state[0, -1]
        lg = hf.proj_out(h).float()
        if model.suppress_mask is not None:
            lg = lg.masked_fill(model.suppress_mask, float("-inf"))
        top = lg.topk(2)
    return float(top.values[0] - top.values[1]), top.indices.tolist()


@pytest.mark.parametrize("arch,dtype,n_mels", [("whisper-small", torch.float16, 80),
                                               ("whisper-large-v3", torch.bfloat16, 128)])
def test_serving_sequences_match_hf_decoder(arch, dtype, n_mels):
    model = PretrainedWhisperModel(config=whisper_config(arch), device=DEV, dtype=dtype, seed=0)
    reqs = synthetic_requests(N_REQ, n_mels, seed=2024, out_lo=N_TOK, out_hi=N_TOK)
    sched, dec = _engine(model, dtype)
    prompt = WHISPER_DEFAULT_PREFIX_TOKENS
    r = run_engine(sched, reqs, prompt)
    assert r["requests"] == N_REQ and r["failed"] == 0
    ours = r["tokens_by_request"]
    assert all(t is not None and len(t) == N_TOK for t in ours)
    mels = torch.stack([q.mel for q in reqs])
    ref = hf_greedy_tokens(model, mels, prompt, N_TOK, batch=32)
    agree = sequence_agreement(ours, ref)
    report = []
    for i, (a, b) in enumerate(zip(ours, ref)):
        if a != b:
            k = next(j for j, (x, y) in enumerate(zip(a, b)) if x != y)
            m, top = _margin_at(model, reqs[i].mel, prompt, b[:k])
            report.append({"request": i, "first_divergence": k, "ours": a[k], "hf": b[k], "hf_margin": round(m, 5),
                           "hf_top2": top})
    print(f"{arch} {dtype}: {agree['identical']}/{agree['requests']} sequences identical; mismatches: {report}")
    assert dec.allocated_block_count == 0
    assert agree["identical_frac"] >= 0.99, report
