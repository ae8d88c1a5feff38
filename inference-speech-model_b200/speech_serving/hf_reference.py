"""Greedy tokens from the unpatched Hugging Face Whisper decoder: the parity reference for
the serving path.

The reference engine's HF path (speech_serving/models.py:545-610 of the reference) runs
the HF encoder, projects every decoder layer's cross K/V with that layer's
``encoder_attn.k_proj`` / ``v_proj`` (cuBLAS, one pair of GEMMs per layer), then steps the
HF ``WhisperDecoder`` with an ``EncoderDecoderCache`` (self: DynamicCache grown each step;
cross: the projections, marked as already computed), applies ``proj_out``, the
``suppress_tokens`` mask and argmax.  ``hf_greedy_tokens`` runs exactly that arithmetic,
batched, on the model's own device and dtype, and returns what a greedy request gets
back: ``max_new_tokens`` tokens, the first one from the prompt forward.  The reference's
serving-parity gate compares whole sequences against such HF tokens
(scripts/evaluate_real_speech.py:723-725: a request matches when its token list is equal).

Nothing here touches the B200 kernels; it is the checker for them.
"""
from __future__ import annotations

from typing import List, Sequence, Union

import torch


@torch.no_grad()
def hf_greedy_tokens(model, mels: torch.Tensor, prompt: Sequence[int], max_new_tokens: Union[int, Sequence[int]],
                     batch: int = 64) -> List[List[int]]:
    """Greedy sequences of ``mels`` ([N, n_mels, frames]) through ``model.hf_model``
    (a ``PretrainedWhisperModel``), ``batch`` requests at a time, with EOS ignored."""
    from transformers.cache_utils import DynamicCache, EncoderDecoderCache

    hf = model.hf_model
    dev = next(hf.parameters()).device
    dtype = next(hf.parameters()).dtype
    n = mels.shape[0]
    lens = [int(max_new_tokens)] * n if isinstance(max_new_tokens, int) else [int(x) for x in max_new_tokens]
    H = hf.config.decoder_attention_heads
    D = hf.config.d_model // H
    suppress = getattr(model, "suppress_mask", None)
    out: List[List[int]] = []
    for lo in range(0, n, batch):
        hi = min(n, lo + batch)
        b = hi - lo
        enc = hf.model.encoder(mels[lo:hi].to(dev, dtype)).last_hidden_state
        T = enc.shape[1]
        cross = DynamicCache()
        for l, layer in enumerate(hf.model.decoder.layers):
            k = layer.encoder_attn.k_proj(enc).view(b, T, H, D).transpose(1, 2).contiguous()
            v = layer.encoder_attn.v_proj(enc).view(b, T, H, D).transpose(1, 2).contiguous()
            cross.update(k, v, layer_idx=l)
        cache = EncoderDecoderCache(DynamicCache(), cross)
        for l in range(len(hf.model.decoder.layers)):
            cache.is_updated[l] = True
        placeholder = torch.empty((b, T, hf.config.d_model), device=dev, dtype=dtype)
        ids = torch.tensor([list(prompt)] * b, dtype=torch.long, device=dev)
        steps = max(lens[lo:hi])
        toks = torch.empty((b, steps), dtype=torch.long, device=dev)
        for i in range(steps):
            o = hf.model.decoder(input_ids=ids, encoder_hidden_states=placeholder, past_key_values=cache,
                                 use_cache=True)
            logits = hf.proj_out(o.last_hidden_state[:, -1])
            if suppress is not None:
                logits = logits.masked_fill(suppress, float("-inf"))
            nxt = logits.argmax(dim=-1)
            toks[:, i] = nxt
            ids = nxt[:, None]
            cache = o.past_key_values
        rows = toks.tolist()
        out.extend(r[:lens[lo + j]] for j, r in enumerate(rows))
    return out


def sequence_agreement(ours: Sequence[Sequence[int]], ref: Sequence[Sequence[int]]) -> dict:
    """Fraction of requests whose whole token sequence equals the reference's, and the
    first divergent position of each request that differs."""
    if len(ours) != len(ref):
        raise ValueError(f"{len(ours)} sequences against {len(ref)}")
    firsts = []
    for a, b in zip(ours, ref):
        if list(a) != list(b):
            k = next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))
            firsts.append(k)
    n = len(ours)
    return {"requests": n, "identical": n - len(firsts), "identical_frac": (n - len(firsts)) / n if n else 1.0,
            "first_divergence": firsts}
