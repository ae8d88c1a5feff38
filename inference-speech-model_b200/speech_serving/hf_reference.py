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

import math
from typing import List, Sequence, Tuple, Union

import torch

# A divergence counts as a near-tie when the HF decoder's own top-1 minus top-2 logit at
# that position is within this many steps of the dtype's grid at the top-1 magnitude.
NEAR_TIE_STEPS = 8


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


@torch.no_grad()
def hf_top2_margins(model, mels: torch.Tensor, prompt: Sequence[int], seqs: Sequence[Sequence[int]],
                    batch: int = 16) -> List[List[Tuple[float, float]]]:
    """For every request, the HF decoder's (top-1 minus top-2 logit, top-1 logit) at each
    position of ``seqs``, teacher-forced on the prompt and the sequence so far, in the
    model's dtype with the suppress mask applied."""
    hf = model.hf_model
    dev = next(hf.parameters()).device
    dtype = next(hf.parameters()).dtype
    suppress = getattr(model, "suppress_mask", None)
    out: List[List[Tuple[float, float]]] = []
    for lo in range(0, len(seqs), batch):
        hi = min(len(seqs), lo + batch)
        group = seqs[lo:hi]
        width = max(len(s) for s in group)
        # ragged sequences are right-padded with their own last token; the padded tail is
        # causal-masked away from the positions that are kept
        ids = torch.tensor([list(prompt) + list(s[:-1]) + [s[-1]] * (width - len(s)) for s in group], device=dev)
        e = hf.model.encoder(mels[lo:hi].to(dev, dtype)).last_hidden_state
        h = hf.model.decoder(input_ids=ids, encoder_hidden_states=e).last_hidden_state[:, len(prompt) - 1:]
        lg = hf.proj_out(h)
        if suppress is not None:
            lg = lg.masked_fill(suppress, float("-inf"))
        top = lg.float().topk(2, dim=-1).values
        for s, marg, best in zip(group, (top[..., 0] - top[..., 1]).tolist(), top[..., 0].tolist()):
            out.append(list(zip(marg, best))[:len(s)])
    return out


def grid_step(x: float, dtype) -> float:
    """Spacing of ``dtype`` numbers at magnitude |x|."""
    return float(torch.finfo(dtype).eps) * 2.0 ** math.floor(math.log2(max(abs(x), 1e-30)))


def near_tie_divergences(ours: Sequence[Sequence[int]], ref: Sequence[Sequence[int]],
                         margins: Sequence[Sequence[Tuple[float, float]]], dtype,
                         steps: int = NEAR_TIE_STEPS) -> dict:
    """Classify where ``ours`` leaves the HF sequences ``ref``: each first divergence with
    the HF top-2 margin there (in grid steps of ``dtype``) and whether it is a near-tie,
    plus how the requests whose HF path has no near-tie at all agree."""
    near = [[m <= steps * grid_step(top, dtype) for m, top in row] for row in margins]
    div = []
    for i, (a, b) in enumerate(zip(ours, ref)):
        if list(a) != list(b):
            k = next((j for j, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))
            if k >= len(margins[i]):
                div.append({"request": i, "position": k, "near_tie": False, "length_mismatch": True})
                continue
            m, top = margins[i][k]
            div.append({"request": i, "position": k, "ours": int(a[k]), "hf": int(b[k]), "hf_margin": round(m, 5),
                        "steps": round(m / grid_step(top, dtype), 2), "near_tie": bool(near[i][k])})
    clean = [i for i in range(len(ref)) if not any(near[i])]
    return {"divergences": div, "at_near_tie": sum(d["near_tie"] for d in div),
            "requests_without_near_tie": len(clean),
            "identical_without_near_tie": sum(list(ours[i]) == list(ref[i]) for i in clean)}
