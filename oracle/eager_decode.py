"""CPU oracle for end-to-end greedy decoding of the Whisper-class model — TEST
INFRASTRUCTURE, not product code.

Restates the reference engine's eager path on CPU with plain torch tensor arithmetic
(F.linear / matmul / softmax / layer_norm), reading the weights from a state dict whose
names are the reference model's (speech_serving/models.py:298-347):

* encoder front end and layers: models.py:349-367 (conv1 -> GELU -> conv2 (stride 2) ->
  GELU, then non-causal layers whose self-attention K/V are handed to the decoder);
* one layer: models.py:110-208 (norm1 -> q/k/v, cat past K/V, softmax(q k^T / sqrt(D))
  with a causal mask for multi-token decoder input, out-projection; cross-attention over
  the encoder K/V after norm2; MLP after norm3 (norm2 without cross-attention));
* decoding: models.py:369-423 (embedding, layers, decoder_norm, lm_head) driven as the
  scheduler does (phase_aware_scheduler.py:664-700 prompt prefill, then :771-1044 one
  token per step, greedy argmax, ``max_new_tokens`` counting the prefill token).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use it.
Pinned against the reference's own config-1 run (tests/golden/config1_tokens.json).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

Tensor = torch.Tensor


def _heads(t: Tensor, H: int) -> Tensor:
    B, T, _ = t.shape
    return t.view(B, T, H, -1).transpose(1, 2)


def _ln(sd: Dict[str, Tensor], name: str, x: Tensor) -> Tensor:
    return F.layer_norm(x, (x.shape[-1],), sd[name + ".weight"], sd[name + ".bias"])


def layer(sd: Dict[str, Tensor], p: str, x: Tensor, H: int, causal: bool,
          past: Optional[Tuple[Tensor, Tensor]] = None,
          enc_kv: Optional[Tuple[Tensor, Tensor]] = None) -> Tuple[Tensor, Tuple[Tensor, Tensor]]:
    """One layer (models.py:110-208); returns (x, (K, V) of the self-attention)."""
    B, T, _ = x.shape
    h = _ln(sd, p + "norm1", x)
    q = _heads(F.linear(h, sd[p + "self_attn_q.weight"]), H)
    k = _heads(F.linear(h, sd[p + "self_attn_k.weight"]), H)
    v = _heads(F.linear(h, sd[p + "self_attn_v.weight"]), H)
    if past is not None:
        k = torch.cat([past[0], k], 2)
        v = torch.cat([past[1], v], 2)
    scale = 1.0 / math.sqrt(q.shape[-1])
    w = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal and T > 1:
        w = w + torch.triu(torch.full((T, k.shape[2]), float("-inf"), dtype=x.dtype), diagonal=1)
    a = torch.matmul(F.softmax(w, -1), v).transpose(1, 2).reshape(B, T, -1)
    x = x + F.linear(a, sd[p + "self_attn_out.weight"])
    if enc_kv is not None:
        cq = _heads(F.linear(_ln(sd, p + "norm2", x), sd[p + "cross_attn_q.weight"]), H)
        cw = torch.matmul(cq, enc_kv[0].transpose(-2, -1)) * scale
        ca = torch.matmul(F.softmax(cw, -1), enc_kv[1]).transpose(1, 2).reshape(B, T, -1)
        x = x + F.linear(ca, sd[p + "cross_attn_out.weight"])
    h = _ln(sd, p + ("norm3" if enc_kv is not None else "norm2"), x)
    h = F.linear(F.gelu(F.linear(h, sd[p + "mlp.0.weight"], sd[p + "mlp.0.bias"])), sd[p + "mlp.2.weight"],
                 sd[p + "mlp.2.bias"])
    return x + h, (k, v)


def encode(sd: Dict[str, Tensor], mel: Tensor, H: int) -> List[Tuple[Tensor, Tensor]]:
    """[B, n_mels, F] -> per encoder layer (K, V) [B, H, T, D] (models.py:349-367)."""
    x = F.gelu(F.conv1d(mel, sd["conv1.weight"], sd["conv1.bias"], padding=1))
    x = F.gelu(F.conv1d(x, sd["conv2.weight"], sd["conv2.bias"], stride=2, padding=1)).transpose(1, 2)
    kv = []
    i = 0
    while f"encoder_layers.{i}.norm1.weight" in sd:
        x, (k, v) = layer(sd, f"encoder_layers.{i}.", x, H, causal=False)
        kv.append((k, v))
        i += 1
    return kv


def _decoder(sd, ids: Tensor, H: int, enc_kv, past) -> Tuple[Tensor, list]:
    x = F.embedding(ids, sd["decoder_embed.weight"])
    new = []
    i = 0
    while f"decoder_layers.{i}.norm1.weight" in sd:
        x, kv = layer(sd, f"decoder_layers.{i}.", x, H, causal=True, past=None if past is None else past[i],
                      enc_kv=enc_kv[i] if i < len(enc_kv) else None)
        new.append(kv)
        i += 1
    return F.linear(_ln(sd, "decoder_norm", x), sd["lm_head.weight"]), new


@torch.no_grad()
def greedy_decode(sd: Dict[str, Tensor], mels: Tensor, prompt: Sequence[int], max_new_tokens: int,
                  num_heads: int) -> List[List[int]]:
    """Greedy tokens for a batch of mels [B, n_mels, F] (EOS disabled): the prefill
    token, then ``max_new_tokens - 1`` single-token steps."""
    sd = {k: v.float() for k, v in sd.items()}
    enc_kv = encode(sd, mels.float(), num_heads)
    B = mels.shape[0]
    logits, past = _decoder(sd, torch.tensor([list(prompt)] * B), num_heads, enc_kv, None)
    toks = [logits[:, -1].argmax(-1)]
    for _ in range(max_new_tokens - 1):
        logits, past = _decoder(sd, toks[-1][:, None], num_heads, enc_kv, past)
        toks.append(logits[:, -1].argmax(-1))
    return torch.stack(toks, 1).tolist()
