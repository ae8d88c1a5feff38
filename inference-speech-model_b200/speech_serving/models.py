"""Whisper-class encoder-decoder models whose single-token decode step runs on the B200
decode kernels.

``WhisperClassSpeechEncoderDecoderModel`` keeps the module structure and parameter names
of the reference model (speech_serving/models.py:298-347 and DecoderLayer :79-108), so a
seeded random init produces the same weights and reference state dicts load unchanged.
``encode`` (:349-367) and the multi-token ``decode_step`` used for prompt prefill
(:369-423) are plain PyTorch.  ``decode_step_paged`` is the hot path and replaces
``decode_step_graph_fixed`` (:425-487): per layer it runs the paged self-attention
kernel, which also writes the new token's K/V into its pool block (ops 1 + 3), then
cross-attention straight from the graph-slot cross-KV buffer (op 2), with no bucket
buffers and no masks.  It allocates no workspace and never syncs, so it can be
captured in a CUDA graph.

``PretrainedWhisperModel`` wraps a Hugging Face ``WhisperForConditionalGeneration``
(reference :490-610).  It is built from a checkpoint or, without one, from a
``WhisperConfig`` with random weights.  Its ``encode`` projects every decoder layer's
cross K/V with ONE tcgen05 GEMM (op 4) into the graph-slot layout, and
``decode_step_paged`` runs the HF decoder's arithmetic on the same kernels.
"""
from __future__ import annotations

import math
import os
from typing import Any, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

os.environ.setdefault("USE_TF", "0")


def _fused_qkv(model: nn.Module, projs, q_scale: float = 1.0):
    """Per layer, the q / k / v projection weights stacked for one batched GEMM:
    (W [3, d_in, H*D] with W[i] = weight_i^T, bias [3, 1, H*D] (zeros where a projection
    has none)); the q rows are multiplied by ``q_scale``.  Built on first use and rebuilt
    when a weight has been replaced or modified in place."""
    key = tuple((p.weight.data_ptr(), p.weight._version) for trio in projs for p in trio) + (q_scale,)
    cache = model.__dict__.get("_qkv_cache")
    if cache is not None and cache[0] == key:
        return cache[1]
    out = []
    with torch.no_grad():
        for qp, kp, vp in projs:
            w = torch.stack([qp.weight * q_scale, kp.weight, vp.weight]).transpose(1, 2).contiguous()
            bs = [qp.bias * q_scale if qp.bias is not None else None, kp.bias, vp.bias]
            bias = torch.stack([b if b is not None else torch.zeros_like(qp.weight[:, 0]) for b in bs]).unsqueeze(1)
            out.append((w, bias))
    model.__dict__["_qkv_cache"] = (key, out)
    return out


def _fused_qkv_aug(model: nn.Module, projs, q_scale: float = 1.0):
    """``_fused_qkv`` with the bias folded into the GEMM: per layer W [3, d_in + 8, H*D]
    whose row d_in holds the biases (rows d_in+1.. are zero), for an input whose column
    d_in is 1 (``_qkv_input``).  One batched GEMM then gives q, k and v with their biases,
    with no copy of a broadcast bias into the output first."""
    base = _fused_qkv(model, projs, q_scale)
    key = tuple(w.data_ptr() for w, _ in base) + (q_scale,)
    cache = model.__dict__.get("_qkv_aug_cache")
    if cache is not None and cache[0] == key and cache[2] is base:
        return cache[1]
    with torch.no_grad():
        out = []
        for w, bias in base:
            pad = torch.zeros((3, 7, w.shape[2]), dtype=w.dtype, device=w.device)
            out.append(torch.cat([w, bias, pad], dim=1).contiguous())
    model.__dict__["_qkv_aug_cache"] = (key, out, base)
    return out


def _qkv_input(model: nn.Module, n: int, d: int, like: torch.Tensor) -> torch.Tensor:
    """The q/k/v GEMM's input rows [n, d + 8]: columns [0, d) take the LayerNorm output,
    column d is 1 (it picks up the bias row of ``_fused_qkv_aug``'s weights), the rest 0.
    One buffer per batch size, kept on the model."""
    bufs = model.__dict__.setdefault("_qkv_in", {})
    key = (n, d, like.dtype, like.device)
    if key not in bufs:
        t = torch.zeros((n, d + 8), dtype=like.dtype, device=like.device)
        t[:, d] = 1
        bufs[key] = t
    return bufs[key]


def _scaled_linears(model: nn.Module, linears, scale: float):
    """(weight * scale, bias * scale) per Linear, cached like ``_fused_qkv``."""
    key = tuple((p.weight.data_ptr(), p.weight._version) for p in linears) + (scale,)
    cache = model.__dict__.get("_scaled_cache")
    if cache is not None and cache[0] == key:
        return cache[1]
    with torch.no_grad():
        out = [(p.weight * scale, p.bias * scale if p.bias is not None else None) for p in linears]
    model.__dict__["_scaled_cache"] = (key, out)
    return out


def _padded_head(model: nn.Module, linear: nn.Linear, multiple: int = 64) -> torch.Tensor:
    """The output projection's weight with its rows (the vocabulary) padded with zeros to a
    multiple of ``multiple``, so the per-step head GEMM gets an aligned output row; the
    caller drops the padded columns.  Cached like ``_fused_qkv``."""
    w = linear.weight
    key = (w.data_ptr(), w._version, multiple)
    cache = model.__dict__.get("_head_cache")
    if cache is not None and cache[0] == key:
        return cache[1]
    v = w.shape[0]
    vp = (v + multiple - 1) // multiple * multiple
    with torch.no_grad():
        wp = torch.zeros((vp, w.shape[1]), dtype=w.dtype, device=w.device)
        wp[:v].copy_(w)
    model.__dict__["_head_cache"] = (key, wp)
    return wp


def _tc_linear_ok(x: torch.Tensor, K: int) -> bool:
    """True when ``ops.linear`` (the small-batch tcgen05 GEMM) takes this input: 16-bit,
    at most 64 rows, K a multiple of 64.  The decode steps use it for the MLP of models
    up to TC_MLP_MAX_WEIGHT_BYTES per layer: fc1 with its GELU fused (one launch instead
    of a GEMM and an elementwise kernel) and fc2.  The q/k/v and d x d projections and
    the vocabulary-padded head stay on cuBLAS, which measured faster for those shapes
    (profile_cases.py linear_table, and the decode_small / decode_large steps)."""
    return x.dtype in (torch.float16, torch.bfloat16) and x.shape[0] <= 64 and K % 64 == 0


# An MLP Linear runs on the tcgen05 kernel up to this weight size, else on cuBLAS (plus a
# GELU kernel after fc1).  Whole decode steps at batch 64 decided it: Whisper-small
# (4.7 MB per layer) 1,253 us with both MLP layers on the kernel against 1,256 us on
# cuBLAS; large-v3 (13.1 MB) 4,725 us against 4,691 us.
TC_MLP_MAX_WEIGHT_BYTES = 8 << 20


def _tc_mlp_ok(x: torch.Tensor, lin: nn.Linear) -> bool:
    return (_tc_linear_ok(x, lin.in_features)
            and lin.weight.numel() * lin.weight.element_size() <= TC_MLP_MAX_WEIGHT_BYTES)


def _mlp(h: torch.Tensor, fc1: nn.Linear, fc2: nn.Linear, act_is_gelu: bool, act) -> torch.Tensor:
    """fc2(act(fc1(h))), with fc1 + GELU and fc2 on the tcgen05 kernel where that measured
    faster (TC_MLP_MAX_WEIGHT_BYTES)."""
    if act_is_gelu and _tc_mlp_ok(h, fc1):
        u = ops.linear(h.contiguous(), fc1.weight, fc1.bias, gelu=True)
    else:
        u = act(fc1(h))
    if _tc_mlp_ok(u, fc2):
        return ops.linear(u.contiguous(), fc2.weight, fc2.bias)
    return fc2(u)


def _head_logits(model: nn.Module, h: torch.Tensor, head: nn.Linear) -> torch.Tensor:
    """[n, >= vocab] logits of the output projection: cuBLAS on the vocabulary-padded
    weight (an unpadded vocabulary makes cuBLAS pick a slow kernel)."""
    if head.bias is not None:
        return F.linear(h, head.weight, head.bias)
    return F.linear(h, _padded_head(model, head))


class _LayerKV:
    """Keys/values of one decoder layer ([B, H, T, D]), named like a DynamicCache layer."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor):
        self.keys, self.values = keys, values


class KVCache:
    """Per-layer keys/values returned by the multi-token ``decode_step`` (prefill)."""

    def __init__(self, layers: Sequence[_LayerKV]):
        self.layers = list(layers)


class ModelOutput:
    def __init__(self, logits: torch.Tensor, past_key_values: Optional[KVCache]):
        self.logits = logits
        self.past_key_values = past_key_values


class DecoderLayer(nn.Module):
    """Pre-norm transformer layer with self-attention, optional cross-attention and an
    MLP; attribute names and creation order follow speech_serving/models.py:82-108."""

    def __init__(self, hidden_dim: int, num_heads: int, head_dim: int, is_decoder: bool = True):
        super().__init__()
        self.hidden_dim, self.num_heads, self.head_dim, self.is_decoder = hidden_dim, num_heads, head_dim, is_decoder
        inner = num_heads * head_dim
        self.self_attn_q = nn.Linear(hidden_dim, inner, bias=False)
        self.self_attn_k = nn.Linear(hidden_dim, inner, bias=False)
        self.self_attn_v = nn.Linear(hidden_dim, inner, bias=False)
        self.self_attn_out = nn.Linear(inner, hidden_dim, bias=False)
        self.cross_attn_q = nn.Linear(hidden_dim, inner, bias=False)
        self.cross_attn_k = nn.Linear(hidden_dim, inner, bias=False)
        self.cross_attn_v = nn.Linear(hidden_dim, inner, bias=False)
        self.cross_attn_out = nn.Linear(inner, hidden_dim, bias=False)
        self.norm1 = nn.LayerNorm(hidden_dim)
        self.norm2 = nn.LayerNorm(hidden_dim)
        self.norm3 = nn.LayerNorm(hidden_dim)
        self.mlp = nn.Sequential(nn.Linear(hidden_dim, hidden_dim * 4), nn.GELU(), nn.Linear(hidden_dim * 4, hidden_dim))

    def _heads(self, t: torch.Tensor) -> torch.Tensor:  # [B, T, H*D] -> [B, H, T, D]
        return t.view(t.shape[0], t.shape[1], self.num_heads, self.head_dim).transpose(1, 2)

    def forward(self, x, past_key_values=None, encoder_hidden_states=None, encoder_past_kv=None, attention_mask=None,
                encoder_attention_mask=None):
        """Multi-token forward (encoder layers and decoder prefill), same arithmetic as the
        reference's eager path (speech_serving/models.py:110-208)."""
        B, T, _ = x.shape
        neg = torch.finfo(x.dtype).min
        h = self.norm1(x)
        q, k, v = self._heads(self.self_attn_q(h)), self._heads(self.self_attn_k(h)), self._heads(self.self_attn_v(h))
        if past_key_values is not None:
            k = torch.cat([past_key_values[0].to(q.dtype), k], dim=2)
            v = torch.cat([past_key_values[1].to(q.dtype), v], dim=2)
        scale = 1.0 / math.sqrt(self.head_dim)
        w = torch.matmul(q, k.transpose(-2, -1)) * scale
        if attention_mask is not None:
            m = attention_mask
            m = m[:, None, None, :] if m.dim() == 2 else (m[:, None] if m.dim() == 3 else m)
            if m.dtype == torch.bool:
                w = w.masked_fill(~m, neg)
            elif torch.isin(m, torch.tensor([0, 1], device=m.device)).all():
                w = w.masked_fill(m == 0, neg)
            else:
                w = w + m.to(q.dtype)
        if self.is_decoder and T > 1:
            w = w + torch.triu(torch.full((T, k.shape[2]), float("-inf"), device=x.device, dtype=q.dtype), diagonal=1)
        a = torch.matmul(F.softmax(w, dim=-1), v).transpose(1, 2).reshape(B, T, -1)
        x = x + self.self_attn_out(a)
        new_kv = (k, v)
        cross = encoder_hidden_states is not None or encoder_past_kv is not None
        if cross:
            hc = self.norm2(x)
            cq = self._heads(self.cross_attn_q(hc))
            if encoder_past_kv is not None:
                ck, cv = encoder_past_kv[0].to(cq.dtype), encoder_past_kv[1].to(cq.dtype)
            else:
                ck = self._heads(self.cross_attn_k(encoder_hidden_states))
                cv = self._heads(self.cross_attn_v(encoder_hidden_states))
            cw = torch.matmul(cq, ck.transpose(-2, -1)) * scale
            if encoder_attention_mask is not None:
                if encoder_attention_mask.dtype == torch.bool:
                    cw = cw.masked_fill(~encoder_attention_mask, neg)
                else:
                    cw = cw + encoder_attention_mask.to(cq.dtype)
            ca = torch.matmul(F.softmax(cw, dim=-1), cv).transpose(1, 2).reshape(B, T, -1)
            x = x + self.cross_attn_out(ca)
        x = x + self.mlp((self.norm3 if cross else self.norm2)(x))
        return x, new_kv, None


class WhisperClassSpeechEncoderDecoderModel(nn.Module):
    """Random-init Whisper-class model; constructor and parameters as in the reference
    (speech_serving/models.py:304-347)."""

    def __init__(self, num_encoder_layers: int = 4, num_decoder_layers: int = 4, num_heads: int = 4,
                 hidden_dim: int = 256, mel_dim: int = 80, vocab_size: int = 51200):
        super().__init__()
        self.num_encoder_layers, self.num_decoder_layers = num_encoder_layers, num_decoder_layers
        self.num_heads, self.head_dim, self.hidden_dim = num_heads, hidden_dim // num_heads, hidden_dim
        self.vocab_size = vocab_size
        self.num_decoder_kv_heads = num_heads

        class Config:
            pass

        self.config = Config()
        self.config.num_hidden_layers = num_decoder_layers
        self.config.num_attention_heads = num_heads
        self.config.num_key_value_heads = num_heads
        self.config.hidden_size = hidden_dim
        self.config.vocab_size = vocab_size
        self.config.encoder_num_layers = num_encoder_layers
        self.conv1 = nn.Conv1d(mel_dim, hidden_dim, kernel_size=3, padding=1)
        self.conv2 = nn.Conv1d(hidden_dim, hidden_dim, kernel_size=3, stride=2, padding=1)
        self.encoder_layers = nn.ModuleList(
            [DecoderLayer(hidden_dim, num_heads, self.head_dim, is_decoder=False) for _ in range(num_encoder_layers)])
        self.encoder_norm = nn.LayerNorm(hidden_dim)
        self.decoder_embed = nn.Embedding(vocab_size, hidden_dim)
        self.decoder_layers = nn.ModuleList(
            [DecoderLayer(hidden_dim, num_heads, self.head_dim, is_decoder=True) for _ in range(num_decoder_layers)])
        self.decoder_norm = nn.LayerNorm(hidden_dim)
        self.lm_head = nn.Linear(hidden_dim, vocab_size, bias=False)

    @property
    def dtype(self) -> torch.dtype:
        return self.decoder_norm.weight.dtype

    def encode(self, mel_features: torch.Tensor) -> Tuple[torch.Tensor, List[Tuple[torch.Tensor, torch.Tensor]]]:
        """[B, mel, frames] -> (hidden [B, T, d], per encoder layer (K, V) [B, H, T, D]).
        The decoder's cross-attention reads encoder layer i's self-attention K/V."""
        x = F.gelu(self.conv1(mel_features))
        x = F.gelu(self.conv2(x)).transpose(1, 2)
        kv = []
        for layer in self.encoder_layers:
            x, (k, v), _ = layer(x)
            kv.append((k, v))
        return self.encoder_norm(x), kv

    def decode_step(self, input_ids, past_key_values=None, encoder_past_kv_list=None, encoder_hidden_states=None,
                    attention_mask=None, encoder_attention_mask=None, position_ids=None, use_cache=True, **kwargs):
        """Multi-token decoder forward (prompt prefill); returns logits and per-layer K/V."""
        x = self.decoder_embed(input_ids).to(self.dtype)
        layers = []
        for i, layer in enumerate(self.decoder_layers):
            past = None
            if past_key_values is not None and i < len(past_key_values.layers):
                past = (past_key_values.layers[i].keys, past_key_values.layers[i].values)
            enc = encoder_past_kv_list[i] if encoder_past_kv_list is not None and i < len(encoder_past_kv_list) else None
            x, (k, v), _ = layer(x, past_key_values=past, encoder_hidden_states=None if enc is not None else
                                 encoder_hidden_states, encoder_past_kv=enc, attention_mask=attention_mask,
                                 encoder_attention_mask=encoder_attention_mask)
            layers.append(_LayerKV(k, v))
        return ModelOutput(self.lm_head(self.decoder_norm(x)), KVCache(layers) if use_cache else None)

    # ---- decode hot path -------------------------------------------------------------
    def cross_kv_from_encoder(self, encoder_kv_list, slots: torch.Tensor, slot: int) -> int:
        """Copies one request's encoder K/V (direct handoff) into graph slot ``slot`` of
        ``slots`` [S, L, 2, H, T, D]; returns the encoder length."""
        T = encoder_kv_list[0][0].shape[2]
        for l, (k, v) in enumerate(encoder_kv_list):
            slots[slot, l, 0, :, :T].copy_(k[0])
            slots[slot, l, 1, :, :T].copy_(v[0])
        return T

    def decode_step_paged(self, st, n: int) -> torch.Tensor:
        """One decode step for slots [0, n) of the paged decode state ``st``
        (graph_decode_buffers.PagedDecodeState): tokens st.token_ids[:n], attended lengths
        st.ctx_lens[:n] (including the new token; 0 = inactive slot), block tables
        st.block_tables[:n], cross K/V st.cross_kv[:n] with lengths st.cross_lens[:n].
        Returns the greedy next tokens [n] (int64)."""
        x = self.decoder_embed(st.token_ids[:n]).to(self.dtype)  # [n, d]
        H, D = self.num_heads, self.head_dim
        scale = 1.0 / math.sqrt(D)
        fused = _fused_qkv(self, [(lay.self_attn_q, lay.self_attn_k, lay.self_attn_v) for lay in self.decoder_layers])
        layers = self.decoder_layers
        # each residual add runs fused with the LayerNorm after it (x is updated in place)
        x, h = ops.add_layernorm(x, None, layers[0].norm1)
        for l, layer in enumerate(layers):
            w, _ = fused[l]
            qkv = torch.bmm(h.unsqueeze(0).expand(3, n, h.shape[-1]), w)  # [3, n, H*D]: q, k, v
            q, k, v = qkv[0].view(n, H, D), qkv[1].view(n, H, D), qkv[2].view(n, H, D)
            a = ops.paged_decode_attention(q, st.key_pool[l], st.value_pool[l], st.block_tables[:n], st.ctx_lens[:n],
                                           scale=scale, k_new=k, v_new=v, workspace=st.paged_ws[n])
            x, h = ops.add_layernorm(x, layer.self_attn_out(a.view(n, -1)), layer.norm2)
            cq = layer.cross_attn_q(h).view(n, H, D)
            c = ops.cross_attention(cq, st.cross_kv[:n, l, 0], st.cross_kv[:n, l, 1], st.cross_lens[:n], scale=scale,
                                    workspace=st.cross_ws[n])
            x, h = ops.add_layernorm(x, layer.cross_attn_out(c.view(n, -1)), layer.norm3)
            nxt = layers[l + 1].norm1 if l + 1 < len(layers) else self.decoder_norm
            mlp = _mlp(h, layer.mlp[0], layer.mlp[2], isinstance(layer.mlp[1], nn.GELU) and
                       layer.mlp[1].approximate == "none", layer.mlp[1])
            x, h = ops.add_layernorm(x, mlp, nxt)
        return ops.argmax_rows(_head_logits(self, h, self.lm_head), self.vocab_size)


class PretrainedWhisperModel(nn.Module):
    """Hugging Face Whisper wrapper (reference speech_serving/models.py:490-610).

    Build it from ``model_name_or_path`` (a local checkpoint) or, with no checkpoint at
    hand, from ``config`` (a ``WhisperConfig``) with random weights drawn under
    ``seed``."""

    def __init__(self, model_name_or_path: Optional[str] = None, device: str = "cuda",
                 dtype: torch.dtype = torch.float16, local_files_only: bool = True, config: Any = None,
                 seed: int = 0):
        from transformers import WhisperForConditionalGeneration

        if isinstance(dtype, str):
            dtype = getattr(torch, dtype)
        super().__init__()
        self.device, self.dtype_ = device, dtype
        if config is not None:
            # random weights drawn on the target device (seeded): large-v3 is 1.5 B
            # parameters, slow to initialise on the host with several ranks at once
            torch.manual_seed(seed)
            with torch.device(device):
                hf = WhisperForConditionalGeneration(config)
        else:
            hf = WhisperForConditionalGeneration.from_pretrained(model_name_or_path, dtype=dtype,
                                                                 local_files_only=local_files_only)
        self.hf_model = hf.to(device=device, dtype=dtype).eval()
        cfg = self.hf_model.config
        self.config = cfg
        self.num_encoder_layers, self.num_decoder_layers = cfg.encoder_layers, cfg.decoder_layers
        self.num_heads = cfg.decoder_attention_heads
        self.num_decoder_kv_heads = self.num_encoder_kv_heads = self.num_heads
        self.head_dim = cfg.d_model // self.num_heads
        self.hidden_dim, self.vocab_size = cfg.d_model, cfg.vocab_size
        suppress = getattr(cfg, "suppress_tokens", None)
        if suppress:
            m = torch.zeros(self.vocab_size, dtype=torch.bool, device=device)
            m[list(suppress)] = True
            self.register_buffer("suppress_mask", m)
        else:
            self.suppress_mask = None
        self._w_kv = None

    # encode() can write the cross K/V straight into graph slots (direct handoff)
    encodes_into_slots = True

    @property
    def dtype(self) -> torch.dtype:
        return self.dtype_

    def stacked_cross_kv_weights(self) -> Tuple[torch.Tensor, torch.Tensor]:
        if self._w_kv is None:
            self._w_kv = ops.stack_cross_kv_weights(self.hf_model.model.decoder.layers)
        return self._w_kv

    def encode(self, mel_features: torch.Tensor, out_slots: Optional[torch.Tensor] = None,
               slot_ids: Optional[torch.Tensor] = None):
        """Encoder forward, then every decoder layer's cross K/V by one GEMM (op 4).

        Without ``out_slots`` a [B, L, 2, H, T, D] buffer is allocated and the return
        value matches the reference: (enc_out, [(K, V)] per layer, K/V [B, H, T, D]).
        With ``out_slots`` ([S, L, 2, H, T_out, D]) and ``slot_ids`` (int32 [B]) the
        projections are written straight into those slots and the K/V list is None."""
        enc_out = self.hf_model.model.encoder(mel_features.to(self.dtype)).last_hidden_state.contiguous()
        B, T, d = enc_out.shape
        L, H, D = self.num_decoder_layers, self.num_heads, self.head_dim
        if self.dtype not in (torch.float16, torch.bfloat16):
            # the tcgen05 projection takes 16-bit operands; fp32 models project per layer
            # with their own k_proj / v_proj, as the reference does (models.py:554-561)
            kv = []
            for l, layer in enumerate(self.hf_model.model.decoder.layers):
                att = layer.encoder_attn
                k = att.k_proj(enc_out).view(B, T, H, D).transpose(1, 2)
                v = att.v_proj(enc_out).view(B, T, H, D).transpose(1, 2)
                if out_slots is not None:
                    idx = slot_ids.long() if slot_ids is not None else torch.arange(B, device=enc_out.device)
                    out_slots[idx, l, 0, :, :T] = k
                    out_slots[idx, l, 1, :, :T] = v
                kv.append((k, v))
            return enc_out, (None if slot_ids is not None else kv)
        w, b = self.stacked_cross_kv_weights()
        if out_slots is None:
            out_slots = torch.empty((B, L, 2, H, T, D), dtype=self.dtype, device=enc_out.device)
            slot_ids = None
        ops.cross_kv_project(enc_out, w, b, out_slots, slot_ids=slot_ids)
        if slot_ids is not None:
            return enc_out, None
        return enc_out, [(out_slots[:B, l, 0, :, :T], out_slots[:B, l, 1, :, :T]) for l in range(L)]

    def cross_kv_from_encoder(self, encoder_kv_list, slots: torch.Tensor, slot: int) -> int:
        T = encoder_kv_list[0][0].shape[2]
        for l, (k, v) in enumerate(encoder_kv_list):
            slots[slot, l, 0, :, :T].copy_(k[0])
            slots[slot, l, 1, :, :T].copy_(v[0])
        return T

    # ---- encoder + projection as CUDA graphs, one per batch bucket ----------------------
    def encode_into_slots(self, mel_features: torch.Tensor, out_slots: torch.Tensor, slots: Sequence[int],
                          spare_slot: int, buckets: Sequence[int], use_graphs: bool = True) -> torch.Tensor:
        """Encoder forward and the op-4 projection of a batch straight into graph slots
        ``slots`` of ``out_slots`` ([S, L, 2, H, T_out, D]).  With 16-bit weights and
        full-length inputs (2 * max_source_positions frames) the pair runs as a CUDA graph
        captured per batch bucket (the batch is padded to the bucket; padding rows project
        into ``spare_slot``, which decoding never reads), so a batch costs one replay
        instead of one launch per encoder op.  Returns the encoder output [B, T, d]."""
        n = mel_features.shape[0]
        frames = 2 * self.config.max_source_positions
        graphable = (use_graphs and self.dtype in (torch.float16, torch.bfloat16) and mel_features.shape[-1] == frames
                     and n <= max(buckets) and str(out_slots.device).startswith("cuda"))
        dev = out_slots.device
        if not graphable:
            ids = torch.tensor(list(slots), dtype=torch.int32).to(dev, non_blocking=True)
            enc, _ = self.encode(mel_features, out_slots=out_slots, slot_ids=ids)
            return enc
        bucket = min(b for b in buckets if b >= n)
        graphs = self.__dict__.setdefault("_enc_graphs", {})
        key = (bucket, out_slots.data_ptr())
        if key not in graphs:
            self._capture_encoder_graphs(out_slots, spare_slot, buckets)
        g, mel_buf, ids_buf, hidden = graphs[key]
        mel_buf[:n].copy_(mel_features, non_blocking=True)
        ids = torch.full((bucket,), spare_slot, dtype=torch.int32)
        ids[:n] = torch.tensor(list(slots), dtype=torch.int32)
        ids_buf.copy_(ids.pin_memory(), non_blocking=True)
        g.replay()
        return hidden[:n]

    def _capture_encoder_graphs(self, out_slots: torch.Tensor, spare_slot: int, buckets: Sequence[int]) -> None:
        """Captures encoder + projection for every bucket at once (they share one memory
        pool and are replayed one at a time)."""
        graphs = self.__dict__.setdefault("_enc_graphs", {})
        dev = out_slots.device
        frames = 2 * self.config.max_source_positions
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        pool = self.__dict__.get("_enc_pool")
        for bucket in sorted(buckets):
            key = (bucket, out_slots.data_ptr())
            if key in graphs:
                continue
            mel_buf = torch.zeros((bucket, self.config.num_mel_bins, frames), dtype=self.dtype, device=dev)
            ids_buf = torch.full((bucket,), spare_slot, dtype=torch.int32, device=dev)
            with torch.cuda.stream(side), torch.no_grad():
                for _ in range(2):
                    self.encode(mel_buf, out_slots=out_slots, slot_ids=ids_buf)
            side.synchronize()
            g = torch.cuda.CUDAGraph()
            kw = {"pool": pool} if pool is not None else {}
            with torch.cuda.graph(g, stream=side, **kw), torch.no_grad():
                hidden, _ = self.encode(mel_buf, out_slots=out_slots, slot_ids=ids_buf)
            if pool is None:
                pool = g.pool()
                self.__dict__["_enc_pool"] = pool
            graphs[key] = (g, mel_buf, ids_buf, hidden)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)

    def decode_step(self, input_ids, past_key_values=None, encoder_past_kv_list=None, encoder_hidden_states=None,
                    attention_mask=None, encoder_attention_mask=None, position_ids=None, use_cache=True, **kwargs):
        """Multi-token HF decoder forward (prompt prefill), cross K/V from the encoder's
        projections (reference speech_serving/models.py:563-610)."""
        from transformers.cache_utils import DynamicCache, EncoderDecoderCache

        B = input_ids.shape[0]
        T = encoder_past_kv_list[0][0].shape[2] if encoder_past_kv_list is not None else 1500
        cross = DynamicCache()
        if encoder_past_kv_list is not None:
            for l, (k, v) in enumerate(encoder_past_kv_list):
                cross.update(k.contiguous(), v.contiguous(), layer_idx=l)
        selfc = DynamicCache()
        if past_key_values is not None:
            for l, lay in enumerate(past_key_values.layers):
                selfc.update(lay.keys, lay.values, layer_idx=l)
        cache = EncoderDecoderCache(selfc, cross)
        for l in range(len(cross.layers)):
            cache.is_updated[l] = True
        dummy = torch.empty((B, T, self.hidden_dim), device=input_ids.device, dtype=self.dtype)
        out = self.hf_model.model.decoder(input_ids=input_ids, encoder_hidden_states=dummy, past_key_values=cache,
                                          attention_mask=attention_mask, position_ids=position_ids, use_cache=True)
        logits = self.hf_model.proj_out(out.last_hidden_state)
        if self.suppress_mask is not None:
            logits = logits.masked_fill(self.suppress_mask, float("-inf"))
        sc = out.past_key_values.self_attention_cache
        layers = [_LayerKV(sc.layers[l].keys, sc.layers[l].values) for l in range(self.num_decoder_layers)]
        return ModelOutput(logits, KVCache(layers) if use_cache else None)

    def decode_step_paged(self, st, n: int) -> torch.Tensor:
        """One HF-Whisper decode step for slots [0, n) on the paged kernels (same contract
        as WhisperClassSpeechEncoderDecoderModel.decode_step_paged).  Query scaling
        follows WhisperAttention: q = q_proj(h) * head_dim**-0.5, attention scale 1."""
        dec = self.hf_model.model.decoder
        H, D = self.num_heads, self.head_dim
        pos = (st.ctx_lens[:n] - 1).clamp_(min=0).long()
        x = dec.embed_tokens(st.token_ids[:n]) * dec.embed_scale + dec.embed_positions.weight[pos]
        # q, k and v of a layer as one batched GEMM; WhisperAttention's query scaling is
        # folded into the q weights when it is a power of two (exact), else applied after
        fold = math.log2(dec.layers[0].self_attn.scaling).is_integer()
        fused = _fused_qkv_aug(self, [(lay.self_attn.q_proj, lay.self_attn.k_proj, lay.self_attn.v_proj)
                                      for lay in dec.layers], q_scale=dec.layers[0].self_attn.scaling if fold else 1.0)
        cross_q = _scaled_linears(self, [lay.encoder_attn.q_proj for lay in dec.layers],
                                  dec.layers[0].encoder_attn.scaling) if fold else None
        layers = dec.layers
        # each residual add runs fused with the LayerNorm after it (x is updated in place);
        # the LayerNorm before a self-attention writes straight into the q/k/v GEMM's input
        d = self.hidden_dim
        qkv_in = _qkv_input(self, n, d, x)
        x, _ = ops.add_layernorm(x.contiguous(), None, layers[0].self_attn_layer_norm, out_y=qkv_in[:, :d])
        for l, layer in enumerate(layers):
            sa = layer.self_attn
            qkv = torch.bmm(qkv_in.unsqueeze(0).expand(3, n, d + 8), fused[l])  # [3, n, H*D], biases included
            q = qkv[0] if fold else qkv[0] * sa.scaling
            q, k, v = q.view(n, H, D), qkv[1].view(n, H, D), qkv[2].view(n, H, D)
            a = ops.paged_decode_attention(q, st.key_pool[l], st.value_pool[l], st.block_tables[:n], st.ctx_lens[:n],
                                           scale=1.0, k_new=k, v_new=v, workspace=st.paged_ws[n])
            x, h = ops.add_layernorm(x, sa.out_proj(a.view(n, -1)), layer.encoder_attn_layer_norm)
            ea = layer.encoder_attn
            if fold:
                wq, bq = cross_q[l]
                cq = F.linear(h, wq, bq).view(n, H, D)
            else:
                cq = (ea.q_proj(h) * ea.scaling).view(n, H, D)
            c = ops.cross_attention(cq, st.cross_kv[:n, l, 0], st.cross_kv[:n, l, 1], st.cross_lens[:n], scale=1.0,
                                    workspace=st.cross_ws[n])
            x, h = ops.add_layernorm(x, ea.out_proj(c.view(n, -1)), layer.final_layer_norm)
            mlp = _mlp(h, layer.fc1, layer.fc2, self.config.activation_function == "gelu", layer.activation_fn)
            if l + 1 < len(layers):
                x, _ = ops.add_layernorm(x, mlp, layers[l + 1].self_attn_layer_norm, out_y=qkv_in[:, :d])
            else:
                x, h = ops.add_layernorm(x, mlp, dec.layer_norm)
        # the suppress mask and the argmax over the vocabulary in one kernel
        return ops.argmax_rows(_head_logits(self, h, self.hf_model.proj_out), self.vocab_size, self.suppress_mask)
