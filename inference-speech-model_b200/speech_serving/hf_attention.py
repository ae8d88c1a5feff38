"""Drop-in forwards for the attention modules of a Hugging Face Whisper decoder.

The reference's paging benchmark switches an HF decoder to a direct paged kernel by
replacing ``layer.self_attn.forward`` (scripts/evaluate_paging_variants.py:615-646): the
new forward projects q (times ``scaling``), k and v of the one new token, writes k and v
into the token's pool block at position ``context_lens[b]`` (a per-sequence ``.item()``
loop there), runs the Triton paged kernel over ``context_lens + 1`` positions and applies
``out_proj``.  Its cross-attention stays HF's, over cross K/V held in an
``EncoderDecoderCache``.

Here the same swap runs on the B200 kernels:

* ``paged_self_attn_forward`` is the self-attention forward.  One launch of op 1 with op 3
  fused writes the new K/V row and attends over it; there is no host loop and no sync, so
  a decoder step with these forwards can be captured in a CUDA graph.
* ``cross_attn_forward`` is the matching ``encoder_attn`` forward over precomputed cross
  K/V (op 2), e.g. the graph-slot layout that op 4 writes at handoff.
* ``PagedDecodeState`` holds what the forwards of one decoder share: the per-layer pools,
  the int32 block tables and lengths, and the cross K/V with their valid lengths.
* ``patch_decoder`` swaps the forwards of every layer and returns a handle that restores
  the originals, as the reference restores ``original_forwards`` after its run.

The forwards keep the HF signature ``forward(hidden_states, past_key_values=None,
attention_mask=None, **kwargs) -> (attn_output, None)`` and ignore the HF caches; the HF
decoder's position ids come from its cache length unless the caller passes
``position_ids`` (the reference passes a fresh, empty cache every step).
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence

import torch

from . import ops


class PagedDecodeState:
    """Device state shared by the patched attention forwards of one decoder.

    key_pools / value_pools: per decoder layer, ``[num_blocks, block_size, H, D]`` (the
    ``BlockManager.key_pool[l]`` / ``value_pool[l]`` layout).  block_tables: int32
    ``[B, max_blocks]``.  context_lens: int32 ``[B]``, tokens already cached for each
    sequence; the current step's token goes to position ``context_lens[b]``.  The caller
    sets or advances ``context_lens`` between steps (``advance``), as the reference sets
    ``triton_context_lens`` before each step.

    cross_k / cross_v (optional): per layer ``[B, H, T, D]`` with contiguous rows (any batch
    and head strides, so slot-buffer views work); cross_lens: int32 ``[B]`` valid encoder
    positions per sequence.
    """

    def __init__(self, key_pools: Sequence[torch.Tensor], value_pools: Sequence[torch.Tensor],
                 block_tables: torch.Tensor, context_lens: torch.Tensor,
                 cross_k: Optional[Sequence[torch.Tensor]] = None, cross_v: Optional[Sequence[torch.Tensor]] = None,
                 cross_lens: Optional[torch.Tensor] = None):
        if len(key_pools) != len(value_pools) or not key_pools:
            raise ValueError("PagedDecodeState: one key and one value pool per layer expected")
        if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
            raise ValueError("PagedDecodeState: block_tables and context_lens must be int32")
        if block_tables.dim() != 2 or context_lens.shape != (block_tables.shape[0],):
            raise ValueError("PagedDecodeState: block_tables [B, max_blocks] and context_lens [B] expected")
        if (cross_k is None) != (cross_v is None) or (cross_k is not None and cross_lens is None):
            raise ValueError("PagedDecodeState: cross_k, cross_v and cross_lens go together")
        if cross_lens is not None and (cross_lens.dtype != torch.int32 or cross_lens.shape != context_lens.shape):
            raise ValueError("PagedDecodeState: cross_lens must be int32 [B]")
        self.key_pools, self.value_pools = list(key_pools), list(value_pools)
        self.block_tables, self.context_lens = block_tables, context_lens
        self.cross_k = list(cross_k) if cross_k is not None else None
        self.cross_v = list(cross_v) if cross_v is not None else None
        self.cross_lens = cross_lens
        # positions attended this step (context_lens + 1), refreshed by layer 0's forward
        self.attend_lens = torch.empty_like(context_lens)

    @property
    def num_layers(self) -> int:
        return len(self.key_pools)

    def begin_step(self) -> None:
        """Positions attended by this step's self-attention: the cached ones plus the new."""
        torch.add(self.context_lens, 1, out=self.attend_lens)

    def advance(self, n: int = 1) -> None:
        """After a step: the step's token is now cached."""
        self.context_lens.add_(n)


def paged_self_attn_forward(attn: torch.nn.Module, layer_idx: int, state: PagedDecodeState) -> Callable:
    """HF ``WhisperAttention`` self-attention forward on ops 1 + 3 for layer ``layer_idx``
    (reference: scripts/evaluate_paging_variants.py:616-646, ``triton_forward``)."""
    H, D = attn.num_heads, attn.head_dim

    def forward(hidden_states, past_key_values=None, attention_mask=None, **kwargs):
        B, T, _ = hidden_states.shape
        if T != 1:
            raise RuntimeError("paged self-attention forward: one new token per sequence expected")
        if layer_idx == 0:
            state.begin_step()
        q = attn.q_proj(hidden_states).view(B, H, D)
        k = attn.k_proj(hidden_states).view(B, H, D)
        v = attn.v_proj(hidden_states).view(B, H, D)
        o = ops.paged_decode_attention(q, state.key_pools[layer_idx], state.value_pools[layer_idx],
                                       state.block_tables, state.attend_lens, scale=attn.scaling, k_new=k, v_new=v)
        return attn.out_proj(o.view(B, 1, H * D)), None

    return forward


def cross_attn_forward(attn: torch.nn.Module, layer_idx: int, state: PagedDecodeState) -> Callable:
    """HF ``WhisperAttention`` cross-attention (``encoder_attn``) forward on op 2 over the
    state's cross K/V of layer ``layer_idx`` (reference: HF's encoder_attn over the
    ``EncoderDecoderCache`` cross entries, scripts/evaluate_paging_variants.py:677-693)."""
    H, D = attn.num_heads, attn.head_dim

    def forward(hidden_states, key_value_states=None, past_key_values=None, attention_mask=None, **kwargs):
        B, T, _ = hidden_states.shape
        if T != 1:
            raise RuntimeError("cross-attention forward: one new token per sequence expected")
        q = attn.q_proj(hidden_states).view(B, H, D)
        o = ops.cross_attention(q, state.cross_k[layer_idx], state.cross_v[layer_idx], state.cross_lens,
                                scale=attn.scaling)
        return attn.out_proj(o.view(B, 1, H * D)), None

    return forward


class PatchHandle:
    """Restores the original attention forwards of a patched decoder."""

    def __init__(self, saved: List[tuple]):
        self._saved = saved

    def restore(self) -> None:
        for module, fwd in self._saved:
            if fwd is None:
                module.__dict__.pop("forward", None)
            else:
                module.forward = fwd
        self._saved = []


def patch_decoder(decoder: torch.nn.Module, state: PagedDecodeState, cross: bool = True) -> PatchHandle:
    """Swaps ``self_attn.forward`` (and, with ``cross`` and cross K/V in the state,
    ``encoder_attn.forward``) of every layer of an HF Whisper decoder for the kernel
    forwards.  Returns the handle that undoes it."""
    layers = decoder.layers
    if len(layers) != state.num_layers:
        raise ValueError(f"patch_decoder: {len(layers)} decoder layers, state has {state.num_layers}")
    if cross and state.cross_k is None:
        raise ValueError("patch_decoder: cross=True needs cross K/V in the state")
    saved = []
    for l, layer in enumerate(layers):
        mods = [(layer.self_attn, paged_self_attn_forward)]
        if cross:
            mods.append((layer.encoder_attn, cross_attn_forward))
        for mod, make in mods:
            saved.append((mod, mod.__dict__.get("forward")))
            mod.forward = make(mod, l, state)
    return PatchHandle(saved)
