"""CPU oracle for the speech-decode hot path — TEST INFRASTRUCTURE, not product code.

A plain numpy restatement of the reference engine's arithmetic for the five decode-path
operations.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import it, and only as the checker or the timed CPU baseline; the product path
(``speech_serving``) never calls it.

Pinned against golden vectors produced by running the reference itself (see
``tests/golden/make_golden.py`` and ``tests/test_oracle_golden.py``).

All arithmetic is fp32 (inputs of any float dtype are upcast), matching the reference's
fp32 CPU path; softmax uses the max-subtracted form of torch.softmax.
"""
from __future__ import annotations

import numpy as np


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def gather_sequence(pool: np.ndarray, table, T: int) -> np.ndarray:
    """pool[table].view(-1, H, D)[:T].permute(1, 0, 2) -> [H, T, D].

    Follows speech_serving/phase_aware_scheduler.py:617-622 and
    speech_serving/encoder_attention.py:50-58."""
    nb, bs, H, D = pool.shape
    g = pool[np.asarray(table, dtype=np.int64)].reshape(-1, H, D)[:T]
    return np.ascontiguousarray(g.transpose(1, 0, 2))


def softmax_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """softmax(q·kᵀ·scale)·v for q [H, D], k/v [H, T, D] -> [H, D].

    Follows speech_serving/models.py:140-164 (self) and :184-202 (cross) for one query."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    s = np.einsum("hd,htd->ht", q, k).astype(np.float32) * np.float32(scale)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s).astype(np.float32)
    p = p / p.sum(axis=1, keepdims=True)
    return np.einsum("ht,htd->hd", p, v).astype(np.float32)


def paged_decode_attention(q, k_pool, v_pool, block_tables, context_lens, scale=None) -> np.ndarray:
    """Op (1): q [B, H, D]; pools [num_blocks, bs, H, D]; tables [B, max_blocks];
    context_lens [B].  Rows with context <= 0 are zeros (the reference Triton kernel
    returns early, scripts/evaluate_paging_variants.py:78-80, leaving its zero output)."""
    q = _f32(q)
    B, H, D = q.shape
    scale = (1.0 / np.sqrt(D)) if scale is None else scale
    out = np.zeros((B, H, D), np.float32)
    for b in range(B):
        T = int(context_lens[b])
        if T <= 0:
            continue
        nblk = -(-T // k_pool.shape[1])
        table = np.asarray(block_tables[b][:nblk])
        k = gather_sequence(_f32(k_pool), table, T)
        v = gather_sequence(_f32(v_pool), table, T)
        out[b] = softmax_attention(q[b], k, v, scale)
    return out


def cross_attention(q, k, v, valid_lens, scale=None) -> np.ndarray:
    """Op (2): q [B, H, D]; k/v [B, H, T, D]; attend t < valid_lens[b] (the reference's
    bool mask, speech_serving/models.py:196-197).  valid <= 0 gives zeros."""
    q = _f32(q)
    B, H, D = q.shape
    scale = (1.0 / np.sqrt(D)) if scale is None else scale
    out = np.zeros((B, H, D), np.float32)
    for b in range(B):
        T = min(int(valid_lens[b]), k.shape[2])
        if T <= 0:
            continue
        out[b] = softmax_attention(q[b], _f32(k[b, :, :T]), _f32(v[b, :, :T]), scale)
    return out


def kv_append(k_src, v_src, k_pool, v_pool, block_tables, positions) -> None:
    """Op (3), in place: for each b with positions[b] >= 0 and t < T,
    pool[table[b][(p+t)//bs], (p+t)%bs] = src[b, :, t, :].

    Follows speech_serving/phase_aware_scheduler.py:1004-1010 (one token) and :678-690
    (prompt rows)."""
    B, H, T, D = k_src.shape
    bs = k_pool.shape[1]
    for b in range(B):
        p0 = int(positions[b])
        if p0 < 0:
            continue
        for t in range(T):
            pos = p0 + t
            blk = int(block_tables[b][pos // bs])
            k_pool[blk, pos % bs] = k_src[b, :, t, :]
            if v_pool is not None:
                v_pool[blk, pos % bs] = v_src[b, :, t, :]


def block_gather(pool, block_tables, seq_lens, T_out: int) -> np.ndarray:
    """Op (5): [B, H, T_out, D], zero padded beyond seq_lens[b]
    (speech_serving/phase_aware_scheduler.py:874-881 builds the same zero-padded batch)."""
    nb, bs, H, D = pool.shape
    B = len(seq_lens)
    out = np.zeros((B, H, T_out, D), pool.dtype)
    for b in range(B):
        T = int(seq_lens[b])
        if T <= 0:
            continue
        nblk = -(-T // bs)
        out[b, :, :T] = gather_sequence(pool, np.asarray(block_tables[b][:nblk]), T)
    return out


def cross_kv_project(enc_out, w_k_list, w_v_list, b_v_list, H: int) -> list:
    """Op (4): per decoder layer l, K = enc_out @ Wk[l]ᵀ, V = enc_out @ Wv[l]ᵀ + bv[l],
    reshaped [B, T, H, D] -> [B, H, T, D] (speech_serving/models.py:554-561; k_proj has
    no bias, v_proj has one)."""
    x = _f32(enc_out)
    B, T, d = x.shape
    D = w_k_list[0].shape[0] // H
    res = []
    for wk, wv, bv in zip(w_k_list, w_v_list, b_v_list):
        k = x @ _f32(wk).T
        v = x @ _f32(wv).T
        if bv is not None:
            v = v + _f32(bv)
        res.append((k.reshape(B, T, H, D).transpose(0, 2, 1, 3), v.reshape(B, T, H, D).transpose(0, 2, 1, 3)))
    return res
