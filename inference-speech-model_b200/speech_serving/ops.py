"""Torch-tensor front end of the five decode-path kernels (C ABI in include/spd_b200.h).

Each function checks shapes, dtypes, devices and strides, then calls the extension
through ctypes on ``torch.cuda.current_stream()`` (the capture stream inside
``torch.cuda.graph``).  Nothing here synchronises or reads device values, so every op
can be captured in a CUDA graph.  CPU tensors raise ``RuntimeError``: the product path
has no CPU implementation.

Ops and the reference code they replace:
  paged_decode_attention  scripts/evaluate_paging_variants.py:56-133 (Triton kernel),
                          speech_serving/models.py:126-165 and :443-466
  cross_attention         speech_serving/models.py:167-203 and :468-479
  kv_append               speech_serving/phase_aware_scheduler.py:1004-1010, :678-690;
                          speech_serving/models.py:449-454
  block_gather            speech_serving/phase_aware_scheduler.py:613-624, :859-882;
                          speech_serving/encoder_attention.py:50-63
  cross_kv_project        speech_serving/models.py:554-561
  linear                  the decode step's Linear layers (speech_serving/models.py:127-129,
                          :159, :178-180, :202, :205-207, :487)
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Tuple

import torch

from . import _native as N

_DTYPES = {torch.float32: N.SPD_F32, torch.float16: N.SPD_F16, torch.bfloat16: N.SPD_BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise RuntimeError(f"dtype {dt} is not supported by the decode kernels (float32/float16/bfloat16)")


def _require_cuda(name: str, *tensors: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name}: CUDA tensors required (the B200 kernels have no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name}: tensors on different devices ({dev} vs {t.device})")
    return dev


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


# ----------------------------------------------------------------------------- workspace
_WORKSPACES: Dict[Tuple, torch.Tensor] = {}


def paged_attn_workspace(B: int, H: int, D: int, max_blocks: int, device: torch.device) -> torch.Tensor:
    """Zero-filled workspace for ``paged_decode_attention`` over ``B`` sequences with
    block tables of ``max_blocks`` columns (reusable on one stream)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = N.load().spd_paged_decode_attn_workspace_size(B, H, D, max_blocks, idx)
    if n == 0:
        raise RuntimeError("paged_attn_workspace: could not size workspace (no CUDA device?)")
    return torch.zeros(n, dtype=torch.uint8, device=device)


def cross_attn_workspace(B: int, H: int, D: int, device: torch.device) -> torch.Tensor:
    """Zero-filled workspace for ``cross_attention`` (reusable on one stream)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    n = N.load().spd_cross_attn_workspace_size(B, H, D, idx)
    if n == 0:
        raise RuntimeError("cross_attn_workspace: could not size workspace (no CUDA device?)")
    return torch.zeros(n, dtype=torch.uint8, device=device)


def _cached_workspace(kind: str, B: int, H: int, D: int, device: torch.device, max_blocks: int = 0) -> torch.Tensor:
    """One zero-initialised workspace per (op, geometry, device, stream).  The counter and
    partial regions are laid out by geometry, so a workspace is never shared between
    geometries (stale partials would otherwise land in another call's counters)."""
    key = (kind, B, H, D, max_blocks, device, torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None:
        ws = (paged_attn_workspace(B, H, D, max_blocks, device) if kind == "paged"
              else cross_attn_workspace(B, H, D, device))
        _WORKSPACES[key] = ws
    return ws


def read_error_word(buf: torch.Tensor) -> int:
    """Reads the device error word (SPD_DEVERR_* flags) at the start of a workspace or
    int32 error buffer.  Synchronises the current stream; not for use during capture."""
    word = N.C.c_int32(0)
    N.check(N.load().spd_read_error_word(buf.data_ptr(), N.C.byref(word), _stream_handle()),
            "spd_read_error_word")
    return int(word.value)


def clear_error_word(buf: torch.Tensor) -> None:
    buf.view(torch.uint8)[:4].zero_()


# ----------------------------------------------------------------------------- op (1)
def paged_decode_attention(
    q: torch.Tensor,
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None,
    k_new: Optional[torch.Tensor] = None,
    v_new: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Single-query attention over a paged K/V pool, walking the block tables.

    q [B, H, D] (or [B, H, 1, D]); k_pool/v_pool [num_blocks, block_size, H, D];
    block_tables int32 [B, max_blocks]; context_lens int32 [B] (tokens attended,
    including the new one).  When k_new/v_new [B, H, D] are given they are written to
    position context_lens-1 first (op 3 fused).  Returns out [B, H, D].
    """
    dev = _require_cuda("paged_decode_attention", q, k_pool, v_pool, block_tables, context_lens, out, k_new, v_new)
    if q.dim() == 4:
        q = q.reshape(q.shape[0], q.shape[1], q.shape[3])
    B, H, D = q.shape
    if k_pool.dim() != 4 or k_pool.shape[2] != H or k_pool.shape[3] != D or v_pool.shape != k_pool.shape:
        raise RuntimeError(f"paged_decode_attention: pools {tuple(k_pool.shape)} do not match q {tuple(q.shape)}")
    num_blocks, block_size = k_pool.shape[0], k_pool.shape[1]
    if block_tables.dtype != torch.int32 or context_lens.dtype != torch.int32:
        raise RuntimeError("paged_decode_attention: block_tables and context_lens must be int32")
    if block_tables.dim() != 2 or block_tables.shape[0] != B or context_lens.shape != (B,):
        raise RuntimeError("paged_decode_attention: block_tables [B, max_blocks], context_lens [B] expected")
    for t, n in ((q, "q"), (k_pool, "k_pool"), (v_pool, "v_pool"), (block_tables, "block_tables"),
                 (context_lens, "context_lens")):
        if not t.is_contiguous():
            raise RuntimeError(f"paged_decode_attention: {n} must be contiguous")
    if k_pool.dtype != q.dtype or v_pool.dtype != q.dtype:
        raise RuntimeError("paged_decode_attention: q and pools must share a dtype")
    if (k_new is None) != (v_new is None):
        raise RuntimeError("paged_decode_attention: give both k_new and v_new or neither")
    if k_new is not None:
        k_new = k_new.reshape(B, H, D)
        v_new = v_new.reshape(B, H, D)
        if not (k_new.is_contiguous() and v_new.is_contiguous()) or k_new.dtype != q.dtype or v_new.dtype != q.dtype:
            raise RuntimeError("paged_decode_attention: k_new/v_new must be contiguous [B, H, D] of q's dtype")
    if out is None:
        out = torch.empty((B, H, D), dtype=q.dtype, device=dev)
    elif out.shape != (B, H, D) or not out.is_contiguous() or out.dtype != q.dtype:
        raise RuntimeError("paged_decode_attention: out must be a contiguous [B, H, D] tensor of q's dtype")
    if workspace is None:
        workspace = _cached_workspace("paged", B, H, D, dev, block_tables.shape[1])
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    lib = N.load()
    rc = lib.spd_paged_decode_attn(
        q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), block_tables.data_ptr(), context_lens.data_ptr(),
        out.data_ptr(), B, H, D, block_size, block_tables.shape[1], num_blocks, float(scale), dtype_code(q.dtype),
        _ptr(k_new), _ptr(v_new), workspace.data_ptr(), workspace.numel(), _stream_handle())
    N.check(rc, "spd_paged_decode_attn")
    return out


# ----------------------------------------------------------------------------- op (2)
def cross_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    valid_lens: torch.Tensor,
    scale: Optional[float] = None,
    out: Optional[torch.Tensor] = None,
    workspace: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Single-query attention over contiguous encoder K/V [B, H, T, D] (any batch and
    head strides, rows contiguous), attending positions t < valid_lens[b]."""
    dev = _require_cuda("cross_attention", q, k, v, valid_lens, out)
    if q.dim() == 4:
        q = q.reshape(q.shape[0], q.shape[1], q.shape[3])
    B, H, D = q.shape
    if k.dim() != 4 or k.shape[0] != B or k.shape[1] != H or k.shape[3] != D or v.shape != k.shape:
        raise RuntimeError(f"cross_attention: k/v {tuple(k.shape)} do not match q {tuple(q.shape)}")
    T = k.shape[2]
    if k.stride(3) != 1 or k.stride(2) != D or v.stride() != k.stride():
        raise RuntimeError("cross_attention: k and v need contiguous [T, D] rows and identical strides")
    if valid_lens.dtype != torch.int32 or valid_lens.shape != (B,) or not valid_lens.is_contiguous():
        raise RuntimeError("cross_attention: valid_lens must be a contiguous int32 [B] tensor")
    if not q.is_contiguous() or k.dtype != q.dtype or v.dtype != q.dtype:
        raise RuntimeError("cross_attention: q must be contiguous and share k/v's dtype")
    if out is None:
        out = torch.empty((B, H, D), dtype=q.dtype, device=dev)
    if workspace is None:
        workspace = _cached_workspace("cross", B, H, D, dev)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rc = N.load().spd_cross_attn(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), valid_lens.data_ptr(), out.data_ptr(), B, H, D, T,
        k.stride(0), k.stride(1), float(scale), dtype_code(q.dtype), workspace.data_ptr(), workspace.numel(),
        _stream_handle())
    N.check(rc, "spd_cross_attn")
    return out


# ----------------------------------------------------------------------------- op (3)
def kv_append(
    k_src: torch.Tensor,
    v_src: Optional[torch.Tensor],
    k_pool: torch.Tensor,
    v_pool: Optional[torch.Tensor],
    block_tables: torch.Tensor,
    positions: torch.Tensor,
    error_word: Optional[torch.Tensor] = None,
) -> None:
    """Writes T tokens per sequence into the paged pools, bit-exactly.

    k_src/v_src [B, H, T, D] (any strides, D contiguous; [B, H, D] means T=1);
    positions int32 [B] = first position written (< 0 skips the sequence)."""
    _require_cuda("kv_append", k_src, v_src, k_pool, v_pool, block_tables, positions, error_word)
    if k_src.dim() == 3:
        k_src = k_src.unsqueeze(2)
        v_src = None if v_src is None else v_src.unsqueeze(2)
    B, H, T, D = k_src.shape
    if k_src.stride(3) != 1 or (v_src is not None and (v_src.shape != k_src.shape or v_src.stride() != k_src.stride())):
        raise RuntimeError("kv_append: sources need a contiguous last dim and identical K/V strides")
    if k_pool.dim() != 4 or k_pool.shape[2] != H or k_pool.shape[3] != D or not k_pool.is_contiguous():
        raise RuntimeError("kv_append: pool must be contiguous [num_blocks, block_size, H, D]")
    if (v_src is None) != (v_pool is None) or (v_pool is not None and v_pool.shape != k_pool.shape):
        raise RuntimeError("kv_append: v_src and v_pool must both be given (same shape as K) or both omitted")
    if k_src.dtype != k_pool.dtype or (v_src is not None and v_src.dtype != k_pool.dtype):
        raise RuntimeError("kv_append: source and pool dtypes differ")
    if block_tables.dtype != torch.int32 or positions.dtype != torch.int32 or not block_tables.is_contiguous():
        raise RuntimeError("kv_append: block_tables and positions must be int32 (tables contiguous)")
    rc = N.load().spd_kv_append(
        k_src.data_ptr(), _ptr(v_src), k_src.stride(0), k_src.stride(1), k_src.stride(2), k_pool.data_ptr(),
        _ptr(v_pool), block_tables.data_ptr(), positions.data_ptr(), B, T, H, D, k_pool.shape[1],
        block_tables.shape[1], k_pool.shape[0], dtype_code(k_pool.dtype), _ptr(error_word), _stream_handle())
    N.check(rc, "spd_kv_append")


# ----------------------------------------------------------------------------- op (5)
def block_gather(
    pool: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    T_out: int,
    out: Optional[torch.Tensor] = None,
    zero_pad: bool = True,
    error_word: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Gathers paged blocks into head-major [B, H, T_out, D]: bit-exactly
    ``pool[table].view(-1, H, D)[:T].permute(1, 0, 2)`` per sequence, zero padded."""
    dev = _require_cuda("block_gather", pool, block_tables, seq_lens, out, error_word)
    num_blocks, block_size, H, D = pool.shape
    if block_tables.dim() != 2 or block_tables.dtype != torch.int32 or not block_tables.is_contiguous():
        raise RuntimeError("block_gather: block_tables must be contiguous int32 [B, max_blocks]")
    B = block_tables.shape[0]
    if seq_lens.dtype != torch.int32 or seq_lens.shape != (B,) or not pool.is_contiguous():
        raise RuntimeError("block_gather: seq_lens int32 [B] and a contiguous pool required")
    if out is None:
        out = (torch.zeros if not zero_pad else torch.empty)((B, H, T_out, D), dtype=pool.dtype, device=dev)
    if out.shape != (B, H, T_out, D) or out.stride(3) != 1 or out.stride(2) != D or out.stride(1) != T_out * D:
        raise RuntimeError("block_gather: out must be [B, H, T_out, D] with contiguous [H, T_out, D] per batch")
    rc = N.load().spd_block_gather(
        pool.data_ptr(), block_tables.data_ptr(), seq_lens.data_ptr(), out.data_ptr(), B, H, D, block_size,
        block_tables.shape[1], num_blocks, T_out, out.stride(0), int(bool(zero_pad)), dtype_code(pool.dtype),
        _ptr(error_word), _stream_handle())
    N.check(rc, "spd_block_gather")
    return out


# ----------------------------------------------------------------------------- op (4)
def stack_cross_kv_weights(layers) -> Tuple[torch.Tensor, torch.Tensor]:
    """Stacks every decoder layer's cross-attention k_proj / v_proj into the GEMM operand
    of ``cross_kv_project``: W [L*2*H*D, d_model] in (layer, k|v, head, dim) row order and
    the matching bias (zeros for k_proj, which has none; speech_serving/models.py:557-559,
    transformers WhisperAttention k_proj bias=False, v_proj bias=True)."""
    ws, bs = [], []
    for layer in layers:
        att = layer.encoder_attn
        for proj in (att.k_proj, att.v_proj):
            ws.append(proj.weight)
            bs.append(proj.bias if proj.bias is not None else torch.zeros(proj.weight.shape[0], dtype=proj.weight.dtype,
                                                                          device=proj.weight.device))
    return torch.cat(ws, 0).contiguous(), torch.cat(bs, 0).contiguous()


def cross_kv_project(
    enc_out: torch.Tensor,
    w_kv: torch.Tensor,
    b_kv: Optional[torch.Tensor],
    out: torch.Tensor,
    slot_ids: Optional[torch.Tensor] = None,
    error_word: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One tcgen05 GEMM that projects the encoder output into every decoder layer's
    cross-attention K and V, written into the graph-slot layout.

    enc_out [B, T, d_model]; w_kv [L*2*H*D, d_model] (``stack_cross_kv_weights``);
    b_kv [L*2*H*D] or None; out [S, L, 2, H, T_out, D] with T <= T_out (rows t >= T
    untouched); slot_ids int32 [B] picks each request's slot (default: slot b)."""
    _require_cuda("cross_kv_project", enc_out, w_kv, b_kv, out, slot_ids, error_word)
    if enc_out.dim() != 3 or not enc_out.is_contiguous() or not w_kv.is_contiguous():
        raise RuntimeError("cross_kv_project: enc_out [B, T, d_model] and w_kv must be contiguous")
    B, T, d = enc_out.shape
    if out.dim() != 6 or not out.is_contiguous():
        raise RuntimeError("cross_kv_project: out must be a contiguous [S, L, 2, H, T_out, D] tensor")
    S, L, two, H, T_out, D = out.shape
    if two != 2 or w_kv.shape != (L * 2 * H * D, d) or T > T_out:
        raise RuntimeError(f"cross_kv_project: w_kv {tuple(w_kv.shape)} / out {tuple(out.shape)} / T={T} mismatch")
    if b_kv is not None and (b_kv.shape != (L * 2 * H * D,) or not b_kv.is_contiguous()):
        raise RuntimeError("cross_kv_project: b_kv must be a contiguous [L*2*H*D] tensor")
    for t in (w_kv, b_kv, out):
        if t is not None and t.dtype != enc_out.dtype:
            raise RuntimeError("cross_kv_project: all tensors must share enc_out's dtype")
    if slot_ids is not None:
        if slot_ids.dtype != torch.int32 or slot_ids.shape != (B,):
            raise RuntimeError("cross_kv_project: slot_ids must be int32 [B]")
    elif B > S:
        raise RuntimeError("cross_kv_project: more requests than slots and no slot_ids")
    rc = N.load().spd_cross_kv_project(
        enc_out.data_ptr(), w_kv.data_ptr(), _ptr(b_kv), out.data_ptr(), _ptr(slot_ids), B, T, d, L, H, D, T_out,
        out.stride(0), dtype_code(enc_out.dtype), _ptr(error_word), _stream_handle())
    N.check(rc, "spd_cross_kv_project")
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None, gelu: bool = False,
           out: Optional[torch.Tensor] = None, groups: int = 1,
           error_word: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``act(x @ weight.T + bias)`` for a small batch (x [M, K], M <= 64, K a multiple
    of 64; weight [N, K] as nn.Linear keeps it; 16-bit dtypes) on the tensor cores, GELU
    (erf form) fused when ``gelu``.  With ``groups`` > 1 the N output columns are split into
    that many equal groups written as separate [M, N / groups] tensors, stacked:
    out [groups, M, N / groups] (a packed q|k|v weight gives q, k and v)."""
    _require_cuda("linear", x, weight, bias, out, error_word)
    if x.dim() != 2 or weight.dim() != 2 or not x.is_contiguous() or not weight.is_contiguous():
        raise RuntimeError("linear: x [M, K] and weight [N, K] must be contiguous 2-D tensors")
    M, K = x.shape
    Nf = weight.shape[0]
    if weight.shape[1] != K or Nf % groups:
        raise RuntimeError(f"linear: weight {tuple(weight.shape)} does not match x {tuple(x.shape)} / groups={groups}")
    for t in (weight, bias, out):
        if t is not None and t.dtype != x.dtype:
            raise RuntimeError("linear: all tensors must share x's dtype")
    if bias is not None and (bias.shape != (Nf,) or not bias.is_contiguous()):
        raise RuntimeError("linear: bias must be a contiguous [N] tensor")
    gc = Nf // groups
    shape = (groups, M, gc) if groups > 1 else (M, Nf)
    if out is None:
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
    elif tuple(out.shape) != shape or not out.is_contiguous():
        raise RuntimeError(f"linear: out must be a contiguous {shape} tensor")
    rc = N.load().spd_linear(x.data_ptr(), weight.data_ptr(), _ptr(bias), out.data_ptr(), M, Nf, K, gc, M * gc,
                             N.SPD_ACT_GELU if gelu else N.SPD_ACT_NONE, dtype_code(x.dtype), _ptr(error_word),
                             _stream_handle())
    N.check(rc, "spd_linear")
    return out


# ----------------------------------------------------------------------------- decoder-layer glue
def add_layernorm(x: torch.Tensor, delta: Optional[torch.Tensor], ln, out_y: Optional[torch.Tensor] = None):
    """``x += delta`` (in place, rounded to x's dtype) and ``LayerNorm(x)`` in one kernel;
    ``ln`` is an ``nn.LayerNorm`` over the last dimension.  Returns (x, y).  With
    ``delta`` None only y = LayerNorm(x) is computed.  ``out_y`` may be a [rows, cols] view
    of a wider row-major buffer (unit column stride)."""
    _require_cuda("add_layernorm", x, delta)
    cols = x.shape[-1]
    if not x.is_contiguous() or (delta is not None and (delta.shape != x.shape or not delta.is_contiguous())):
        raise RuntimeError("add_layernorm: x and delta must be contiguous and of one shape")
    w, b = ln.weight, ln.bias
    if w is None or b is None or w.dtype != x.dtype or b.dtype != x.dtype or (delta is not None and delta.dtype != x.dtype):
        raise RuntimeError("add_layernorm: one dtype for x, delta and the LayerNorm's weight and bias")
    rows = x.numel() // cols
    y = torch.empty_like(x) if out_y is None else out_y
    if out_y is not None and (y.dtype != x.dtype or y.shape[-1] != cols or y.numel() != x.numel() or y.stride(-1) != 1
                              or (y.dim() > 1 and rows > 1 and y.dim() != 2)):
        raise RuntimeError("add_layernorm: out_y must be [rows, cols] of x's dtype with unit column stride")
    y_ld = y.stride(0) if (y.dim() == 2 and rows > 1) else cols
    rc = N.load().spd_add_layernorm(x.data_ptr(), _ptr(delta), w.data_ptr(), b.data_ptr(),
                                    x.data_ptr() if delta is not None else None, y.data_ptr(), rows, cols, y_ld,
                                    float(ln.eps), dtype_code(x.dtype), _stream_handle())
    N.check(rc, "spd_add_layernorm")
    return x, y


def argmax_rows(x: torch.Tensor, cols: Optional[int] = None, skip: Optional[torch.Tensor] = None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy pick over the first ``cols`` columns of each row of ``x`` [rows, ld]:
    ``torch.argmax(x[:, :cols].masked_fill(skip, -inf), dim=-1)`` in one kernel (the first
    maximal column; a NaN wins), with ``skip`` a bool [cols] mask or None.  Returns int64
    [rows]."""
    _require_cuda("argmax_rows", x, skip, out)
    if x.dim() != 2 or x.stride(1) != 1:
        raise RuntimeError("argmax_rows: x must be [rows, ld] with unit column stride")
    rows = x.shape[0]
    cols = x.shape[1] if cols is None else int(cols)
    if not 0 < cols <= x.shape[1]:
        raise RuntimeError(f"argmax_rows: cols {cols} outside [1, {x.shape[1]}]")
    if skip is not None and (skip.dtype != torch.bool or skip.numel() < cols or not skip.is_contiguous()):
        raise RuntimeError("argmax_rows: skip must be a contiguous bool mask of at least cols entries")
    if out is None:
        out = torch.empty(rows, dtype=torch.long, device=x.device)
    elif out.dtype != torch.long or out.shape != (rows,) or not out.is_contiguous():
        raise RuntimeError("argmax_rows: out must be a contiguous int64 [rows] tensor")
    ld = x.stride(0) if rows > 1 else x.shape[1]
    rc = N.load().spd_argmax_rows(x.data_ptr(), rows, cols, ld, _ptr(skip), out.data_ptr(), dtype_code(x.dtype),
                                  _stream_handle())
    N.check(rc, "spd_argmax_rows")
    return out
