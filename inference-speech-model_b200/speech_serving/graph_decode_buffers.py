"""Decode slots and CUDA-graph replay for the paged decode hot path.

Same role and method names as the reference's GraphDecodeBuffers
(speech_serving/graph_decode_buffers.py:124-638: assign_slot, release_slot,
capture_all_buckets, prepare_replay, replay_step, should_readback, sync_tokens,
vram_overhead_mb).  The design differs where the reference worked around the lack of
a paged kernel:

* Self-K/V stays in the decoder BlockManager's paged pool.  Each slot owns an int32 row
  of block ids [S, max_blocks] and an attended length; the graph reads the pool
  directly.  So there are no length-bucketed K/V copies, no bucket promotion copies
  (:483-500), no attention masks (:513-537), and no `-10000` fills.
* Graphs are captured per BATCH bucket (1, 2, 4, ... up to max_slots): a replay covers
  slots [0, n), where n is the smallest bucket above the highest active slot.  Slots are
  handed out lowest-first.
* Per step the host uploads nothing.  Tokens and lengths advance on the device inside
  the graph; only slot assignment/release touch device state (stream-ordered
  non-blocking copies).  New tokens are copied into a pinned host ring after each
  replay and read back every `readback_k` steps (:586-621).
* Cross K/V of the slots live in one [S, L, 2, H, T_max, D] buffer, filled once at
  handoff (direct copy, block gather, or the projection GEMM writing straight into it).
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from . import ops

SELF_KV_BUCKETS = [64, 128, 256, 448]  # the reference's length buckets; kept for callers
BATCH_BUCKETS = [1, 2, 4, 8, 16, 32, 64]
MAX_SLOTS = 4
DEFAULT_READBACK_K = 1
MAX_BLOCKS = 64


def batch_buckets(max_slots: int) -> List[int]:
    return sorted(set([b for b in BATCH_BUCKETS if b < max_slots] + [max_slots]))


class SlotInfo:
    """Host-side metadata of one decode slot (reference :102-121)."""

    def __init__(self, slot_idx: int):
        self.slot_idx = slot_idx
        self.active = False
        self.req = None
        self.decoder_seq_len = 0
        self.last_token_id = 0
        self.generated_count = 0
        self.max_new_tokens = 0
        self.eos_token_id = None
        self.enc_seq_len = 0
        self.readback_start = 0
        self.assignment_count = 0
        self.reused = False
        self.pending_tokens: List[int] = []
        self.last_readback_trace: List[Dict[str, int]] = []


class PagedDecodeState:
    """Device-resident decode state of all slots, read by the models' decode_step_paged."""

    def __init__(self, model: Any, block_manager: Any, max_slots: int, max_blocks: int = MAX_BLOCKS,
                 max_enc_len: int = 1500, device: str = "cuda", dtype: Optional[torch.dtype] = None):
        self.model = model
        self.device = torch.device(device)
        self.dtype = dtype or block_manager.dtype
        self.max_slots, self.max_blocks, self.max_enc_len = max_slots, max_blocks, max_enc_len
        self.num_decoder_layers, self.num_heads = model.num_decoder_layers, model.num_heads
        self.head_dim, self.hidden_dim = model.head_dim, model.hidden_dim
        self.block_manager = block_manager
        self.key_pool, self.value_pool = block_manager.key_pool, block_manager.value_pool
        S, L, H, D = max_slots, self.num_decoder_layers, self.num_heads, self.head_dim
        dev = self.device
        self.token_ids = torch.zeros(S, dtype=torch.long, device=dev)
        self.next_tokens = torch.zeros(S, dtype=torch.long, device=dev)
        self.ctx_lens = torch.zeros(S, dtype=torch.int32, device=dev)  # attended length incl. new token; 0 = idle
        self.cross_lens = torch.zeros(S, dtype=torch.int32, device=dev)
        self.block_tables = torch.zeros((S, max_blocks), dtype=torch.int32, device=dev)
        self.cross_kv = torch.zeros((S, L, 2, H, max_enc_len, D), dtype=self.dtype, device=dev)
        self.buckets = batch_buckets(S)
        self.paged_ws = {n: ops.paged_attn_workspace(n, H, D, max_blocks, dev) for n in self.buckets}
        self.cross_ws = {n: ops.cross_attn_workspace(n, H, D, dev) for n in self.buckets}

    def bucket_for(self, highest_slot: int) -> int:
        for b in self.buckets:
            if b > highest_slot:
                return b
        return self.buckets[-1]

    def upload_slot(self, slot: int, token: int, ctx_len: int, cross_len: int, table: Sequence[int]) -> None:
        """Stream-ordered, non-blocking writes of one slot's row from pinned host memory."""
        row = torch.zeros(self.max_blocks, dtype=torch.int32)
        if len(table) > self.max_blocks:
            raise RuntimeError(f"block table of {len(table)} blocks exceeds max_blocks={self.max_blocks}")
        if table:
            row[: len(table)] = torch.tensor(list(table), dtype=torch.int32)
        scal = torch.tensor([ctx_len, cross_len], dtype=torch.int32)
        tok = torch.tensor([token], dtype=torch.long)
        row, scal, tok = row.pin_memory(), scal.pin_memory(), tok.pin_memory()
        self.block_tables[slot].copy_(row, non_blocking=True)
        self.ctx_lens[slot : slot + 1].copy_(scal[:1], non_blocking=True)
        self.cross_lens[slot : slot + 1].copy_(scal[1:], non_blocking=True)
        self.token_ids[slot : slot + 1].copy_(tok, non_blocking=True)

    def set_table(self, slot: int, table: Sequence[int]) -> None:
        row = torch.zeros(self.max_blocks, dtype=torch.int32)
        row[: len(table)] = torch.tensor(list(table), dtype=torch.int32)
        self.block_tables[slot].copy_(row.pin_memory(), non_blocking=True)

    def deactivate(self, slot: int) -> None:
        self.ctx_lens[slot].zero_()
        self.cross_lens[slot].zero_()

    def forward_step(self, n: int) -> None:
        """One decode step over slots [0, n); graph-capturable."""
        nxt = self.model.decode_step_paged(self, n)
        self.next_tokens[:n].copy_(nxt)
        self.token_ids[:n].copy_(nxt)
        self.ctx_lens[:n] += (self.ctx_lens[:n] > 0).to(torch.int32)


class GraphDecodeBuffers(PagedDecodeState):
    """Slots + per-batch-bucket CUDA graphs (reference speech_serving/graph_decode_buffers.py:124)."""

    def __init__(self, model: Any, device: str = "cuda", dtype: Optional[torch.dtype] = None,
                 max_slots: int = MAX_SLOTS, readback_k: int = DEFAULT_READBACK_K, max_blocks: int = MAX_BLOCKS,
                 max_enc_len: int = 1500, non_blocking_copies: bool = True, zero_slot_buffers_on_release: bool = False,
                 force_bucket: Optional[int] = None, block_manager: Any = None, use_graphs: bool = True):
        if block_manager is None:
            raise ValueError("GraphDecodeBuffers needs the decoder BlockManager whose pool the slots read")
        super().__init__(model, block_manager, max_slots, max_blocks, max_enc_len, device, dtype)
        self.readback_k = max(1, readback_k)
        self.non_blocking_copies = non_blocking_copies
        self.zero_slot_buffers_on_release = zero_slot_buffers_on_release
        if force_bucket is not None and force_bucket not in self.buckets:
            raise ValueError(f"force_bucket must be one of {self.buckets}, got {force_bucket}")
        self.force_bucket = force_bucket
        self.use_graphs = use_graphs and self.device.type == "cuda"
        self.slots = [SlotInfo(i) for i in range(max_slots)]
        # one contiguous pinned row per step of the readback window
        self.h_token_ring = torch.zeros((self.readback_k, max_slots), dtype=torch.long).pin_memory()
        self._step_in_k = 0
        self._step_counter = 0
        self._window_buckets: List[int] = []
        self._readback_event = torch.cuda.Event()
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self._graph_pool = None
        if self.use_graphs:
            self.capture_all_buckets()

    # The reference keeps length-bucketed cross caches in ``cross_cache`` and the graph's
    # cross K/V in ``g_cross_kv``; here the one slot buffer is both.
    cross_cache = None

    @property
    def g_cross_kv(self) -> torch.Tensor:
        return self.cross_kv

    # ---- slots ---------------------------------------------------------------------------
    def find_free_slot(self) -> Optional[int]:
        for s in self.slots:
            if not s.active:
                return s.slot_idx
        return None

    def active_slot_count(self) -> int:
        return sum(1 for s in self.slots if s.active)

    def reserve_slot(self) -> int:
        idx = self.find_free_slot()
        if idx is None:
            raise RuntimeError("No free slot available in GraphDecodeBuffers!")
        s = self.slots[idx]
        s.active = True  # reserved; activated by assign_slot
        s.req = None
        s.reused = s.assignment_count > 0
        s.assignment_count += 1
        return idx

    def assign_slot(self, req: Any, enc_kv_layers: Optional[List[Tuple[torch.Tensor, torch.Tensor]]], prompt_len: int,
                    initial_tok: int, initial_self_kv: Any = None, slot_idx: Optional[int] = None,
                    enc_seq_len: Optional[int] = None) -> int:
        """Activates a slot for a request whose prompt K/V is already in its decoder blocks.
        Cross K/V come from ``enc_kv_layers`` (copied in) unless the caller already wrote
        them into ``cross_kv[slot]`` (block gather or projection GEMM) and passes
        ``enc_seq_len``."""
        if slot_idx is None:
            slot_idx = self.reserve_slot()
        s = self.slots[slot_idx]
        if enc_kv_layers is not None:
            enc_seq_len = self.model.cross_kv_from_encoder(enc_kv_layers, self.cross_kv, slot_idx)
        T = min(int(enc_seq_len or self.max_enc_len), self.max_enc_len)
        s.active, s.req = True, req
        s.decoder_seq_len = prompt_len
        s.last_token_id = initial_tok
        s.generated_count = 1
        s.max_new_tokens = req.max_new_tokens
        s.eos_token_id = req.eos_token_id
        s.enc_seq_len = T
        s.pending_tokens = [initial_tok]
        s.readback_start = self._step_in_k
        s.last_readback_trace = []
        self.upload_slot(slot_idx, initial_tok, prompt_len + 1, T, req.decoder_block_table)
        return slot_idx

    def release_slot(self, slot_idx: int) -> None:
        s = self.slots[slot_idx]
        s.active, s.req = False, None
        s.pending_tokens, s.readback_start, s.last_readback_trace = [], 0, []
        self.deactivate(slot_idx)
        if self.zero_slot_buffers_on_release:
            self.cross_kv[slot_idx].zero_()

    # ---- graphs ----------------------------------------------------------------------------
    def capture_all_buckets(self, warmup_steps: int = 3) -> None:
        """One CUDA graph per batch bucket, sharing one memory pool (reference :389-431).
        Captured with every slot idle, so no K/V is written while capturing."""
        saved = self.ctx_lens.clone(), self.cross_lens.clone(), self.token_ids.clone()
        self.ctx_lens.zero_()
        self.cross_lens.zero_()
        side = torch.cuda.Stream(device=self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            for n in self.buckets:
                for _ in range(warmup_steps):
                    self.forward_step(n)
        torch.cuda.current_stream(self.device).wait_stream(side)
        for n in self.buckets:
            g = torch.cuda.CUDAGraph()
            kw = {"pool": self._graph_pool} if self._graph_pool is not None else {}
            with torch.cuda.graph(g, stream=side, **kw):
                self.forward_step(n)
            if self._graph_pool is None:
                self._graph_pool = g.pool()
            self.graphs[n] = g
        torch.cuda.synchronize(self.device)
        self.ctx_lens.copy_(saved[0])
        self.cross_lens.copy_(saved[1])
        self.token_ids.copy_(saved[2])

    def prepare_replay(self) -> int:
        """Bucket covering every active slot; nothing is uploaded per step."""
        if self.force_bucket is not None:
            return self.force_bucket
        hi = max((s.slot_idx for s in self.slots if s.active), default=0)
        return self.bucket_for(hi)

    def replay_step(self, bucket: int) -> None:
        if self.use_graphs:
            self.graphs[bucket].replay()
        else:
            self.forward_step(bucket)
        if self._step_in_k < self.readback_k:
            self.h_token_ring[self._step_in_k].copy_(self.next_tokens, non_blocking=self.non_blocking_copies)
            self._window_buckets.append(bucket)
            self._step_in_k += 1
        self._step_counter += 1
        for s in self.slots:
            if s.active and s.req is not None:
                s.decoder_seq_len += 1
                s.generated_count += 1

    def should_readback(self) -> bool:
        if self._step_in_k >= self.readback_k:
            return True
        return any(s.active and s.req is not None and s.generated_count >= s.max_new_tokens for s in self.slots)

    def sync_tokens(self) -> List[Tuple[SlotInfo, List[int]]]:
        self._readback_event.record()
        self._readback_event.synchronize()
        ring = self.h_token_ring.tolist()
        results = []
        for i, s in enumerate(self.slots):
            if s.active and s.req is not None:
                toks = [ring[k][i] for k in range(s.readback_start, self._step_in_k)]
                s.last_readback_trace = [{"bucket": self._window_buckets[k], "readback_position": k}
                                         for k in range(s.readback_start, self._step_in_k)]
                if toks:
                    s.last_token_id = toks[-1]
                    s.pending_tokens.extend(toks)
                results.append((s, toks))
                s.readback_start = 0
        self._step_in_k = 0
        self._window_buckets = []
        return results

    def vram_overhead_mb(self) -> float:
        """Slot buffers owned here (the self-K/V lives in the BlockManager's pool)."""
        b = self.cross_kv.numel() * self.cross_kv.element_size() + self.block_tables.numel() * 4
        b += sum(w.numel() for w in self.paged_ws.values()) + sum(w.numel() for w in self.cross_ws.values())
        return b / 1024 ** 2
