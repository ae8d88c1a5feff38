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
  non-blocking copies).
* Prompt prefill can be folded into the graph: a slot assigned with its prompt starts at
  position 0 and, while its position is inside the prompt, the step feeds the next prompt
  token instead of the argmax.  Each prompt token's K/V is written by the fused append of
  the paged kernel; the outputs of the first P-1 steps are dropped at readback.  New tokens are copied into a pinned host ring after each
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
MAX_FOLDED_PROMPT = 8  # longest prompt the graph can prefill


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
        self.skip_steps = 0  # folded prefill: steps whose outputs are prompt positions
        self.drop_tokens = 0  # ring entries still to drop at readback


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
        self.prompt_ids = torch.zeros((S, MAX_FOLDED_PROMPT), dtype=torch.long, device=dev)
        self.prompt_lens = torch.zeros(S, dtype=torch.int32, device=dev)  # 0: prefilled outside the graph
        # S slots plus one spare that batched encoder graphs write their padding rows into
        self.cross_kv_all = torch.zeros((S + 1, L, 2, H, max_enc_len, D), dtype=self.dtype, device=dev)
        self.cross_kv = self.cross_kv_all[:S]
        self.spare_slot = S
        self.buckets = batch_buckets(S)
        self.paged_ws = {n: ops.paged_attn_workspace(n, H, D, max_blocks, dev) for n in self.buckets}
        self.cross_ws = {n: ops.cross_attn_workspace(n, H, D, dev) for n in self.buckets}

    def bucket_for(self, highest_slot: int) -> int:
        for b in self.buckets:
            if b > highest_slot:
                return b
        return self.buckets[-1]

    def upload_slot(self, slot: int, token: int, ctx_len: int, cross_len: int, table: Sequence[int],
                    prompt: Optional[Sequence[int]] = None) -> None:
        """Stream-ordered, non-blocking writes of one slot's row from pinned host memory.
        With ``prompt`` the slot starts at position 0 on prompt[0] (folded prefill)."""
        if len(table) > self.max_blocks:
            raise RuntimeError(f"block table of {len(table)} blocks exceeds max_blocks={self.max_blocks}")
        i32 = torch.zeros(self.max_blocks + 3, dtype=torch.int32)
        if table:
            i32[: len(table)] = torch.tensor(list(table), dtype=torch.int32)
        i64 = torch.zeros(1 + MAX_FOLDED_PROMPT, dtype=torch.long)
        if prompt is not None:
            if not 1 <= len(prompt) <= MAX_FOLDED_PROMPT:
                raise ValueError(f"folded prompts hold 1..{MAX_FOLDED_PROMPT} tokens, got {len(prompt)}")
            i64[0] = int(prompt[0])
            i64[1 : 1 + len(prompt)] = torch.tensor(list(prompt), dtype=torch.long)
            i32[self.max_blocks :] = torch.tensor([1, cross_len, len(prompt)], dtype=torch.int32)
        else:
            i64[0] = int(token)
            i32[self.max_blocks :] = torch.tensor([ctx_len, cross_len, 0], dtype=torch.int32)
        i32, i64 = i32.pin_memory(), i64.pin_memory()
        mb = self.max_blocks
        self.block_tables[slot].copy_(i32[:mb], non_blocking=True)
        self.ctx_lens[slot : slot + 1].copy_(i32[mb : mb + 1], non_blocking=True)
        self.cross_lens[slot : slot + 1].copy_(i32[mb + 1 : mb + 2], non_blocking=True)
        self.prompt_lens[slot : slot + 1].copy_(i32[mb + 2 : mb + 3], non_blocking=True)
        self.token_ids[slot : slot + 1].copy_(i64[:1], non_blocking=True)
        if prompt is not None:
            self.prompt_ids[slot].copy_(i64[1:], non_blocking=True)

    def set_table(self, slot: int, table: Sequence[int]) -> None:
        row = torch.zeros(self.max_blocks, dtype=torch.int32)
        row[: len(table)] = torch.tensor(list(table), dtype=torch.int32)
        self.block_tables[slot].copy_(row.pin_memory(), non_blocking=True)

    def deactivate(self, slot: int) -> None:
        self.ctx_lens[slot].zero_()
        self.cross_lens[slot].zero_()
        self.prompt_lens[slot].zero_()

    def forward_step(self, n: int) -> None:
        """One decode step over slots [0, n); graph-capturable.  A slot whose next
        position is still inside its folded prompt is fed that prompt token."""
        nxt = self.model.decode_step_paged(self, n)
        self.next_tokens[:n].copy_(nxt)
        pos = self.ctx_lens[:n]  # position of the token fed next
        forced = self.prompt_ids[:n].gather(1, pos.clamp(max=MAX_FOLDED_PROMPT - 1).long()[:, None])[:, 0]
        self.token_ids[:n].copy_(torch.where(pos < self.prompt_lens[:n], forced, nxt))
        self.ctx_lens[:n] += (pos > 0).to(torch.int32)


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
                    initial_tok: Optional[int], initial_self_kv: Any = None, slot_idx: Optional[int] = None,
                    enc_seq_len: Optional[int] = None, fold_prompt: Optional[Sequence[int]] = None) -> int:
        """Activates a slot.  Either the prompt K/V is already in the request's decoder
        blocks and ``initial_tok`` is its first token, or ``fold_prompt`` holds the prompt
        and the graph prefills it.  Cross K/V come from ``enc_kv_layers`` (copied in)
        unless the caller already wrote them into ``cross_kv[slot]`` (block gather or
        projection GEMM) and passes ``enc_seq_len``."""
        if slot_idx is None:
            slot_idx = self.reserve_slot()
        s = self.slots[slot_idx]
        if enc_kv_layers is not None:
            enc_seq_len = self.model.cross_kv_from_encoder(enc_kv_layers, self.cross_kv, slot_idx)
        T = min(int(enc_seq_len or self.max_enc_len), self.max_enc_len)
        s.active, s.req = True, req
        s.max_new_tokens = req.max_new_tokens
        s.eos_token_id = req.eos_token_id
        s.enc_seq_len = T
        s.readback_start = self._step_in_k
        s.last_readback_trace = []
        if fold_prompt is not None:
            s.decoder_seq_len, s.last_token_id, s.generated_count = 0, int(fold_prompt[-1]), 0
            s.pending_tokens = []
            s.skip_steps = s.drop_tokens = len(fold_prompt) - 1
            self.upload_slot(slot_idx, 0, 1, T, req.decoder_block_table, prompt=fold_prompt)
        else:
            s.decoder_seq_len, s.last_token_id, s.generated_count = prompt_len, initial_tok, 1
            s.pending_tokens = [initial_tok]
            s.skip_steps = s.drop_tokens = 0
            self.upload_slot(slot_idx, initial_tok, prompt_len + 1, T, req.decoder_block_table)
        return slot_idx

    def release_slot(self, slot_idx: int) -> None:
        s = self.slots[slot_idx]
        s.active, s.req = False, None
        s.pending_tokens, s.readback_start, s.last_readback_trace = [], 0, []
        s.skip_steps = s.drop_tokens = 0
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
                if s.skip_steps > 0:
                    s.skip_steps -= 1
                else:
                    s.generated_count += 1

    def reset_window(self) -> None:
        """Drops the current readback window (after a failed step: its tokens are void)."""
        self._step_in_k = 0
        self._window_buckets = []
        for s in self.slots:
            s.readback_start = 0

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
                first = min(self._step_in_k, s.readback_start + s.drop_tokens)
                s.drop_tokens -= first - s.readback_start
                toks = [ring[k][i] for k in range(first, self._step_in_k)]
                s.last_readback_trace = [{"bucket": self._window_buckets[k], "readback_position": k}
                                         for k in range(first, self._step_in_k)]
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
        b = self.cross_kv_all.numel() * self.cross_kv_all.element_size() + self.block_tables.numel() * 4
        b += sum(w.numel() for w in self.paged_ws.values()) + sum(w.numel() for w in self.cross_ws.values())
        return b / 1024 ** 2
