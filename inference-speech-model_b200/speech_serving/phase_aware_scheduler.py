"""Phase-aware scheduler for Whisper-class models on the B200 decode hot path.

Operator surface of the reference's PhaseAwareSpeechScheduler
(speech_serving/phase_aware_scheduler.py:125-1243): the same constructor flags, the
``DualCacheRequest`` record, ``submit`` with high-water-mark back-pressure (:224-329),
the encode phase with full-input encoder caching and batching (:385-560), the handoff
(:562-719), decode steps (:722-1044), deterministic release (:1046-1081), and the
telemetry getters (:1163-1228).

What runs underneath is new:

* Every decode step — eager (``graph_decode=False``) or CUDA graph — is one call of the
  model's ``decode_step_paged`` over device-resident slots (``GraphDecodeBuffers``).  The
  paged kernel reads the decoder pool through int32 block tables and writes each new
  token's K/V into its block in the same launch.  There are no per-request working
  buffers grown with ``torch.cat`` (:1012-1018), no per-step masks, and no per-request
  Python write loops (:1004-1010).
* Cross K/V enter a request's slot once at handoff:
  - by direct copy (``graph_direct_encoder_kv``);
  - by the block-gather kernel from the encoder pool (op 5, the non-direct path, after
    the K/V were stored with the paged write kernel, op 3);
  - or, for ``PretrainedWhisperModel``, straight from the projection GEMM (op 4).

  ``cache_cross_kv`` and ``avoid_redundant_cross_kv`` therefore change nothing: the
  gather already happens once per request.
* A full-input encoder-cache hit (:492-530) skips the encoder and then runs the same
  handoff from the cached blocks, so the request is prefilled and decoded like a miss.
* Prompt K/V from the prefill are written into the decoder blocks by op 3 (:672-690).
  In graph mode (``graph_fold_prefill``, default on) prompts of up to eight tokens are
  not prefilled at handoff at all: the slot starts at position 0 and the decode graph
  feeds the prompt tokens, writing their K/V with the fused append; the first token then
  arrives with a readback like every other token.
"""
from __future__ import annotations

import enum
import hashlib
import logging
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from . import ops
from .dual_cache_manager import DualCacheManager
from .graph_decode_buffers import DEFAULT_READBACK_K, MAX_BLOCKS, MAX_FOLDED_PROMPT, GraphDecodeBuffers
from .memory_guard import MemoryGuard
from .phase_timing import PhaseTimer

logger = logging.getLogger("SpeechScheduler")

WHISPER_SOT_TOKEN_ID = 50258
WHISPER_LANG_EN_TOKEN_ID = 50259
WHISPER_TRANSCRIBE_TOKEN_ID = 50359
WHISPER_NO_TIMESTAMPS_TOKEN_ID = 50363
WHISPER_EOS_TOKEN_ID = 50257
WHISPER_DEFAULT_PREFIX_TOKENS = [WHISPER_SOT_TOKEN_ID, WHISPER_LANG_EN_TOKEN_ID, WHISPER_TRANSCRIBE_TOKEN_ID,
                                 WHISPER_NO_TIMESTAMPS_TOKEN_ID]


class RequestPhase(enum.Enum):
    QUEUED = "QUEUED"
    ENCODE_PHASE = "ENCODE_PHASE"
    DECODE_PHASE = "DECODE_PHASE"
    COMPLETED = "COMPLETED"
    FAILED = "FAILED"


@dataclass
class DualCacheRequest:
    """One request (fields as in the reference, speech_serving/phase_aware_scheduler.py:73-122)."""
    id: int
    mel_features: torch.Tensor
    prompt_token_ids: torch.Tensor
    max_new_tokens: int
    arrival_time: float = 0.0
    eos_token_id: Optional[int] = None
    full_input_hash: Optional[str] = None
    phase: RequestPhase = RequestPhase.QUEUED
    encoder_seq_len: int = 0
    encoder_block_table: List[int] = field(default_factory=list)
    decoder_seq_len: int = 0
    decoder_block_table: List[int] = field(default_factory=list)
    generated_tokens: List[int] = field(default_factory=list)
    generated_count: int = 0
    last_token_id: Optional[int] = None
    done: bool = False
    slot_idx: Optional[int] = None
    graph_slot_idx: Optional[int] = None
    graph_slot_reused: bool = False
    graph_token_trace: List[Dict[str, int]] = field(default_factory=list)
    graph_extra_slot_steps: int = 0
    cached_encoder_kv: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None
    cached_decoder_kv: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None
    submission_time: Optional[float] = None
    arrival_wall_time: Optional[float] = None
    queue_wait_time: Optional[float] = None
    start_time: Optional[float] = None
    encode_done_time: Optional[float] = None
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    phase_timing: Optional[Dict[str, Any]] = None
    enc_ready: Optional[Any] = None  # CUDA event: the encoder stream has written this request's slot


class PhaseAwareSpeechScheduler:
    def __init__(
        self,
        model: Any,
        dual_cache_manager: DualCacheManager,
        memory_guard: Optional[MemoryGuard] = None,
        max_batch_size: int = 32,
        retain_encoder_cache: bool = False,
        step_delay: float = 0.0,
        verbose: bool = False,
        device: str = "cuda",
        eos_token_id: Optional[int] = None,
        max_cached_encoder_inputs: int = 100,
        cache_cross_kv: bool = False,
        batch_encoder: bool = False,
        no_sync_decode: bool = False,
        avoid_redundant_cross_kv: bool = False,
        graph_decode: bool = False,
        graph_readback_k: int = DEFAULT_READBACK_K,
        graph_non_blocking_copies: bool = True,
        graph_zero_slot_buffers_on_release: bool = False,
        graph_force_bucket: Optional[int] = None,
        graph_direct_encoder_kv: bool = False,
        phase_timing: bool = False,
        max_enc_len: int = 1500,
        max_blocks: int = MAX_BLOCKS,
        graph_fold_prefill: bool = True,
        graph_encoder: bool = True,
    ):
        self.model = model
        self.dual_cache = dual_cache_manager
        self.memory_guard = memory_guard or MemoryGuard()
        self.max_batch_size = max_batch_size
        self.retain_encoder_cache = retain_encoder_cache
        self.step_delay = step_delay
        self.verbose = verbose
        self.device = device
        self.eos_token_id = eos_token_id
        self.max_cached_encoder_inputs = max_cached_encoder_inputs
        self.cache_cross_kv = cache_cross_kv
        self.batch_encoder = batch_encoder
        self.no_sync_decode = no_sync_decode
        self.avoid_redundant_cross_kv = avoid_redundant_cross_kv
        self.graph_decode = graph_decode
        self.graph_readback_k = graph_readback_k if graph_decode else 1
        self.graph_direct_encoder_kv = bool(graph_direct_encoder_kv)
        if self.graph_direct_encoder_kv and (not self.graph_decode or self.retain_encoder_cache):
            raise ValueError("graph_direct_encoder_kv requires graph_decode=True and retain_encoder_cache=False")
        self.phase_timing = bool(phase_timing)
        self.phase_timer = PhaseTimer(self.phase_timing, device=self.device)
        self._graph_kwargs = dict(non_blocking_copies=graph_non_blocking_copies,
                                  zero_slot_buffers_on_release=graph_zero_slot_buffers_on_release,
                                  force_bucket=graph_force_bucket)
        self.max_enc_len, self.max_blocks = max_enc_len, max_blocks
        # graph mode: prompts of up to MAX_FOLDED_PROMPT tokens are prefilled by the decode graph
        self.graph_fold_prefill = bool(graph_fold_prefill) and self.graph_decode
        # graph mode + direct handoff: encoder and projection replayed as per-bucket graphs
        self.graph_encoder = bool(graph_encoder) and self.graph_decode
        self._buffers: Optional[GraphDecodeBuffers] = None

        self.queue: List[DualCacheRequest] = []
        self.active_encode: List[DualCacheRequest] = []
        self.active_decode: List[DualCacheRequest] = []
        self.completed: List[DualCacheRequest] = []
        self._next_id = 0
        self.peak_in_flight_requests = 0
        self.peak_actually_used_bytes = 0
        self.rejected_requests_count = 0
        self.in_flight_history: List[int] = []
        self.queue_wait_times: List[float] = []
        self.retained_encoder_caches: Dict[int, Tuple[List[int], float]] = {}
        self.encoder_calls = 0
        self.encoder_calls_skipped = 0
        self.encode_time_saved_s = 0.0
        self._full_input_enc_cache: Dict[str, Dict[str, Any]] = {}
        self.decode_steps = 0
        self.decode_time_s = 0.0
        # graph mode: the encoder runs on its own stream; requests it has handed off wait
        # here (slot reserved, blocks allocated) until their encoder event has completed,
        # then join the decode graph at the next step
        self._enc_stream: Optional[torch.cuda.Stream] = None
        self._pending_activation: List[Tuple[DualCacheRequest, int, int, int, List[int]]] = []

    # ---- slots (created on first use, so admission logic also runs without a GPU) --------
    @property
    def graph_buffers(self) -> GraphDecodeBuffers:
        if self._buffers is None:
            self._buffers = GraphDecodeBuffers(
                self.model, device=self.device, dtype=self.dual_cache.decoder_bm.dtype, max_slots=self.max_batch_size,
                readback_k=self.graph_readback_k, max_blocks=self.max_blocks, max_enc_len=self.max_enc_len,
                block_manager=self.dual_cache.decoder_bm, use_graphs=self.graph_decode, **self._graph_kwargs)
        return self._buffers

    # ---- admission --------------------------------------------------------------------------
    def _blocks(self, n: int, bs: int) -> int:
        return (n + bs - 1) // bs

    def submit(self, mel_features: torch.Tensor, prompt_token_ids: Optional[torch.Tensor] = None,
               max_new_tokens: int = 50, arrival_time: float = 0.0, eos_token_id: Optional[int] = None,
               arrival_wall_time: Optional[float] = None) -> Optional[int]:
        """Queues a request, or returns None when admitting it would push a pool past the
        memory guard's high-water mark even after evicting retained encoder caches."""
        enc_bm, dec_bm = self.dual_cache.encoder_bm, self.dual_cache.decoder_bm
        mel_in = mel_features.unsqueeze(0) if mel_features.dim() == 2 else mel_features
        full_hash = self._compute_full_input_hash(mel_in) if self.retain_encoder_cache else None
        is_hit = bool(full_hash and full_hash in self._full_input_enc_cache)
        enc_len = (mel_features.shape[-1] + 1) // 2
        direct = self.graph_direct_encoder_kv
        req_enc = 0 if is_hit or direct else self._blocks(enc_len, enc_bm.block_size)
        req_dec = self._blocks(max_new_tokens, dec_bm.block_size)
        q_enc = 0 if direct else sum(
            0 if (self.retain_encoder_cache and r.full_input_hash in self._full_input_enc_cache)
            else self._blocks((r.mel_features.shape[-1] + 1) // 2, enc_bm.block_size) for r in self.queue)
        q_dec = sum(self._blocks(r.max_new_tokens, dec_bm.block_size) for r in self.queue)

        def projected():
            e, d = enc_bm.get_stats(), dec_bm.get_stats()
            pe = (e["allocated_blocks"] + q_enc + req_enc) / e["num_blocks"] * 100.0 if e["num_blocks"] else 0.0
            pd = (d["allocated_blocks"] + q_dec + req_dec) / d["num_blocks"] * 100.0 if d["num_blocks"] else 0.0
            return pe, pd

        pe, pd = projected()
        hwm = self.memory_guard.high_water_mark_pct
        if pe >= hwm or pd >= hwm:
            freed = self._evict_retained_encoder_caches()
            if freed > 0:
                self.memory_guard.trigger_bulk_eviction_cleanup(freed, reason="high_water_mark_eviction")
            pe, pd = projected()
            if pe >= hwm or pd >= hwm:
                logger.warning(f"[BACKPRESSURE] utilization would reach {max(pe, pd):.1f}%; request rejected")
                self.rejected_requests_count += 1
                return None
        if prompt_token_ids is None:
            prefix = WHISPER_DEFAULT_PREFIX_TOKENS if getattr(self.model, "vocab_size", 0) >= 50364 else [1]
            prompt_token_ids = torch.tensor([prefix], dtype=torch.long)
        eos = eos_token_id if eos_token_id is not None else self.eos_token_id
        if eos is None and getattr(self.model, "vocab_size", 0) >= 50258:
            eos = WHISPER_EOS_TOKEN_ID
        now = time.perf_counter()
        req = DualCacheRequest(id=self._next_id, mel_features=mel_features.to(self.device),
                               prompt_token_ids=prompt_token_ids.to(self.device), max_new_tokens=max_new_tokens,
                               arrival_time=arrival_time,
                               arrival_wall_time=arrival_wall_time if arrival_wall_time is not None else now,
                               submission_time=now, eos_token_id=eos, full_input_hash=full_hash)
        self._next_id += 1
        self.queue.append(req)
        return req.id

    def _evict_retained_encoder_caches(self, min_blocks_to_free: int = 1) -> int:
        freed = 0
        for k in sorted(self.retained_encoder_caches, key=lambda k: self.retained_encoder_caches[k][1]):
            table, _ = self.retained_encoder_caches.pop(k)
            freed += self.dual_cache.encoder_bm.release_blocks(table)
            if min_blocks_to_free > 0 and freed >= min_blocks_to_free:
                return freed
        for h in sorted(self._full_input_enc_cache, key=lambda h: self._full_input_enc_cache[h]["last_access_time"]):
            entry = self._full_input_enc_cache.pop(h)
            if entry.get("held_by_cache", False):
                freed += self.dual_cache.encoder_bm.release_blocks(entry["block_table"])
            if min_blocks_to_free > 0 and freed >= min_blocks_to_free:
                return freed
        return freed

    def flush_retained_caches(self) -> int:
        freed = self._evict_retained_encoder_caches(min_blocks_to_free=0)
        if freed > 0:
            self.memory_guard.trigger_bulk_eviction_cleanup(freed, reason="flush_retained_caches")
        return freed

    @staticmethod
    def _compute_full_input_hash(mel_in: torch.Tensor) -> str:
        """MD5 of the whole input (fp32 bytes + dtype tag): the encoder is bidirectional,
        so only identical full inputs may share encoder K/V (reference :360-383)."""
        flat = mel_in.detach().cpu().to(torch.float32).numpy().tobytes()
        return hashlib.md5(flat + str(mel_in.dtype).encode()).hexdigest()

    # ---- encode phase ------------------------------------------------------------------------
    def _admit(self, req: DualCacheRequest, batched: bool) -> None:
        req.start_time = time.perf_counter()
        ref = req.arrival_wall_time if req.arrival_wall_time is not None else req.submission_time
        if ref is not None:
            req.queue_wait_time = req.start_time - ref
            self.queue_wait_times.append(req.queue_wait_time)
            self.phase_timer.add([req], "queue_admission_wait", req.queue_wait_time * 1000.0, 0.0)
        if self.phase_timing:
            self.phase_timer.ensure(req)["encoder_batched"] = batched
        req.phase = RequestPhase.ENCODE_PHASE

    def _process_encode_phase(self) -> None:
        enc_bm = self.dual_cache.encoder_bm
        free_slots = self.max_batch_size - self._occupied()
        if self.batch_encoder and free_slots > 1 and len(self.queue) > 1 and not self.retain_encoder_cache:
            batch, need = [], 0
            while self.queue and len(batch) < free_slots:
                n = self._blocks((self.queue[0].mel_features.shape[-1] + 1) // 2, enc_bm.block_size)
                if not self.graph_direct_encoder_kv and enc_bm.num_free_blocks < need + n:
                    break
                if self.queue[0].mel_features.shape[-1] != (batch[0].mel_features.shape[-1] if batch else
                                                           self.queue[0].mel_features.shape[-1]):
                    break  # a batch needs equal mel lengths
                r = self.queue.pop(0)
                self._admit(r, batched=True)
                batch.append(r)
                need += n
            if len(batch) > 1:
                mels = torch.stack([r.mel_features.squeeze(0) if r.mel_features.dim() == 3 else r.mel_features
                                    for r in batch]).to(self.device)
                t0 = time.perf_counter()
                with self.phase_timer.measure(batch, "encoder_forward"), torch.no_grad():
                    hidden, kv = self._encode(batch, mels)
                enc_time = time.perf_counter() - t0
                self.encoder_calls += 1
                for i, r in enumerate(batch):
                    self._setup_safely(r, hidden[i:i + 1], None if kv is None else
                                       [(k[i:i + 1], v[i:i + 1]) for k, v in kv], None, enc_time)
                return
            if batch:
                self.queue.insert(0, batch[0])

        while self._occupied() < self.max_batch_size and self.queue:
            nxt = self.queue[0]
            mel_in = nxt.mel_features.unsqueeze(0) if nxt.mel_features.dim() == 2 else nxt.mel_features
            full_hash = self._compute_full_input_hash(mel_in)
            nxt.full_input_hash = full_hash
            hit = self.retain_encoder_cache and full_hash in self._full_input_enc_cache
            need = 0 if hit or self.graph_direct_encoder_kv else self._blocks(
                (nxt.mel_features.shape[-1] + 1) // 2, enc_bm.block_size)
            if enc_bm.num_free_blocks < need:
                freed = self._evict_retained_encoder_caches()
                if freed > 0:
                    self.memory_guard.trigger_bulk_eviction_cleanup(freed, reason="encode_phase_capacity")
                if enc_bm.num_free_blocks < need:
                    break
            req = self.queue.pop(0)
            self._admit(req, batched=False)
            try:
                if hit:
                    entry = self._full_input_enc_cache[full_hash]
                    entry["last_access_time"] = time.perf_counter()
                    for blk in entry["block_table"]:
                        enc_bm.ref_counts[blk] += 1
                        enc_bm.total_lookups += 1
                        enc_bm.cache_hits += 1
                    req.encoder_block_table = list(entry["block_table"])
                    self.encoder_calls_skipped += 1
                    self.encode_time_saved_s += entry.get("encode_time", 0.0)
                    self._setup_request_after_encode(req, None, None, full_hash, 0.0, hit_entry=entry)
                else:
                    t0 = time.perf_counter()
                    with self.phase_timer.measure([req], "encoder_forward"), torch.no_grad():
                        hidden, kv = self._encode([req], mel_in)
                    enc_time = time.perf_counter() - t0
                    self.encoder_calls += 1
                    self._setup_request_after_encode(req, hidden, kv, full_hash, enc_time)
            except Exception as e:
                logger.error(f"Error in ENCODE_PHASE for req {req.id}: {e}", exc_info=True)
                self._complete_request(req, status=RequestPhase.FAILED)

    def _reserve_slot(self, req: DualCacheRequest) -> int:
        buf = self.graph_buffers
        slot = buf.reserve_slot()
        req.slot_idx = req.graph_slot_idx = slot
        req.graph_slot_reused = buf.slots[slot].reused
        return slot

    def _encode(self, reqs: List[DualCacheRequest], mels: torch.Tensor):
        """Encoder forward.  With direct handoff and a model whose projection can target
        the graph slots, each request's slot is reserved first and the cross K/V are
        written straight into it (no K/V list is returned then)."""
        if self.graph_direct_encoder_kv and getattr(self.model, "encodes_into_slots", False):
            slots = [self._reserve_slot(r) for r in reqs]
            buf = self.graph_buffers
            if hasattr(self.model, "encode_into_slots"):
                if not self.graph_encoder:
                    hidden = self.model.encode_into_slots(mels, buf.cross_kv_all, slots, buf.spare_slot, buf.buckets,
                                                          use_graphs=False)
                    return hidden, None
                # on the encoder stream, overlapping the decode graph of the requests in flight
                main = torch.cuda.current_stream(buf.device)
                if self._enc_stream is None:
                    self._enc_stream = torch.cuda.Stream(device=buf.device)
                es = self._enc_stream
                es.wait_stream(main)
                mels.record_stream(es)
                with torch.cuda.stream(es):
                    hidden = self.model.encode_into_slots(mels, buf.cross_kv_all, slots, buf.spare_slot, buf.buckets)
                ev = torch.cuda.Event()
                ev.record(es)
                for r in reqs:
                    r.enc_ready = ev
                return hidden, None
            ids = torch.tensor(slots, dtype=torch.int32).to(buf.device, non_blocking=True)
            return self.model.encode(mels, out_slots=buf.cross_kv, slot_ids=ids)
        return self.model.encode(mels)

    def _setup_safely(self, req, hidden, kv, full_hash, enc_time) -> None:
        try:
            self._setup_request_after_encode(req, hidden, kv, full_hash, enc_time)
        except Exception as e:
            logger.error(f"Error in ENCODE_PHASE for req {req.id}: {e}", exc_info=True)
            self._complete_request(req, status=RequestPhase.FAILED)

    # ---- handoff ------------------------------------------------------------------------------
    def _setup_request_after_encode(self, req: DualCacheRequest, encoder_hidden: Optional[torch.Tensor],
                                    encoder_kv_list, full_hash: Optional[str], enc_time: float,
                                    hit_entry: Optional[Dict[str, Any]] = None) -> None:
        enc_bm, dec_bm = self.dual_cache.encoder_bm, self.dual_cache.decoder_bm
        buf = self.graph_buffers
        slot = req.slot_idx if req.slot_idx is not None else self._reserve_slot(req)
        dev = buf.device
        if hit_entry is not None:
            enc_len = hit_entry["enc_seq_len"]
        else:
            enc_len = encoder_hidden.shape[1]
        req.encoder_seq_len = enc_len
        T = min(enc_len, buf.max_enc_len)
        L = min(len(encoder_kv_list) if encoder_kv_list is not None else enc_bm.num_layers, buf.num_decoder_layers)

        if self.graph_direct_encoder_kv:
            if encoder_kv_list is not None:  # else the encoder already wrote the slot
                with self.phase_timer.measure([req], "cross_kv_contiguous_or_graph_copy"):
                    buf.model.cross_kv_from_encoder(encoder_kv_list, buf.cross_kv, slot)
        else:
            if hit_entry is None:
                with self.phase_timer.measure([req], "block_allocate"):
                    for _ in range(self._blocks(enc_len, enc_bm.block_size)):
                        blk, _ = enc_bm.allocate_block(content_hash=None)
                        req.encoder_block_table.append(blk)
                with self.phase_timer.measure([req], "cross_kv_pool_copy"):
                    for l, (k, v) in enumerate(encoder_kv_list):  # op 3: encoder K/V into its blocks
                        enc_bm.store_sequence(req.encoder_block_table, l, k[:1], v[:1])
            with self.phase_timer.measure([req], "cross_kv_contiguous_or_graph_copy"):
                tab = torch.tensor([req.encoder_block_table], dtype=torch.int32).to(dev, non_blocking=True)
                lens = torch.tensor([T], dtype=torch.int32).to(dev, non_blocking=True)
                for l in range(L):  # op 5: blocks -> this request's cross-KV slot
                    ops.block_gather(enc_bm.key_pool[l], tab, lens, buf.max_enc_len, out=buf.cross_kv[slot:slot + 1, l, 0])
                    ops.block_gather(enc_bm.value_pool[l], tab, lens, buf.max_enc_len,
                                     out=buf.cross_kv[slot:slot + 1, l, 1])
            if self.retain_encoder_cache and full_hash and hit_entry is None:
                for blk in req.encoder_block_table:
                    enc_bm.ref_counts[blk] += 1
                while len(self._full_input_enc_cache) >= self.max_cached_encoder_inputs:
                    oldest = min(self._full_input_enc_cache, key=lambda h: self._full_input_enc_cache[h]["last_access_time"])
                    ev = self._full_input_enc_cache.pop(oldest)
                    if ev.get("held_by_cache", False):
                        enc_bm.release_blocks(ev["block_table"])
                self._full_input_enc_cache[full_hash] = {"block_table": list(req.encoder_block_table),
                                                         "enc_seq_len": enc_len, "last_access_time": time.perf_counter(),
                                                         "held_by_cache": True, "encode_time": enc_time}
        req.cached_encoder_kv = [(buf.cross_kv[slot:slot + 1, l, 0, :, :T], buf.cross_kv[slot:slot + 1, l, 1, :, :T])
                                 for l in range(buf.num_decoder_layers)]

        # decoder blocks: graph mode reserves prompt + max_new + one readback window
        req.encode_done_time = time.perf_counter()
        req.phase = RequestPhase.DECODE_PHASE
        P = req.prompt_token_ids.shape[1]
        req.decoder_seq_len = P
        total = P + req.max_new_tokens + (buf.readback_k if self.graph_decode else 0)
        n_blocks = self._blocks(total if self.graph_decode else P, dec_bm.block_size)
        with self.phase_timer.measure([req], "block_allocate"):
            for _ in range(n_blocks):
                req.decoder_block_table.append(self.dual_cache.allocate_decoder_block())

        if self.graph_fold_prefill and P <= MAX_FOLDED_PROMPT:
            # the decode graph prefills the prompt; the first token arrives with a readback
            prompt = req.prompt_token_ids[0].tolist()
            if req.enc_ready is not None:  # its encoder is still running on the encoder stream
                self._pending_activation.append((req, slot, P, T, prompt))
                return
            buf.assign_slot(req, None, P, None, slot_idx=slot, enc_seq_len=T, fold_prompt=prompt)
            self.active_decode.append(req)
            return
        if req.enc_ready is not None:  # the prefill below reads the slot's cross K/V
            torch.cuda.current_stream(buf.device).wait_event(req.enc_ready)
            req.enc_ready = None

        # prefill (multi-token), then its K/V into the decoder blocks (op 3, prompt form)
        with self.phase_timer.measure([req], "prefill"), torch.no_grad():
            out = self.model.decode_step(input_ids=req.prompt_token_ids, encoder_past_kv_list=req.cached_encoder_kv,
                                         use_cache=True)
            tab = torch.tensor([req.decoder_block_table], dtype=torch.int32).to(dev, non_blocking=True)
            zero = torch.zeros(1, dtype=torch.int32, device=dev)
            for l, lay in enumerate(out.past_key_values.layers):
                ops.kv_append(lay.keys.contiguous(), lay.values.contiguous(), dec_bm.key_pool[l], dec_bm.value_pool[l],
                              tab, zero)
            first = int(torch.argmax(out.logits[:, -1, :], dim=-1).item())
        req.last_token_id = first
        req.generated_tokens.append(first)
        req.generated_count = 1
        req.first_token_time = time.perf_counter()
        if (req.eos_token_id is not None and first == req.eos_token_id) or req.generated_count >= req.max_new_tokens:
            self._complete_request(req, status=RequestPhase.COMPLETED)
            return
        buf.assign_slot(req, None, P, first, slot_idx=slot, enc_seq_len=T)
        self.active_decode.append(req)

    # ---- decode phase --------------------------------------------------------------------------
    def _occupied(self) -> int:
        """Requests holding a slot: encoding, decoding, or handed off and waiting for
        their encoder."""
        return len(self.active_encode) + len(self.active_decode) + len(self._pending_activation)

    def _activate_pending(self) -> None:
        """Slots whose encoder has finished join the decode graph; with nothing else to
        decode, wait for the oldest one."""
        if not self._pending_activation:
            return
        buf = self.graph_buffers
        if not self.active_decode:
            self._pending_activation[0][0].enc_ready.synchronize()
        keep = []
        for req, slot, P, T, prompt in self._pending_activation:
            if req.enc_ready.query():
                req.enc_ready = None
                buf.assign_slot(req, None, P, None, slot_idx=slot, enc_seq_len=T, fold_prompt=prompt)
                self.active_decode.append(req)
            else:
                keep.append((req, slot, P, T, prompt))
        self._pending_activation = keep

    def _process_decode_phase(self) -> None:
        self._activate_pending()
        if not self.active_decode:
            return
        buf = self.graph_buffers
        dec_bm = self.dual_cache.decoder_bm
        if not self.graph_decode:
            # eager: a block is added when the next written position (decoder_seq_len, the
            # number of cached tokens) starts a new block (reference :780-783)
            for req in self.active_decode:
                if len(req.decoder_block_table) * dec_bm.block_size <= req.decoder_seq_len:
                    req.decoder_block_table.append(self.dual_cache.allocate_decoder_block())
                    buf.set_table(req.slot_idx, req.decoder_block_table)
        active = list(self.active_decode)
        t0 = time.perf_counter()
        try:
            with self.phase_timer.measure(active, "host_between_replays"):
                bucket = buf.prepare_replay()
            with self.phase_timer.measure(active, "graph_replay"):
                buf.replay_step(bucket)
            self.decode_steps += 1
            if not buf.should_readback():
                self.decode_time_s += time.perf_counter() - t0
                return
            with self.phase_timer.measure(active, "readback_wait"):
                results = buf.sync_tokens()
        except Exception as e:
            # One batched step serves every active request, so a failed step fails all of
            # them; each is released (slot, decoder and encoder blocks) as in the reference's
            # per-request handler (phase_aware_scheduler.py:1037-1039 there).
            logger.error(f"decode step failed for requests {[r.id for r in active]}: {e}")
            buf.reset_window()
            for req in active:
                if not req.done:
                    self._complete_request(req, status=RequestPhase.FAILED)
            self.active_decode = [r for r in self.active_decode if not r.done]
            return
        self.decode_time_s += time.perf_counter() - t0
        done = []
        for slot, toks in results:
            req = slot.req
            for off, (tok, trace) in enumerate(zip(toks, slot.last_readback_trace)):
                if req.done:
                    break
                req.graph_token_trace.append({"token_index": len(req.generated_tokens), "bucket": trace["bucket"],
                                              "readback_position": trace["readback_position"]})
                req.last_token_id = tok
                req.generated_tokens.append(tok)
                req.generated_count = len(req.generated_tokens)
                if req.first_token_time is None:
                    req.first_token_time = time.perf_counter()
                # graph mode counts the last token as cached (reference :753); eager mode
                # counts the tokens whose K/V are in the pool (reference :1022)
                req.decoder_seq_len = req.prompt_token_ids.shape[1] + req.generated_count - \
                    (0 if self.graph_decode else 1)
                is_eos = req.eos_token_id is not None and tok == req.eos_token_id
                if is_eos or req.generated_count >= req.max_new_tokens:
                    req.graph_extra_slot_steps = len(toks) - off - 1
                    if self.phase_timing:
                        self.phase_timer.ensure(req)["slot_hold_steps_after_eos"] = req.graph_extra_slot_steps
                    if is_eos and self.graph_decode and req.generated_count > 1:
                        # graph mode drops EOS and everything after it (reference :759-761); an
                        # EOS first token is kept, as when the prefill produced it (:696-700)
                        req.generated_tokens = req.generated_tokens[: req.generated_tokens.index(tok)]
                    self._complete_request(req, status=RequestPhase.COMPLETED)
                    done.append(req)
                    break
        if done:
            self.active_decode = [r for r in self.active_decode if r not in done]

    # ---- release -------------------------------------------------------------------------------
    def _complete_request(self, req: DualCacheRequest, status: RequestPhase) -> None:
        """Explicit release of every block and the slot (reference :1046-1081)."""
        req.phase, req.done, req.finish_time = status, True, time.perf_counter()
        try:
            with self.phase_timer.measure([req], "block_release"):
                if req.slot_idx is not None and self._buffers is not None:
                    self._buffers.release_slot(req.slot_idx)
                if req.decoder_block_table:
                    self.dual_cache.decoder_bm.free_blocks(req.decoder_block_table)
                    req.decoder_block_table = []
                if req.encoder_block_table:
                    self.dual_cache.encoder_bm.release_blocks(req.encoder_block_table)
                    entry = self._full_input_enc_cache.get(req.full_input_hash)
                    if not self.retain_encoder_cache and entry is not None and all(
                            self.dual_cache.encoder_bm.ref_counts[b] == 0 for b in entry["block_table"]):
                        self._full_input_enc_cache.pop(req.full_input_hash, None)
                    req.encoder_block_table = []
        finally:
            req.slot_idx = None
            req.cached_decoder_kv = None
            req.cached_encoder_kv = None
            if req in self.active_decode:
                self.active_decode.remove(req)
            self.completed.append(req)

    # ---- loop ----------------------------------------------------------------------------------
    def _update_peak_actually_used(self) -> None:
        """Peak pool bytes in use (reference :1083-1107).  Cross K/V live in the fixed slot
        buffer, so there are no per-request contiguous copies to add."""
        enc_bm, dec_bm = self.dual_cache.encoder_bm, self.dual_cache.decoder_bm
        used = enc_bm.allocated_block_count * enc_bm.bytes_per_block + dec_bm.allocated_block_count * \
            dec_bm._bytes_per_block()
        self.peak_pool_blocks_used_bytes = max(getattr(self, "peak_pool_blocks_used_bytes", 0), used)
        self.peak_actually_used_bytes = max(self.peak_actually_used_bytes, used)

    def step(self) -> bool:
        in_flight = self._occupied()
        self.peak_in_flight_requests = max(self.peak_in_flight_requests, in_flight)
        self.in_flight_history.append(in_flight)
        self._update_peak_actually_used()
        if self.verbose:
            self.memory_guard.log_telemetry(in_flight, len(self.queue), self.dual_cache.encoder_bm.get_stats(),
                                            self.dual_cache.decoder_bm.get_stats())
        self._process_encode_phase()
        self._update_peak_actually_used()
        self._process_decode_phase()
        self._update_peak_actually_used()
        if self.step_delay > 0:
            time.sleep(self.step_delay)
        return self.has_work()

    def has_work(self) -> bool:
        return bool(self.queue or self.active_encode or self.active_decode or self._pending_activation)

    def run_until_done(self, max_steps: int = 10000) -> List[DualCacheRequest]:
        steps = 0
        while self.step() and steps < max_steps:
            steps += 1
        return self.completed

    def reset_telemetry(self) -> None:
        self.encoder_calls = self.encoder_calls_skipped = 0
        self.encode_time_saved_s = 0.0
        self.rejected_requests_count = 0
        self.in_flight_history, self.queue_wait_times, self.completed = [], [], []
        self.peak_in_flight_requests = self.peak_actually_used_bytes = 0
        self.decode_steps, self.decode_time_s = 0, 0.0

    def get_concurrency_stats(self) -> Dict[str, Any]:
        enc_bm, dec_bm = self.dual_cache.encoder_bm, self.dual_cache.decoder_bm
        enc_blk, dec_blk = enc_bm.bytes_per_block, dec_bm._bytes_per_block()
        req_enc = self._blocks(1500, enc_bm.block_size)
        req_dec = self._blocks(150, dec_bm.block_size)
        q = self.queue_wait_times or [0.0]
        f = self.in_flight_history or [0]
        return {
            "encoder_pool_blocks": enc_bm.num_blocks, "encoder_pool_mb": enc_bm.num_blocks * enc_blk / 2 ** 20,
            "decoder_pool_blocks": dec_bm.num_blocks, "decoder_pool_mb": dec_bm.num_blocks * dec_blk / 2 ** 20,
            "total_pool_mb": (enc_bm.num_blocks * enc_blk + dec_bm.num_blocks * dec_blk) / 2 ** 20,
            "req_encoder_blocks": req_enc, "req_encoder_mb": req_enc * enc_blk / 2 ** 20,
            "req_decoder_blocks": req_dec, "req_decoder_mb": req_dec * dec_blk / 2 ** 20,
            "avg_in_flight_requests": float(np.mean(f)), "max_in_flight_requests": int(max(f)),
            "queue_wait_time_mean_s": float(np.mean(q)), "queue_wait_time_p50_s": float(np.percentile(q, 50)),
            "queue_wait_time_p95_s": float(np.percentile(q, 95)), "rejections_per_run": self.rejected_requests_count,
            "peak_actually_used_mb": self.peak_actually_used_bytes / 2 ** 20,
        }

    def get_encoder_telemetry(self) -> Dict[str, Any]:
        total = self.encoder_calls + self.encoder_calls_skipped
        return {"encoder_calls": self.encoder_calls, "encoder_calls_skipped": self.encoder_calls_skipped,
                "encode_time_saved_s": round(self.encode_time_saved_s, 4), "total_requests": total,
                "skip_rate_pct": round(self.encoder_calls_skipped / total * 100.0, 2) if total else 0.0,
                "full_input_cache_entries": len(self._full_input_enc_cache),
                "max_cached_encoder_inputs": self.max_cached_encoder_inputs}

    def flush_full_input_cache(self) -> int:
        n = len(self._full_input_enc_cache)
        for entry in self._full_input_enc_cache.values():
            if entry.get("held_by_cache", False):
                self.dual_cache.encoder_bm.release_blocks(entry["block_table"])
        self._full_input_enc_cache.clear()
        return n
