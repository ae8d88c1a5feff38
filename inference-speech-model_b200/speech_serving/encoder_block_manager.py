"""Encoder paged pool with reference counts and prefix (content-hash) sharing.

Same interface and semantics as the reference's EncoderBlockManager
(speech_serving/encoder_block_manager.py:17-221): FIFO allocation (``pop(0)`` at :135,
here an O(1) deque), ref-counted release that frees a block when its count reaches 0
(:144-164), prefix-hash hits that bump the count (:119-127), hit-rate telemetry.

``store_encoder_kv`` writes a block's rows with the paged K/V write kernel (op 3,
replacing :177-192); ``store_sequence`` writes a whole request's encoder K/V into its
block table in one launch per layer.  Storage: one HBM allocation
``[num_layers, 2, num_blocks, block_size, H, D]`` with per-layer views.
"""
from __future__ import annotations

import hashlib
from collections import deque
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from . import ops


class EncoderBlockManager:
    def __init__(
        self,
        num_layers: int,
        num_heads: int,
        head_dim: int,
        block_size: int = 16,
        num_blocks: Optional[int] = None,
        gpu_memory_utilization: float = 0.85,
        dtype: torch.dtype = torch.float16,
        device: str = "cuda",
    ):
        if isinstance(dtype, str):
            dtype = getattr(torch, dtype)
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.dtype = dtype
        self.device = device
        self.gpu_memory_utilization = gpu_memory_utilization
        self.bytes_per_token = num_layers * 2 * num_heads * head_dim * torch.tensor([], dtype=dtype).element_size()
        self.bytes_per_block = self.bytes_per_token * block_size
        if num_blocks is None:
            self.num_blocks, self.available_kv_memory_bytes = self._calculate_available_blocks()
        else:
            self.num_blocks = num_blocks
            self.available_kv_memory_bytes = num_blocks * self.bytes_per_block
        self.pool = torch.zeros((num_layers, 2, self.num_blocks, block_size, num_heads, head_dim), dtype=dtype,
                                device=device)
        self.key_pool: List[torch.Tensor] = [self.pool[l, 0] for l in range(num_layers)]
        self.value_pool: List[torch.Tensor] = [self.pool[l, 1] for l in range(num_layers)]
        self.free_block_list: deque = deque(range(self.num_blocks))
        self.ref_counts: Dict[int, int] = {i: 0 for i in range(self.num_blocks)}
        self.prefix_hash_table: Dict[str, int] = {}
        self.block_to_hash: Dict[int, str] = {}
        self.retained_caches: Dict[str, List[int]] = {}
        self.total_lookups = 0
        self.cache_hits = 0

    def _calculate_available_blocks(self) -> Tuple[int, int]:
        if not torch.cuda.is_available() or str(self.device) == "cpu":
            return 512, 512 * self.bytes_per_block
        free, total = torch.cuda.mem_get_info(torch.device(self.device))
        avail = max(0, int(total * self.gpu_memory_utilization) - (total - free))
        return max(64, avail // self.bytes_per_block), avail

    @staticmethod
    def _hash_audio_block(audio_features_slice: torch.Tensor) -> str:
        return hashlib.md5(audio_features_slice.detach().cpu().numpy().tobytes()).hexdigest()

    def allocate_block(self, content_hash: Optional[str] = None) -> Tuple[int, bool]:
        self.total_lookups += 1
        if content_hash is not None and content_hash in self.prefix_hash_table:
            blk = self.prefix_hash_table[content_hash]
            if self.ref_counts[blk] > 0:
                self.ref_counts[blk] += 1
                self.cache_hits += 1
                return blk, True
            del self.prefix_hash_table[content_hash]
        if not self.free_block_list:
            raise RuntimeError(
                f"Out of Encoder KV-cache blocks! All {self.num_blocks} blocks are allocated or referenced.")
        blk = self.free_block_list.popleft()
        self.ref_counts[blk] = 1
        if content_hash is not None:
            self.prefix_hash_table[content_hash] = blk
            self.block_to_hash[blk] = content_hash
        return blk, False

    def release_block(self, blk_id: int) -> bool:
        if self.ref_counts.get(blk_id, 0) <= 0:
            return False
        self.ref_counts[blk_id] -= 1
        if self.ref_counts[blk_id] == 0:
            h = self.block_to_hash.pop(blk_id, None)
            if h is not None:
                self.prefix_hash_table.pop(h, None)
            self.free_block_list.append(blk_id)
            return True
        return False

    def release_blocks(self, block_ids: Sequence[int]) -> int:
        return sum(1 for b in block_ids if self.release_block(b))

    def store_encoder_kv(self, block_id: int, layer_idx: int, k_tensor: torch.Tensor, v_tensor: torch.Tensor) -> None:
        """Writes [tok_count, H, D] rows into block ``block_id`` of layer ``layer_idx``."""
        tab = torch.tensor([[block_id]], dtype=torch.int32, device=self.pool.device)
        pos = torch.zeros(1, dtype=torch.int32, device=self.pool.device)
        src_k = k_tensor.permute(1, 0, 2).unsqueeze(0)  # [1, H, T, D] view
        src_v = v_tensor.permute(1, 0, 2).unsqueeze(0)
        ops.kv_append(src_k, src_v, self.key_pool[layer_idx], self.value_pool[layer_idx], tab, pos)

    def store_sequence(self, block_table: Sequence[int], layer_idx: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Writes a request's encoder K/V [1 or -, H, T, D] into its blocks (one launch)."""
        tab = torch.tensor([list(block_table)], dtype=torch.int32).to(self.pool.device, non_blocking=True)
        pos = torch.zeros(1, dtype=torch.int32, device=self.pool.device)
        if k.dim() == 3:
            k, v = k.unsqueeze(0), v.unsqueeze(0)
        ops.kv_append(k, v, self.key_pool[layer_idx], self.value_pool[layer_idx], tab, pos)

    @property
    def allocated_block_count(self) -> int:
        return self.num_blocks - len(self.free_block_list)

    @property
    def num_free_blocks(self) -> int:
        return len(self.free_block_list)

    @property
    def hit_rate(self) -> float:
        return 0.0 if self.total_lookups == 0 else round(self.cache_hits / self.total_lookups * 100, 2)

    def get_stats(self) -> Dict[str, Any]:
        allocated = self.allocated_block_count
        return {
            "num_blocks": self.num_blocks,
            "block_size": self.block_size,
            "allocated_blocks": allocated,
            "free_blocks": len(self.free_block_list),
            "utilization_pct": round(allocated / self.num_blocks * 100, 2) if self.num_blocks else 0.0,
            "total_lookups": self.total_lookups,
            "cache_hits": self.cache_hits,
            "prefix_hit_rate_pct": self.hit_rate,
            "pool_memory_mb": round(self.num_blocks * self.bytes_per_block / 1024 ** 2, 2),
        }
