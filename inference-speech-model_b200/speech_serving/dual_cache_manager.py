"""Couples the encoder and decoder pools of a request (same interface as the reference's
speech_serving/dual_cache_manager.py:17-90): encoder allocation rolls back partial
allocations on failure (:46-55) and release is deterministic (:63-83)."""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

from .block_manager import BlockManager
from .encoder_block_manager import EncoderBlockManager


class DualCacheManager:
    def __init__(self, encoder_block_manager: EncoderBlockManager, decoder_block_manager: BlockManager):
        self.encoder_bm = encoder_block_manager
        self.decoder_bm = decoder_block_manager

    def allocate_encoder_blocks(self, seq_len: int,
                                content_hashes: Optional[List[Optional[str]]] = None) -> Tuple[List[int], int]:
        bs = self.encoder_bm.block_size
        table: List[int] = []
        hits = 0
        try:
            for i in range((seq_len + bs - 1) // bs):
                ch = content_hashes[i] if content_hashes is not None and i < len(content_hashes) else None
                blk, hit = self.encoder_bm.allocate_block(content_hash=ch)
                table.append(blk)
                hits += int(hit)
        except Exception:
            self.encoder_bm.release_blocks(table)
            raise
        return table, hits

    def allocate_decoder_block(self) -> int:
        return self.decoder_bm.allocate_block()

    def release_request_resources(self, encoder_block_table: List[int],
                                  decoder_block_table: List[int]) -> Dict[str, int]:
        freed_enc = self.encoder_bm.release_blocks(encoder_block_table)
        n_dec = len(decoder_block_table)
        self.decoder_bm.free_blocks(decoder_block_table)
        return {"freed_encoder_blocks": freed_enc, "freed_decoder_blocks": n_dec}

    def get_stats(self) -> Dict[str, Any]:
        return {"encoder": self.encoder_bm.get_stats(), "decoder": self.decoder_bm.get_stats()}
