"""High-water-mark check and post-eviction cache maintenance (the reference's
speech_serving/memory_guard.py:20-99, same thresholds and telemetry fields)."""
from __future__ import annotations

import logging
import time
from typing import Any, Dict

import torch

logger = logging.getLogger("SpeechMemoryGuard")


class MemoryGuard:
    def __init__(self, high_water_mark_pct: float = 90.0, enable_periodic_gc: bool = True):
        self.high_water_mark_pct = high_water_mark_pct
        self.enable_periodic_gc = enable_periodic_gc
        self.eviction_events_count = 0
        self.last_empty_cache_time = time.perf_counter()
        self.total_freed_blocks_count = 0

    def check_high_water_mark(self, encoder_allocated: int, encoder_total: int, decoder_allocated: int,
                              decoder_total: int) -> bool:
        total = encoder_total + decoder_total
        if total == 0:
            return False
        pct = (encoder_allocated + decoder_allocated) / total * 100.0
        if pct >= self.high_water_mark_pct:
            logger.warning(f"[HIGH WATER MARK EXCEEDED] Utilization={pct:.1f}%")
            return True
        return False

    def trigger_bulk_eviction_cleanup(self, freed_blocks: int, reason: str = "high_water_mark") -> None:
        self.eviction_events_count += 1
        self.total_freed_blocks_count += freed_blocks
        logger.info(f"[BULK EVICTION EVENT #{self.eviction_events_count}] reason={reason} freed={freed_blocks}")
        if self.enable_periodic_gc and torch.cuda.is_available():
            torch.cuda.empty_cache()
            self.last_empty_cache_time = time.perf_counter()

    def log_telemetry(self, active_requests: int, queued_requests: int, encoder_stats: Dict[str, Any],
                      decoder_stats: Dict[str, Any]) -> None:
        logger.info(
            f"[TELEMETRY] ActiveReqs={active_requests} QueuedReqs={queued_requests} | "
            f"EncUtil={encoder_stats['utilization_pct']}% ({encoder_stats['allocated_blocks']}/"
            f"{encoder_stats['num_blocks']} blks) | DecUtil={decoder_stats['utilization_pct']}% "
            f"({decoder_stats['allocated_blocks']}/{decoder_stats['num_blocks']} blks) | "
            f"Evictions={self.eviction_events_count}")
