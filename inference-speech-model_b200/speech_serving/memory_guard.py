"""Pool-occupancy policy used by the scheduler's admission control.

The scheduler asks one question of it — would the pools pass ``high_water_mark_pct`` —
and reports two kinds of events to it: bulk evictions (after which cached allocator
blocks are handed back to the driver, when ``enable_periodic_gc``) and, in verbose mode,
a periodic occupancy line.  Constructor arguments and the counters read by callers
(``eviction_events_count``, ``total_freed_blocks_count``, ``last_empty_cache_time``)
keep the reference's names (speech_serving/memory_guard.py:20-99).
"""
from __future__ import annotations

import logging
import time
from typing import Any, Dict

import torch

log = logging.getLogger(__name__)


def _occupancy(used: int, total: int) -> float:
    return 100.0 * used / total if total else 0.0


class MemoryGuard:
    def __init__(self, high_water_mark_pct: float = 90.0, enable_periodic_gc: bool = True):
        self.high_water_mark_pct = float(high_water_mark_pct)
        self.enable_periodic_gc = bool(enable_periodic_gc)
        self.eviction_events_count = 0
        self.total_freed_blocks_count = 0
        self.last_empty_cache_time = time.perf_counter()

    def check_high_water_mark(self, encoder_allocated: int, encoder_total: int, decoder_allocated: int,
                              decoder_total: int) -> bool:
        """True when both pools together are at or above the mark."""
        pct = _occupancy(encoder_allocated + decoder_allocated, encoder_total + decoder_total)
        over = encoder_total + decoder_total > 0 and pct >= self.high_water_mark_pct
        if over:
            log.warning("pools at %.1f%% of their blocks (mark %.1f%%)", pct, self.high_water_mark_pct)
        return over

    def trigger_bulk_eviction_cleanup(self, freed_blocks: int, reason: str = "high_water_mark") -> None:
        """Counts an eviction of ``freed_blocks`` blocks and trims the caching allocator."""
        self.eviction_events_count += 1
        self.total_freed_blocks_count += int(freed_blocks)
        log.info("eviction %d (%s): %d blocks back in the free lists", self.eviction_events_count, reason,
                 freed_blocks)
        if self.enable_periodic_gc and torch.cuda.is_available():
            torch.cuda.empty_cache()
            self.last_empty_cache_time = time.perf_counter()

    def log_telemetry(self, active_requests: int, queued_requests: int, encoder_stats: Dict[str, Any],
                      decoder_stats: Dict[str, Any]) -> None:
        """One occupancy line: requests in flight and waiting, and both pools' fill."""
        def fill(s: Dict[str, Any]) -> str:
            return f"{s['allocated_blocks']}/{s['num_blocks']} ({s['utilization_pct']}%)"

        log.info("in flight %d, waiting %d; encoder pool %s, decoder pool %s, evictions so far %d",
                 active_requests, queued_requests, fill(encoder_stats), fill(decoder_stats),
                 self.eviction_events_count)
