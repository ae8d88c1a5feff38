"""Default-off per-phase timing (the reference's speech_serving/phase_timing.py:10-94):
wall time and CUDA-event time per named phase, recorded per request."""
from __future__ import annotations

import time
from contextlib import contextmanager
from typing import Any, Dict, Iterable

import torch

PHASES = ("queue_admission_wait", "encoder_forward", "cross_kv_pool_copy", "cross_kv_contiguous_or_graph_copy",
          "prefill", "graph_replay", "host_between_replays", "readback_wait", "block_allocate", "block_release",
          "other_host_between_requests")


def new_phase_record() -> Dict[str, Any]:
    return {"phases": {}, "encoder_batched": None, "slot_hold_steps_after_eos": 0,
            "semantics": "request-experienced elapsed time; shared batch work is recorded for every participating "
                         "request"}


class PhaseTimer:
    def __init__(self, enabled: bool, device: str = "cuda"):
        self.enabled = bool(enabled)
        self.device = device
        self.cuda_enabled = self.enabled and torch.cuda.is_available() and str(device).startswith("cuda")

    @staticmethod
    def ensure(target: Any) -> Dict[str, Any]:
        if isinstance(target, dict):
            return target if "phases" in target else target.setdefault("phase_timing", new_phase_record())
        if getattr(target, "phase_timing", None) is None:
            target.phase_timing = new_phase_record()
        return target.phase_timing

    def add(self, targets: Iterable[Any], phase: str, wall_ms: float, cuda_ms: float, calls: int = 1) -> None:
        if not self.enabled:
            return
        for t in targets:
            item = self.ensure(t)["phases"].setdefault(phase, {"wall_ms": 0.0, "cuda_ms": 0.0, "calls": 0})
            item["wall_ms"] += float(wall_ms)
            item["cuda_ms"] += float(cuda_ms)
            item["calls"] += int(calls)

    @contextmanager
    def measure(self, targets: Iterable[Any], phase: str):
        targets = list(targets)
        if not self.enabled:
            yield
            return
        if self.cuda_enabled:
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
        t0 = time.perf_counter()
        try:
            yield
        finally:
            cuda_ms = 0.0
            if self.cuda_enabled:
                e.record()
                torch.cuda.synchronize()
                cuda_ms = s.elapsed_time(e)
            self.add(targets, phase, (time.perf_counter() - t0) * 1000.0, cuda_ms)


def finalize_phases(record: Dict[str, Any], measured_phases=PHASES) -> Dict[str, Any]:
    phases = record.setdefault("phases", {})
    for p in measured_phases:
        phases.setdefault(p, "not measured")
    return record
