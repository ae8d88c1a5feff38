"""Opt-in per-request phase accounting for the scheduler.

The phase names and the per-request record (``{"phases": {name: {"wall_ms", "cuda_ms",
"calls"}}, ...}``) are the telemetry interface the reference's tooling reads
(speech_serving/phase_timing.py:10-94 defines them there).  The mechanism here is
different: a measured span never synchronises the device.  Each span pushes an NVTX
range (so a profiler timeline shows the phases) and records a CUDA event pair on the
current stream; the host wall time is booked at once, the device time later, when the
span's end event has completed (``collect``, called from ``ensure`` and ``finish``).  A
span whose events have not completed by ``finish`` is booked with its wall time only and
counted under ``"cuda_pending"``.

Disabled (the default), every call is a no-op.
"""
from __future__ import annotations

import time
from collections import deque
from contextlib import contextmanager
from typing import Any, Deque, Dict, Iterable, List, Tuple

import torch

PHASES = ("queue_admission_wait", "encoder_forward", "cross_kv_pool_copy", "cross_kv_contiguous_or_graph_copy",
          "prefill", "graph_replay", "host_between_replays", "readback_wait", "block_allocate", "block_release",
          "other_host_between_requests")

_NOTE = ("per-request totals; a span that serves a whole batch is booked in full on every request of the batch; "
         "cuda_ms is the device time between events recorded around the span on the current stream")


def new_phase_record() -> Dict[str, Any]:
    return {"phases": {}, "encoder_batched": None, "slot_hold_steps_after_eos": 0, "semantics": _NOTE}


def _record_of(target: Any) -> Dict[str, Any]:
    if isinstance(target, dict):
        return target if "phases" in target else target.setdefault("phase_timing", new_phase_record())
    rec = getattr(target, "phase_timing", None)
    if rec is None:
        rec = new_phase_record()
        target.phase_timing = rec
    return rec


def _slot(rec: Dict[str, Any], phase: str) -> Dict[str, Any]:
    return rec["phases"].setdefault(phase, {"wall_ms": 0.0, "cuda_ms": 0.0, "calls": 0})


class PhaseTimer:
    """Books named spans onto request records without synchronising the GPU."""

    def __init__(self, enabled: bool, device: str = "cuda"):
        self.enabled = bool(enabled)
        self.device = device
        self.cuda_enabled = self.enabled and torch.cuda.is_available() and str(device).startswith("cuda")
        # spans whose device time is not booked yet: (start, end, phase, records)
        self._open: Deque[Tuple[Any, Any, str, List[Dict[str, Any]]]] = deque()

    def ensure(self, target: Any) -> Dict[str, Any]:
        """The record of ``target`` (a request or a dict), created on first use."""
        self.collect()
        return _record_of(target)

    def add(self, targets: Iterable[Any], phase: str, wall_ms: float, cuda_ms: float, calls: int = 1) -> None:
        if not self.enabled:
            return
        for t in targets:
            s = _slot(_record_of(t), phase)
            s["wall_ms"] += float(wall_ms)
            s["cuda_ms"] += float(cuda_ms)
            s["calls"] += int(calls)

    def collect(self) -> None:
        """Books the device time of every finished span, oldest first (spans on one stream
        finish in order, so the first unfinished one ends the scan)."""
        while self._open and self._open[0][1].query():
            start, end, phase, recs = self._open.popleft()
            ms = start.elapsed_time(end)
            for r in recs:
                _slot(r, phase)["cuda_ms"] += ms

    def finish(self, target: Any) -> Dict[str, Any]:
        """Books what has completed and returns the record; spans of ``target`` that are
        still running on the device are counted under ``cuda_pending``."""
        self.collect()
        rec = _record_of(target)
        pending = sum(1 for *_, recs in self._open if any(r is rec for r in recs))
        if pending:
            rec["cuda_pending"] = pending
        return rec

    @contextmanager
    def measure(self, targets: Iterable[Any], phase: str):
        if not self.enabled:
            yield
            return
        recs = [_record_of(t) for t in targets]
        start = end = None
        if self.cuda_enabled:
            torch.cuda.nvtx.range_push(phase)
            start = torch.cuda.Event(enable_timing=True)
            start.record()
        t0 = time.perf_counter()
        try:
            yield
        finally:
            wall = (time.perf_counter() - t0) * 1000.0
            for r in recs:
                s = _slot(r, phase)
                s["wall_ms"] += wall
                s["calls"] += 1
            if self.cuda_enabled:
                end = torch.cuda.Event(enable_timing=True)
                end.record()
                torch.cuda.nvtx.range_pop()
                self._open.append((start, end, phase, recs))
                self.collect()


def finalize_phases(record: Dict[str, Any], measured_phases=PHASES) -> Dict[str, Any]:
    """Marks the phases a record never saw, so every record lists every phase."""
    phases = record.setdefault("phases", {})
    for p in measured_phases:
        phases.setdefault(p, "not measured")
    return record
