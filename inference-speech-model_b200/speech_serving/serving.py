"""Synthetic serving workloads and the serving loop for decoder tokens/s.

Workloads follow the reference's benchmark driver (scripts/evaluate_real_speech.py:560-660:
arrival-ordered submission, back-pressure when the queue holds 2x the batch, idle
sleeps until the next arrival; Poisson arrivals :774-779) with synthetic inputs in place
of the LibriSpeech audio: a log-mel of ``100 * seconds`` frames of N(0, 1) values,
zero-padded to 3000 frames, and a seeded output length per request (EOS disabled).

Configurations:
  whisper-small    d_model 768, 12 + 12 layers, 12 heads, 80 mels, vocab 51865, fp16
  whisper-large-v3 d_model 1280, 32 + 32 layers, 20 heads, 128 mels, vocab 51866, bf16
  whisper-tiny     d_model 384, 4 + 4 layers, 6 heads, 80 mels, vocab 51865
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Dict, List, Optional

import numpy as np
import torch

ARCHS = {
    "whisper-tiny": dict(d_model=384, encoder_layers=4, decoder_layers=4, encoder_attention_heads=6,
                         decoder_attention_heads=6, encoder_ffn_dim=1536, decoder_ffn_dim=1536, num_mel_bins=80,
                         vocab_size=51865),
    "whisper-small": dict(d_model=768, encoder_layers=12, decoder_layers=12, encoder_attention_heads=12,
                          decoder_attention_heads=12, encoder_ffn_dim=3072, decoder_ffn_dim=3072, num_mel_bins=80,
                          vocab_size=51865),
    "whisper-large-v3": dict(d_model=1280, encoder_layers=32, decoder_layers=32, encoder_attention_heads=20,
                             decoder_attention_heads=20, encoder_ffn_dim=5120, decoder_ffn_dim=5120,
                             num_mel_bins=128, vocab_size=51866),
}


def whisper_config(arch: str):
    from transformers import WhisperConfig

    v = ARCHS[arch]["vocab_size"]
    return WhisperConfig(**ARCHS[arch], max_source_positions=1500, max_target_positions=448, pad_token_id=v - 1,
                         bos_token_id=50257, eos_token_id=50257, decoder_start_token_id=50258)


@dataclass
class SyntheticRequest:
    mel: torch.Tensor  # [n_mels, 3000] (host)
    audio_s: float
    max_new_tokens: int
    arrival_time: float


def synthetic_requests(n: int, n_mels: int, seed: int, out_lo: int, out_hi: int, audio_lo: float = 2.0,
                       audio_hi: float = 30.0, rate: Optional[float] = None, frames: int = 3000,
                       pin: bool = True) -> List[SyntheticRequest]:
    """n requests: audio length U[audio_lo, audio_hi] s, output length U{out_lo..out_hi},
    burst arrivals (rate None) or Poisson at ``rate`` req/s (first arrival at 0)."""
    rs = np.random.RandomState(seed)
    secs = rs.uniform(audio_lo, audio_hi, size=n)
    outs = rs.randint(out_lo, out_hi + 1, size=n)
    if rate is None:
        arrivals = np.zeros(n)
    else:
        iv = rs.exponential(scale=1.0 / rate, size=n)
        arrivals = np.cumsum(iv) - iv[0]
    g = torch.Generator().manual_seed(seed)
    reqs = []
    for i in range(n):
        mel = torch.zeros(n_mels, frames)
        m = min(frames, int(round(100 * secs[i])))
        mel[:, :m] = torch.randn(n_mels, m, generator=g)
        reqs.append(SyntheticRequest(mel.pin_memory() if pin and torch.cuda.is_available() else mel, float(secs[i]),
                                     int(outs[i]), float(arrivals[i])))
    return reqs


def run_engine(scheduler: Any, requests: List[SyntheticRequest], prompt: List[int], eos_token_id: int = -1,
               queue_factor: int = 2) -> Dict[str, Any]:
    """Drives ``scheduler`` over ``requests`` in arrival order and returns throughput and
    latency figures.  Decoder tokens/s counts every generated token (the prefill token
    included, as ``max_new_tokens`` does) over the wall time of the whole run."""
    dev = scheduler.device
    prompt_t = torch.tensor([prompt], dtype=torch.long, device=dev)
    order = sorted(range(len(requests)), key=lambda i: requests[i].arrival_time)
    ids: Dict[int, int] = {}
    q = 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    d0 = scheduler.decode_time_s
    steps0 = scheduler.decode_steps
    while q < len(order) or scheduler.has_work():
        now = time.perf_counter() - t0
        while q < len(order) and requests[order[q]].arrival_time <= now and \
                len(scheduler.queue) < scheduler.max_batch_size * queue_factor:
            r = requests[order[q]]
            rid = scheduler.submit(r.mel.to(dev, non_blocking=True), prompt_token_ids=prompt_t,
                                   max_new_tokens=r.max_new_tokens, arrival_time=r.arrival_time,
                                   eos_token_id=eos_token_id, arrival_wall_time=t0 + r.arrival_time)
            if rid is None:
                break
            ids[rid] = order[q]
            q += 1
        if scheduler.has_work():
            scheduler.step()
        elif q < len(order):
            wait = requests[order[q]].arrival_time - (time.perf_counter() - t0)
            if wait > 0:
                time.sleep(min(wait, 0.005))
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    done = [r for r in scheduler.completed if r.id in ids]
    toks = sum(len(r.generated_tokens) for r in done)
    ttft = [r.first_token_time - (t0 + requests[ids[r.id]].arrival_time) for r in done]
    lat = [r.finish_time - (t0 + requests[ids[r.id]].arrival_time) for r in done]
    failed = sum(r.phase.value == "FAILED" for r in done)
    by_index = [None] * len(requests)
    for r in done:
        by_index[ids[r.id]] = list(r.generated_tokens)
    return {
        "requests": len(done), "failed": failed, "generated_tokens": toks, "wall_s": round(wall, 4),
        "decoder_tok_s": round(toks / wall, 1),
        "decode_phase_s": round(scheduler.decode_time_s - d0, 4),
        "decode_steps": scheduler.decode_steps - steps0,
        "ttft_p50_s": round(float(np.percentile(ttft, 50)), 4) if ttft else None,
        "latency_p50_s": round(float(np.percentile(lat, 50)), 4) if lat else None,
        "latency_p95_s": round(float(np.percentile(lat, 95)), 4) if lat else None,
        "audio_s": round(sum(requests[ids[r.id]].audio_s for r in done), 2),
        "tokens_by_request": by_index,
    }
