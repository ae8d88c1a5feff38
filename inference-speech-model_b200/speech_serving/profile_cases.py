"""Runs one named kernel workload a few times with plain launches, for profilers.

    python -m speech_serving.profile_cases paged_cfg2 --launches 3
    python -m speech_serving.profile_cases cross_cfg3 --launches 3
    python -m speech_serving.profile_cases cross_dec --launches 3
    python -m speech_serving.profile_cases proj_small --launches 3
    python -m speech_serving.profile_cases cross_cfg3 --time 50   # CUDA-event timing

Cases: paged_cfg2 = paged self-attention B=64 H=12 D=64 bs=16
ctx~U[1,448] fp16 (paged_big: the same with B=512 and every context 448, a launch long
enough that set-up and tail are small); cross_cfg3 = cross-attention B=128 H=20 D=64 T=1500 valid~U[300,1500]
bf16; proj_small / proj_large = the handoff cross-KV projection of one 1500-position
request for Whisper-small (d 768, 12 layers x 12 heads) / large-v3 (d 1280, 32 x 20), bf16.
Each launch reads a different input set so that DRAM counters see cold data.
"""
from __future__ import annotations

import argparse

import torch

from . import ops


WORK = {}  # case -> (algorithmic bytes or flops per launch, unit)


def _paged(dev, sets, B=64, NB=4096, lo=1, name="paged_cfg2"):
    g = torch.Generator().manual_seed(0)
    H, D, bs = 12, 64, 16
    out = []
    for i in range(sets):
        ctx = torch.randint(lo, 449, (B,), generator=g, dtype=torch.int32)
        tables = torch.randperm(NB, generator=g)[: B * 28].view(B, 28).to(torch.int32)
        q = torch.randn(B, H, D, device=dev).half()
        kp = torch.randn(NB, bs, H, D, device=dev).half()
        vp = torch.randn(NB, bs, H, D, device=dev).half()
        out.append((q, kp, vp, tables.to(dev), ctx.to(dev)))
    ws = ops.paged_attn_workspace(B, H, D, 28, dev)
    WORK[name] = (sum(int(o[4].sum()) * H * D * 4 + 2 * B * H * D * 2 for o in out) / sets, "GB/s")
    return lambda i: ops.paged_decode_attention(*out[i % sets], scale=0.125, workspace=ws)


def _cross(dev, sets):
    g = torch.Generator().manual_seed(0)
    B, H, T, D = 128, 20, 1500, 64
    out = []
    for i in range(sets):
        valid = torch.randint(300, 1501, (B,), generator=g, dtype=torch.int32)
        out.append((torch.randn(B, H, D, device=dev).bfloat16(), torch.randn(B, H, T, D, device=dev).bfloat16(),
                    torch.randn(B, H, T, D, device=dev).bfloat16(), valid.to(dev)))
    ws = ops.cross_attn_workspace(B, H, D, dev)
    WORK["cross_cfg3"] = (sum(int(o[3].sum()) * H * D * 4 + 2 * B * H * D * 2 for o in out) / sets, "GB/s")
    return lambda i: ops.cross_attention(*out[i % sets], scale=0.125, workspace=ws)


def _cross_decode(dev, sets):
    """Cross-attention as one layer of a batch-64 Whisper-small decode step reads it: fp16,
    H=12, the graph-slot layout [slot, layer, k|v, H, 1500, D] (two layers), valid encoder
    lengths U[100, 1500] (2-30 s of audio)."""
    g = torch.Generator().manual_seed(0)
    B, L, H, T, D = 64, 2, 12, 1500, 64
    slots = torch.randn(B, L, 2, H, T, D, device=dev).half()
    out = []
    for i in range(sets):
        valid = torch.randint(100, 1501, (B,), generator=g, dtype=torch.int32)
        out.append((torch.randn(B, H, D, device=dev).half(), slots[:, i % L, 0], slots[:, i % L, 1], valid.to(dev)))
    ws = ops.cross_attn_workspace(B, H, D, dev)
    WORK["cross_dec"] = (sum(int(o[3].sum()) * H * D * 4 + 2 * B * H * D * 2 for o in out) / sets, "GB/s")
    return lambda i: ops.cross_attention(*out[i % sets], scale=0.125, workspace=ws)


def _proj(dev, sets, d, L, H):
    D, T = 64, 1500
    enc = [torch.randn(1, T, d, device=dev).bfloat16() for _ in range(sets)]
    w = (torch.randn(L * 2 * H * D, d, device=dev) * 0.02).bfloat16()
    b = torch.zeros(L * 2 * H * D, device=dev).bfloat16()
    out = torch.empty((1, L, 2, H, T, D), device=dev, dtype=torch.bfloat16)
    WORK[f"proj_{d}"] = (2.0 * T * d * L * 2 * H * D, "TFLOP/s")
    return lambda i: ops.cross_kv_project(enc[i % sets], w, b, out)


CASES = {
    "paged_cfg2": lambda dev, n: _paged(dev, n),
    "paged_big": lambda dev, n: _paged(dev, n, B=512, NB=16384, lo=448, name="paged_big"),
    "cross_cfg3": lambda dev, n: _cross(dev, n),
    "cross_dec": lambda dev, n: _cross_decode(dev, n),
    "proj_small": lambda dev, n: _proj(dev, n, 768, 12, 12),
    "proj_large": lambda dev, n: _proj(dev, n, 1280, 32, 20),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--sets", type=int, default=2)
    ap.add_argument("--time", type=int, default=0, help="time this many launches with CUDA events")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    run = CASES[a.case](dev, a.sets)
    for i in range(a.launches):
        run(i)
    torch.cuda.synchronize()
    print(f"{a.case}: {a.launches} launches ok")
    if a.time:
        for i in range(3):
            run(i)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        for i in range(a.time):
            run(i)
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1000.0 / a.time
        key = a.case if a.case in WORK else [k for k in WORK if k.startswith("proj")][0]
        work, unit = WORK[key]
        rate = work / (us * 1e-6) / (1e9 if unit == "GB/s" else 1e12)
        print(f"{a.case}: {us:.2f} us per launch (plain stream launches), {rate:.1f} {unit}")


if __name__ == "__main__":
    main()
