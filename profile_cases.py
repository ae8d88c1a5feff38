"""Named kernel workloads for profilers and timelines (measurement tooling beside bench.py).

    python profile_cases.py paged_cfg2 --launches 3            # plain launches (for ncu)
    python profile_cases.py paged_cfg2 --graph 200             # CUDA-graph timing, as bench.py
    python profile_cases.py paged_cfg2 --graph 32 --trace      # %globaltimer timeline of a launch
    python profile_cases.py cross_cfg3 --time 50               # plain-launch CUDA-event timing
    python profile_cases.py decode_small --launches 3          # batch-64 Whisper-small decode step

Cases:
  paged_cfg2    paged self-attention: fp16 B=64 H=12 D=64 bs=16
                ctx ~ U[1,448], block tables from a permutation of a 4096-block pool
  paged_big     the same with B=512 and every context 448 (set-up and tail are small)
  cross_cfg3    cross-attention: bf16 B=128 H=20 D=64 T=1500 valid ~ U[300,1500]
  cross_dec     cross-attention as one layer of a batch-64 Whisper-small decode step
  proj_small    the handoff cross-KV projection of one 1500-position request, Whisper-small
  proj_large    the same for Whisper-large-v3
  decode_small  one decode step of random-init Whisper-small (fp16) over 64 graph slots
                with the full 1500-position cross contexts (what serving attends) and
                100-token self contexts, replayed
                from its CUDA graph; launches run inside an NVTX range named "steps"
  decode_large  the same for random-init Whisper-large-v3 (bf16)
  linear_table  the decode step's Linear shapes at batch 64, tcgen05 kernel vs cuBLAS with the full
                1500-position cross contexts the serving configuration attends

Each launch reads a different input set (``--sets``) so that DRAM counters see cold data.
``--trace`` loads the trace build of the library (inference-speech-model_b200/csrc/build.py
--trace; built here when missing) and prints, for the last launch of the graph, when each
CTA reached each marked point, relative to the first CTA's entry.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "inference-speech-model_b200"
sys.path[:0] = [str(REPO), str(PKG)]

WORK = {}  # case -> (algorithmic bytes or flops per launch, unit)


def _paged(torch, ops, dev, sets, B=64, NB=4096, lo=1, name="paged_cfg2"):
    g = torch.Generator().manual_seed(0)
    H, D, bs = 12, 64, 16
    out = []
    for i in range(sets):
        ctx = torch.randint(lo, 449, (B,), generator=g, dtype=torch.int32)
        tables = torch.randperm(NB, generator=g)[: B * 28].view(B, 28).to(torch.int32)
        q = torch.randn(B, H, D, device=dev).half()
        kp = torch.randn(NB, bs, H, D, device=dev).half()
        vp = torch.randn(NB, bs, H, D, device=dev).half()
        out.append((q, kp, vp, tables.to(dev), ctx.to(dev), torch.empty(B, H, D, device=dev, dtype=torch.half)))
    ws = ops.paged_attn_workspace(B, H, D, 28, dev)
    per = [int(o[4].sum()) * H * D * 4 + 2 * B * H * D * 2 for o in out]
    WORK[name] = (sum(per) / sets, "GB/s", per)

    def run(i):
        q, kp, vp, t, c, o = out[i % sets]
        ops.paged_decode_attention(q, kp, vp, t, c, scale=0.125, out=o, workspace=ws)
    return run


def _cross(torch, ops, dev, sets):
    g = torch.Generator().manual_seed(0)
    B, H, T, D = 128, 20, 1500, 64
    out = []
    for i in range(sets):
        valid = torch.randint(300, 1501, (B,), generator=g, dtype=torch.int32)
        out.append((torch.randn(B, H, D, device=dev).bfloat16(), torch.randn(B, H, T, D, device=dev).bfloat16(),
                    torch.randn(B, H, T, D, device=dev).bfloat16(), valid.to(dev)))
    ws = ops.cross_attn_workspace(B, H, D, dev)
    per = [int(o[3].sum()) * H * D * 4 + 2 * B * H * D * 2 for o in out]
    WORK["cross_cfg3"] = (sum(per) / sets, "GB/s", per)
    return lambda i: ops.cross_attention(*out[i % sets], scale=0.125, workspace=ws)


def _cross_decode(torch, ops, dev, sets):
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
    per = [int(o[3].sum()) * H * D * 4 + 2 * B * H * D * 2 for o in out]
    WORK["cross_dec"] = (sum(per) / sets, "GB/s", per)
    return lambda i: ops.cross_attention(*out[i % sets], scale=0.125, workspace=ws)


def _proj(torch, ops, dev, sets, d, L, H, name):
    D, T = 64, 1500
    enc = [torch.randn(1, T, d, device=dev).bfloat16() for _ in range(sets)]
    w = (torch.randn(L * 2 * H * D, d, device=dev) * 0.02).bfloat16()
    b = torch.zeros(L * 2 * H * D, device=dev).bfloat16()
    out = torch.empty((1, L, 2, H, T, D), device=dev, dtype=torch.bfloat16)
    WORK[name] = (2.0 * T * d * L * 2 * H * D, "TFLOP/s", None)
    return lambda i: ops.cross_kv_project(enc[i % sets], w, b, out)


def _decode_small(torch, ops, dev, sets, B=64, cross_len=1500, self_len=100, arch="whisper-small",
                  dtype_name="float16", name="decode_small"):
    """One batch-64 decode step of a random-init Whisper model replayed from its graph."""
    from speech_serving.block_manager import BlockManager
    from speech_serving.graph_decode_buffers import PagedDecodeState
    from speech_serving.models import PretrainedWhisperModel
    from speech_serving.serving import whisper_config

    dt = getattr(torch, dtype_name)
    model = PretrainedWhisperModel(config=whisper_config(arch), device=str(dev), dtype=dt, seed=0)
    L, H, D = model.num_decoder_layers, model.num_heads, model.head_dim
    nblk = -(-(self_len + 8) // 16)
    bm = BlockManager(L, H, D, 16, B * nblk + 8, dtype=dt, device=str(dev))
    st = PagedDecodeState(model, bm, B, max_blocks=nblk, device=str(dev))
    g = torch.Generator(device=dev).manual_seed(1)
    st.cross_kv.normal_(generator=g)
    bm.pool.normal_(generator=g)
    st.cross_lens.fill_(cross_len)
    st.block_tables.copy_(torch.arange(B * nblk, dtype=torch.int32, device=dev).view(B, nblk))
    st.token_ids.copy_(torch.randint(0, 50000, (B,), generator=g, device=dev))
    ctx0 = st.ctx_lens.clone().fill_(self_len)
    st.ctx_lens.copy_(ctx0)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.no_grad():
        for _ in range(3):
            st.forward_step(B)
            st.ctx_lens.copy_(ctx0)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side), torch.no_grad():
        st.forward_step(B)
    torch.cuda.synchronize()
    w_bytes = sum(p.numel() * p.element_size() for n, p in model.hf_model.model.decoder.named_parameters()
                  if "embed_" not in n) + model.hf_model.proj_out.weight.numel() * 2
    kv_bytes = L * B * 2 * H * D * 2 * (cross_len + self_len)
    WORK[name] = (w_bytes + kv_bytes, "GB/s", None)

    def run(i):
        st.ctx_lens.copy_(ctx0)  # every replay attends the same self_len positions
        graph.replay()
    run.captures_graph = True
    return run


def _linear_table(torch, ops, dev):
    """The decode step's Linear shapes at batch 64: the tcgen05 kernel against cuBLAS
    (torch F.linear), each timed over 30 launches in a CUDA graph, rotating over enough
    weight copies that every launch reads its weights from HBM (> 256 MB per rotation)."""
    import torch.nn.functional as F

    shapes = [("small q|k|v", 2304, 768, 3, False), ("small d x d", 768, 768, 1, False),
              ("small fc1+gelu", 3072, 768, 1, True), ("small fc2", 768, 3072, 1, False),
              ("small head", 51865, 768, 1, False), ("large q|k|v", 3840, 1280, 3, False),
              ("large d x d", 1280, 1280, 1, False), ("large fc1+gelu", 5120, 1280, 1, True),
              ("large fc2", 1280, 5120, 1, False), ("large head", 51866, 1280, 1, False)]
    M = 64
    for name, Nf, K, groups, gelu in shapes:
        copies = max(2, -(-(256 << 20) // (Nf * K * 2)))
        ws = [(torch.randn(Nf, K, device=dev) * K ** -0.5).half() for _ in range(copies)]
        b = torch.zeros(Nf, device=dev).half()
        x = torch.randn(M, K, device=dev).half()
        outs = {}
        for impl in ("tcgen05", "cublas"):
            def run(i, impl=impl):
                w = ws[i % copies]
                if impl == "tcgen05":
                    return ops.linear(x, w, b, gelu=gelu, groups=groups)
                y = F.linear(x, w, b)
                return F.gelu(y) if gelu else y
            stream = torch.cuda.Stream(device=dev)
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                for i in range(3):
                    run(i)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(30):
                    run(i)
            with torch.cuda.stream(stream):
                g.replay()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                g.replay()
                e1.record(stream)
            torch.cuda.synchronize()
            outs[impl] = e0.elapsed_time(e1) * 1000.0 / 30
            del g
        wb = Nf * K * 2
        print(f"{name:16s} N={Nf:6d} K={K:5d}: tcgen05 {outs['tcgen05']:7.2f} us ({wb / outs['tcgen05'] / 1e3:6.0f} GB/s)"
              f"  cuBLAS {outs['cublas']:7.2f} us ({wb / outs['cublas'] / 1e3:6.0f} GB/s)")
        del ws


def _linear_dxd(torch, ops, dev, sets):
    """One Whisper-small d x d projection at batch 64 (N = K = 768), rotating over enough
    weight copies (> 256 MB) that each launch reads its weights from HBM."""
    copies = 224
    ws = [(torch.randn(768, 768, device=dev) * 0.036).half() for _ in range(copies)]
    b = torch.zeros(768, device=dev).half()
    x = torch.randn(64, 768, device=dev).half()
    out = torch.empty(64, 768, device=dev).half()
    WORK["linear_dxd"] = (768 * 768 * 2, "GB/s", None)
    return lambda i: ops.linear(x, ws[i % copies], b, out=out)


LIN_POINTS = ["entry", "set-up done", "griddepcontrol.wait returned", "first stage landed", "accumulator ready",
              "partials exchanged", "outputs stored", "exit"]


CASES = {
    "paged_cfg2": lambda t, o, dev, n: _paged(t, o, dev, n),
    "paged_big": lambda t, o, dev, n: _paged(t, o, dev, n, B=512, NB=16384, lo=448, name="paged_big"),
    "cross_cfg3": lambda t, o, dev, n: _cross(t, o, dev, n),
    "cross_dec": lambda t, o, dev, n: _cross_decode(t, o, dev, n),
    "proj_small": lambda t, o, dev, n: _proj(t, o, dev, n, 768, 12, 12, "proj_small"),
    "proj_large": lambda t, o, dev, n: _proj(t, o, dev, n, 1280, 32, 20, "proj_large"),
    "decode_small": lambda t, o, dev, n: _decode_small(t, o, dev, n),
    "linear_dxd": lambda t, o, dev, n: _linear_dxd(t, o, dev, n),
    "decode_large": lambda t, o, dev, n: _decode_small(t, o, dev, n, cross_len=1500, arch="whisper-large-v3",
                                                       dtype_name="bfloat16", name="decode_large"),
}

POINTS = {0: ["entry", "first lengths scanned", "first copy issued", "producer out of items", "first stage consumed",
              "warp 0 done", "griddepcontrol.wait returned", "producer done", "last stage landed"],
          1: ["entry", "griddepcontrol.wait returned", "done"]}


def _fetch_trace(lib, fn_name="spd_trace_fetch_paged"):
    import ctypes as C

    import numpy as np

    kernels, ctas, points = 2, 1024, 12
    buf = (C.c_ulonglong * (kernels * ctas * points))()
    fn = getattr(lib, fn_name)
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_size_t]
    if fn(C.addressof(buf), kernels * ctas * points) != 0:
        raise RuntimeError(f"{fn_name} failed")
    return np.frombuffer(buf, dtype=np.uint64).reshape(kernels, ctas, points).astype(np.float64)


def _summarise_trace(tr):
    """Per mark: when the CTAs reached it (µs after the first CTA's entry): min, median, max;
    then, per CTA of the streaming kernel, its stage count against its finishing time."""
    t0 = tr[0][:, 0][tr[0][:, 0] > 0].min()
    print("mark (µs after the first CTA entered)           CTAs    min   median      max")
    for k, names in POINTS.items():
        for pt, name in enumerate(names):
            v = tr[k][:, pt]
            v = v[v > 0]
            if v.size == 0:
                continue
            us = (v - t0) / 1e3
            kname = "stream" if k == 0 else "merge "
            print(f"{kname} {pt} {name:<38s} {v.size:5d} {us.min():7.2f} {float(sorted(us)[len(us) // 2]):8.2f} "
                  f"{us.max():8.2f}")
    live = tr[0][:, 0] > 0
    stages = tr[0][live, 9]
    done = (tr[0][live, 5] - t0) / 1e3
    landed = (tr[0][live, 8] - t0) / 1e3
    order = done.argsort()
    print("stages per CTA (warp 0): min %d median %d max %d" % (stages.min(), sorted(stages)[len(stages) // 2],
                                                               stages.max()))
    print("CTAs by finishing time: (done µs, last landed µs, stages) of the first, median and last five")
    for i in list(order[:5]) + list(order[len(order) // 2:len(order) // 2 + 5]) + list(order[-5:]):
        print(f"  {done[i]:6.2f} {landed[i]:6.2f} {int(stages[i]):3d}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES) + ["linear_table"])
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--sets", type=int, default=2)
    ap.add_argument("--time", type=int, default=0, help="time this many plain launches with CUDA events")
    ap.add_argument("--graph", type=int, default=0, help="time this many launches captured in one CUDA graph")
    ap.add_argument("--trace", action="store_true", help="use the trace build and print the last launch's timeline")
    a = ap.parse_args()
    if a.trace:
        sys.path.insert(0, str(PKG / "csrc"))
        import build as ext_build  # inference-speech-model_b200/csrc/build.py

        os.environ["SPD_B200_LIB"] = str(ext_build.build(trace=True))
    import torch
    from speech_serving import _native, ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if a.case == "linear_table":
        _linear_table(torch, ops, dev)
        return
    run = CASES[a.case](torch, ops, dev, a.sets)
    nvtx = getattr(run, "captures_graph", False)
    if nvtx:
        torch.cuda.nvtx.range_push("steps")
    for i in range(a.launches):
        run(i)
    torch.cuda.synchronize()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    print(f"{a.case}: {a.launches} launches ok")
    work, unit, per = WORK[a.case]
    scale = 1e9 if unit == "GB/s" else 1e12
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
        print(f"{a.case}: {us:.2f} us per launch (plain stream launches), {work / (us * 1e-6) / scale:.1f} {unit}")
    if a.graph or a.trace:
        k = a.graph or 32
        if nvtx:
            raise SystemExit("decode_small replays its own graph: use --time")
        stream = torch.cuda.Stream(device=dev)
        stream.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(k):
                run(i)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            g.replay()  # the GPU is busy while the timed replay is submitted
            s.record(stream)
            g.replay()
            e.record(stream)
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1000.0 / k
        w = sum(per[i % a.sets] for i in range(k)) / k if per else work
        print(f"{a.case}: {us:.2f} us per launch ({k} launches in a CUDA graph), {w / (us * 1e-6) / scale:.1f} {unit}")
        if a.trace and a.case.startswith("linear"):
            tr = _fetch_trace(_native.load(), "spd_trace_fetch_linear")[0]
            live = tr[:, 0] > 0
            t0 = tr[live, 0].min()
            for pt, name in enumerate(LIN_POINTS):
                v = tr[live, pt]
                v = v[v > 0]
                if v.size:
                    us = (v - t0) / 1e3
                    print(f"{pt} {name:<32s} {v.size:5d} {us.min():7.2f} {float(sorted(us)[len(us) // 2]):8.2f} "
                          f"{us.max():8.2f}")
        elif a.trace:
            _summarise_trace(_fetch_trace(_native.load()))


if __name__ == "__main__":
    main()
