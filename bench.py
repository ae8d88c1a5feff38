"""Benchmark of the B200 decode-attention hot path (BASELINE.json metric).

Default workload (N=1): BASELINE config 2 — paged single-query decoder self-attention,
fp16, B=64 sequences, 12 heads, head_dim 64, block_size 16, context ~ U[1,448], block
tables from a seeded permutation of a 4096-block pool, q/K/V ~ N(0,1)*0.5, scale 1/8.
A step is one launch of the paged attention kernel over one batch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  (N > 1: launched by torch.distributed.run, one rank per GPU; each rank is an
   independent replica on its own inputs — weak scaling, no data-path collective)

Timing:
  value  K steps replayed from one CUDA graph, each step reading a different one of 8
         resident input sets (8 x ~44 MB touched > 126 MB L2, so reads come from HBM);
         CUDA events on the replay stream; barrier + synchronize on both sides; the
         max time over ranks; GB/s of algorithmic bytes (valid K/V rows + q + out +
         tables + lengths) summed over ranks.
  e2e    the same metric through the public API (speech_serving.ops) with pinned HOST
         buffers: every step copies q/tables/lengths host->device, runs the op and copies
         the output device->host, timed with CUDA events around the whole loop.
  roofline  bytes per launch / average launch duration (graph replay time / K) against
         the measured HBM copy bandwidth (MEASURED_PEAKS.json hbm_gbs).
  cpu_baseline  the C port of the reference math (oracle/oracle.c, all host threads) on
         a bounded sample of the same workload, rank 0 at N=1 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path[:0] = [str(REPO), str(REPO / "inference-speech-model_b200")]

METRIC = "paged decode-attn HBM GB/s (% of 8 TB/s); decoder tokens/s at 1/2/4/8 GPU"
FALLBACK_HBM_GBS = 6650.0
N_SETS = 8

CFG2 = dict(B=64, H=12, D=64, bs=16, num_blocks=4096, max_ctx=448, scale=0.125)


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def make_inputs(seed: int, device: str = "cpu"):
    """Seeded config-2 batch.  Lengths and block tables come from a CPU generator (the
    same on every host); the pool and query values are drawn on `device`."""
    import torch

    c = CFG2
    g = torch.Generator().manual_seed(seed)
    ctx = torch.randint(1, c["max_ctx"] + 1, (c["B"],), generator=g, dtype=torch.int32)
    maxb = c["max_ctx"] // c["bs"]
    perm = torch.randperm(c["num_blocks"], generator=g).to(torch.int32)
    tables = perm[: c["B"] * maxb].view(c["B"], maxb).contiguous()
    gd = torch.Generator(device=device).manual_seed(seed)
    shape = (c["num_blocks"], c["bs"], c["H"], c["D"])
    q = (torch.randn(c["B"], c["H"], c["D"], generator=gd, device=device) * 0.5).half()
    kp = (torch.randn(shape, generator=gd, device=device) * 0.5).half()
    vp = (torch.randn(shape, generator=gd, device=device) * 0.5).half()
    return dict(q=q, k_pool=kp, v_pool=vp, tables=tables.to(device), ctx=ctx.to(device))


def algorithmic_bytes(ctx) -> int:
    """Bytes one launch must move: every valid K and V row of every head, plus q, out,
    block-table entries actually read and the lengths."""
    c = CFG2
    ctx = [int(x) for x in ctx]
    kv = sum(ctx) * c["H"] * c["D"] * 2 * 2
    qo = 2 * c["B"] * c["H"] * c["D"] * 2
    tab = sum(-(-x // c["bs"]) for x in ctx) * 4 + c["B"] * 4
    return kv + qo + tab


class ClockSampler:
    """Samples nvidia-smi SM clocks and throttle reasons every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.rows = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.rows.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i, v in enumerate(r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def cpu_baseline(seconds: float = 10.0, threads: int | None = None):
    """Times the C port of the reference math on the host cores over config-2 batches."""
    from oracle import c_oracle

    threads = threads or os.cpu_count()
    d = make_inputs(1000)  # on the host
    args = [d["q"].numpy(), d["k_pool"].numpy(), d["v_pool"].numpy(), d["tables"].numpy(), d["ctx"].numpy()]
    nbytes = algorithmic_bytes(d["ctx"])
    c_oracle.paged_decode_attention(*args, CFG2["scale"], threads=threads)  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        c_oracle.paged_decode_attention(*args, CFG2["scale"], threads=threads)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(nbytes * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} config-2 batches (B=64, fp16 pools) in {dt:.1f} s, oracle/oracle.c OpenMP"}


def bench_config(world: int) -> dict:
    """The `config` object of both arms' JSON lines (identical for the same N)."""
    return {"workload": "config 2: paged decode self-attention B=64 H=12 D=64 bs=16 ctx~U[1,448] "
                        "4096-block pool per input set",
            "global_batch": CFG2["B"] * world, "seq_len": CFG2["max_ctx"], "parallelism": f"replicas x{world}",
            "l2": f"each step reads the next of {N_SETS} input sets (rank r: seeds 1000+97r .. 1000+97r+{N_SETS - 1}; "
                  "~46 MB of K/V per set, > 126 MB L2 per rotation)",
            "timing": "K timed steps after W warm-up steps, each step one batch of the workload"}


def dist_setup(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return world, rank, local


def run_reference(args):
    """The reference arm: the reference's arithmetic for this path on the host cores.  The
    reference is PyTorch with no native CPU library, so the timed code is its math ported to
    C (oracle/oracle.c, OpenMP over all host threads), over the same rotation of input sets as
    our arm.  Under torchrun only rank 0 runs and prints."""
    world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import c_oracle

    threads = os.cpu_count()
    sets = []
    for i in range(N_SETS):
        d = make_inputs(1000 + i)
        sets.append(([d["q"].numpy(), d["k_pool"].numpy(), d["v_pool"].numpy(), d["tables"].numpy(),
                      d["ctx"].numpy()], algorithmic_bytes(d["ctx"])))
    for i in range(args.warmup):
        c_oracle.paged_decode_attention(*sets[i % N_SETS][0], CFG2["scale"], threads=threads)
    t0 = time.perf_counter()
    for i in range(args.steps):
        c_oracle.paged_decode_attention(*sets[i % N_SETS][0], CFG2["scale"], threads=threads)
    dt = time.perf_counter() - t0
    nbytes = sum(sets[i % N_SETS][1] for i in range(args.steps))
    v = nbytes / dt / 1e9
    line = {"metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 in, f32 arithmetic", "data": "synthetic",
            "impl": "reference", "config": bench_config(world),
            "timing": "host wall clock around the K steps (rank 0 only under torchrun)",
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{args.steps} config-2 batches rotating over {N_SETS} input sets, "
                                       "oracle/oracle.c OpenMP (the reference is PyTorch with no native CPU "
                                       "library; this is its arithmetic ported to C)"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def ref_triton_leg(sets, steps: int, dev):
    """The reference's own Triton kernel (`paged_decode_attention_kernel`,
    scripts/evaluate_paging_variants.py:56-133 of the reference), launched as the reference
    launches it (:632-642: grid (B, H), q pre-scaled, sm_scale 1.0, explicit strides) on the
    same rotating config-2 sets, K launches in one CUDA graph, CUDA events.  Its source is
    read, unmodified, from the reference checkout installed under baseline/_ref; only the
    kernel's own definition is compiled (the script's module imports audio and model
    libraries the kernel does not use)."""
    import ast

    import torch

    path = REPO / "baseline" / "_ref" / "scripts" / "evaluate_paging_variants.py"
    if not path.exists():
        return {"unavailable": "reference checkout not installed under baseline/_ref"}
    try:
        import triton
        import triton.language as tl

        tree = ast.parse(path.read_text())
        fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "paged_decode_attention_kernel")
        ns = {"triton": triton, "tl": tl}
        # compiled with the file's own name and line numbers, so triton reads the
        # unmodified source lines from the file
        exec(compile(ast.Module(body=[fn], type_ignores=[]), str(path), "exec"), ns)
        kern = ns["paged_decode_attention_kernel"]
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"could not load the reference kernel: {type(e).__name__}: {e}"[:300]}
    c = CFG2
    B, H, D, bs = c["B"], c["H"], c["D"], c["bs"]
    qs = [(s["q"] * c["scale"]).view(B, H, 1, D) for s in sets]  # exact: the scale is a power of two
    outs = [torch.zeros(B, H, 1, D, dtype=torch.float16, device=dev) for _ in sets]

    def launch(i):
        j = i % len(sets)
        s, q, o = sets[j], qs[j], outs[j]
        kc, vc, t = s["k_pool"], s["v_pool"], s["tables"]
        kern[(B, H)](q, kc, vc, t, s["ctx"], o, 1.0,
                     q.stride(0), q.stride(1), q.stride(2), q.stride(3),
                     kc.stride(0), kc.stride(1), kc.stride(2), kc.stride(3),
                     vc.stride(0), vc.stride(1), vc.stride(2), vc.stride(3),
                     t.stride(0), t.stride(1),
                     o.stride(0), o.stride(1), o.stride(2), o.stride(3),
                     BLOCK_SIZE=bs, HEAD_DIM=D)

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for i in range(len(sets)):
            launch(i)  # compiles the kernel
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(steps):
            launch(i)
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()  # keeps the GPU busy while the timed replay is submitted
        s0.record(stream)
        graph.replay()
        s1.record(stream)
    torch.cuda.synchronize()
    ms = s0.elapsed_time(s1)
    nbytes = sum(algorithmic_bytes(sets[i % len(sets)]["ctx"].cpu()) for i in range(steps))
    del graph
    return {"value": round(nbytes / (ms / 1e3) / 1e9, 2), "unit": "GB/s", "launch_us": round(ms * 1e3 / steps, 3),
            "source": "baseline/_ref/scripts/evaluate_paging_variants.py (unmodified kernel definition)",
            "triton": triton.__version__, "outputs": outs}


# ---------------------------------------------------------------------------- serving legs
SERVING = {
    "config1": dict(arch="whisper-class-tiny", dtype="float32", n=4, rate=None, out=(64, 64), mels=80,
                    desc="WhisperClassSpeechEncoderDecoderModel(4,4,6,384,80,51865) seed 0, fp32, 4 requests, "
                         "64 tokens each, graph decode, direct handoff; median of 3 timed runs"),
    "config4": dict(arch="whisper-small", dtype="float16", n=256, rate=None, out=(20, 200), mels=80,
                    desc="random-init Whisper-small, fp16, 256-request burst, audio U[2,30] s, outputs U{20..200}"),
    "config5": dict(arch="whisper-large-v3", dtype="bfloat16", n=2048, rate=64.0, out=(20, 224), mels=128,
                    hf_self_check=True, desc="random-init Whisper-large-v3, bf16, Poisson 64 req/s per GPU, audio U[2,30] s, "
                         "outputs U{20..224}"),
    "config5_burst": dict(arch="whisper-large-v3", dtype="bfloat16", n=512, rate=None, out=(20, 224), mels=128,
                          desc="capacity of the config-5 engine: random-init Whisper-large-v3, bf16, all requests "
                               "arriving at once, audio U[2,30] s, outputs U{20..224}"),
}
AGREEMENT_SAMPLE = 64  # requests of rank 0 re-decoded by the HF decoder after a serving leg


def _serving_model(cfg, dev):
    import torch
    from speech_serving.models import PretrainedWhisperModel, WhisperClassSpeechEncoderDecoderModel
    from speech_serving.serving import whisper_config

    dtype = getattr(torch, cfg["dtype"])
    if cfg["arch"] == "whisper-class-tiny":
        torch.manual_seed(0)
        return WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865).to(dev, dtype).eval(), dtype
    return PretrainedWhisperModel(config=whisper_config(cfg["arch"]), device=str(dev), dtype=dtype, seed=0), dtype


def _serving_scheduler(model, dtype, dev, max_batch=64, dec_blocks=4096):
    from speech_serving import BlockManager, DualCacheManager, EncoderBlockManager, MemoryGuard
    from speech_serving.phase_aware_scheduler import PhaseAwareSpeechScheduler

    L, H, D = model.num_decoder_layers, model.num_heads, model.head_dim
    enc = EncoderBlockManager(L, H, D, 16, 1, dtype=dtype, device=str(dev))  # direct handoff: unused
    dec = BlockManager(L, H, D, 16, dec_blocks, dtype=dtype, device=str(dev))
    return PhaseAwareSpeechScheduler(model, DualCacheManager(enc, dec), MemoryGuard(), max_batch_size=max_batch,
                                     device=str(dev), eos_token_id=-1, batch_encoder=True, graph_decode=True,
                                     graph_readback_k=4, graph_direct_encoder_kv=True)


def serving_leg(name, n_req, dev, rank, world, models):
    """Decoder tokens/s of one serving configuration: every rank serves its own request
    stream (replicas); whole-job tokens/s = tokens of all ranks / slowest rank's wall.
    After the timed run, rank 0 re-decodes a sample of its requests with the unpatched HF
    decoder (the reference's path) and reports how many sequences are identical."""
    import torch
    import torch.distributed as dist
    from speech_serving import replicas
    from speech_serving.phase_aware_scheduler import WHISPER_DEFAULT_PREFIX_TOKENS
    from speech_serving.serving import run_engine, synthetic_requests

    cfg = SERVING[name]
    key = (cfg["arch"], cfg["dtype"])
    if key not in models:
        models.clear()  # one model at a time on the device
        torch.cuda.empty_cache()
        models[key] = _serving_model(cfg, dev)
    model, dtype = models[key]
    sched = _serving_scheduler(model, dtype, dev, max_batch=min(64, max(4, n_req)))
    if name == "config1":
        gen = torch.Generator().manual_seed(1)
        from speech_serving.serving import SyntheticRequest
        reqs = [SyntheticRequest(torch.randn(80, 3000, generator=gen).clamp(-1.5, 1.5).pin_memory(), 30.0, 64, 0.0)
                for _ in range(4)]
        warm = reqs
    else:
        reqs = synthetic_requests(n_req, cfg["mels"], seed=1000 + rank, out_lo=cfg["out"][0], out_hi=cfg["out"][1],
                                  rate=cfg["rate"])
        warm = synthetic_requests(8, cfg["mels"], seed=99, out_lo=8, out_hi=16)
    run_engine(sched, warm, WHISPER_DEFAULT_PREFIX_TOKENS)  # captures the graphs
    # The requests' audio sits in pinned host buffers; a server reuses its pinned staging
    # buffers, while these were just allocated, and the first DMA out of newly pinned pages
    # costs about 4 ms per MB on these boxes.  One untimed copy of each buffer first, all
    # kept alive together so that torch's caching allocator also holds the device memory
    # a burst of uploads needs (a running server's pool would; growing it inside the timed
    # run cost up to 0.3 s of a 1.2 s config-4 run).  The timed run still copies every
    # request's audio to the device.
    staged = [q.mel.to(dev, non_blocking=True) for q in reqs]
    torch.cuda.synchronize()
    del staged
    sched.reset_telemetry()
    if world > 1:
        dist.barrier()
    # config 1 is a 40 ms run, at the mercy of a single host hiccup: the median of three
    runs = []
    for _ in range(3 if name == "config1" else 1):
        sched.reset_telemetry()
        runs.append(run_engine(sched, reqs, WHISPER_DEFAULT_PREFIX_TOKENS))
    r = sorted(runs, key=lambda x: x["wall_s"])[len(runs) // 2]
    wall_max = replicas.max_over_ranks(r["wall_s"])
    toks_all = replicas.sum_over_ranks(r["generated_tokens"])
    leaks = sched.dual_cache.decoder_bm.allocated_block_count
    out = {"workload": cfg["desc"], "requests_per_rank": r["requests"], "failed": r["failed"],
           "decoder_tok_s": round(replicas.whole_job_rate(toks_all, wall_max * 1e3), 1),
           "generated_tokens": int(toks_all), "wall_s_max": round(wall_max, 3),
           "rank0": {k: r[k] for k in ("decoder_tok_s", "decode_steps", "decode_phase_s", "ttft_p50_s",
                                       "latency_p50_s", "latency_p95_s")},
           "leaked_decoder_blocks": leaks, "timing": "wall clock around the serving loop, synchronized both ends"}
    if name == "config1":
        out["tokens"] = r["tokens_by_request"]
    elif rank == 0:
        from speech_serving.hf_reference import (NEAR_TIE_STEPS, hf_greedy_tokens, hf_top2_margins,
                                                 near_tie_divergences, sequence_agreement)

        t_check = time.perf_counter()
        k = min(AGREEMENT_SAMPLE, len(reqs))
        mels = torch.stack([q.mel for q in reqs[:k]])
        lens = [q.max_new_tokens for q in reqs[:k]]
        ours = r["tokens_by_request"][:k]
        ref = hf_greedy_tokens(model, mels, WHISPER_DEFAULT_PREFIX_TOKENS, lens, batch=32)
        a = sequence_agreement(ours, ref)
        ties = near_tie_divergences(ours, ref, hf_top2_margins(model, mels, WHISPER_DEFAULT_PREFIX_TOKENS, ref), dtype)
        agree = {"requests": a["requests"], "identical": a["identical"],
                 "identical_frac": round(a["identical_frac"], 4), "first_divergence": a["first_divergence"],
                 "divergences_at_near_tie": ties["at_near_tie"],
                 "requests_without_near_tie": ties["requests_without_near_tie"],
                 "identical_without_near_tie": ties["identical_without_near_tie"],
                 "near_tie": f"HF top-1 minus top-2 logit within {NEAR_TIE_STEPS} steps of the {cfg['dtype']} grid "
                             "at the divergent position (HF teacher-forced on its own sequence)",
                 "sample": f"the first {k} requests of rank 0, re-decoded greedily by the unpatched HF decoder "
                           "(batch 32) on the same weights, device and dtype"}
        if cfg.get("hf_self_check"):
            # the HF decoder against itself at another batch size: the agreement floor that
            # ties in this dtype leave to any second implementation
            self_a = sequence_agreement(hf_greedy_tokens(model, mels, WHISPER_DEFAULT_PREFIX_TOKENS, lens, batch=8), ref)
            agree["hf_self_agreement"] = {"identical": self_a["identical"], "requests": self_a["requests"],
                                          "what": "HF decoder at batch 8 against HF at batch 32, same requests"}
        agree["check_s"] = round(time.perf_counter() - t_check, 1)
        out["hf_sequence_agreement"] = agree
    del sched
    torch.cuda.empty_cache()
    return out


def serving_cpu_baseline():
    """Config 1 through the CPU eager-decode oracle (the reference's eager arithmetic) on
    all host cores: decoder tokens/s."""
    import torch
    from oracle import eager_decode
    from speech_serving.models import WhisperClassSpeechEncoderDecoderModel
    from speech_serving.phase_aware_scheduler import WHISPER_DEFAULT_PREFIX_TOKENS

    threads = os.cpu_count()
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    sd = WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865).state_dict()
    gen = torch.Generator().manual_seed(1)
    mels = torch.stack([torch.randn(80, 3000, generator=gen).clamp(-1.5, 1.5) for _ in range(4)])
    t0 = time.perf_counter()
    toks = eager_decode.greedy_decode(sd, mels, WHISPER_DEFAULT_PREFIX_TOKENS, 64, num_heads=6)
    dt = time.perf_counter() - t0
    n = sum(len(t) for t in toks)
    return {"value": round(n / dt, 1), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"config 1 end to end (encode + 4x64 greedy tokens) in {dt:.2f} s, oracle/eager_decode.py",
            "tokens": toks}


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_setup(args)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        # every rank drives its own serving loop from the host: give each its own share of
        # the host cores, so N schedulers and their intra-op thread pools do not compete
        cores = sorted(os.sched_getaffinity(0))
        per = max(1, len(cores) // world)
        mine = cores[rank * per:(rank + 1) * per] or cores
        os.sched_setaffinity(0, mine)
        torch.set_num_threads(len(mine))
    from speech_serving import ops, replicas

    c = CFG2
    sets = [make_inputs(1000 + 97 * rank + i, device=dev) for i in range(N_SETS)]
    outs = [torch.empty(c["B"], c["H"], c["D"], dtype=torch.float16, device=dev) for _ in range(N_SETS)]
    ws = ops.paged_attn_workspace(c["B"], c["H"], c["D"], sets[0]["tables"].shape[1], dev)
    bytes_per = [algorithmic_bytes(s["ctx"].cpu()) for s in sets]

    def launch(i):
        s = sets[i % N_SETS]
        ops.paged_decode_attention(s["q"], s["k_pool"], s["v_pool"], s["tables"], s["ctx"], scale=c["scale"],
                                   out=outs[i % N_SETS], workspace=ws)

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            launch(i)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(args.steps):
            launch(i)
    for _ in range(max(args.warmup, 3) // args.steps + 1):
        graph.replay()  # warm the graph itself
    torch.cuda.synchronize()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pr = torch.cuda.get_device_properties(dev)
    sampler = ClockSampler(f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0")

    def sustain(seconds):
        # untimed replays of the same graph so the clock samples see this load
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end:
            graph.replay()
            torch.cuda.synchronize()

    with sampler:
        sustain(0.6)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            # one untimed replay first: the GPU works on it while the host submits the
            # timed replay, so the host's graph-launch latency is not counted as GPU time
            graph.replay()
            start.record(stream)
            graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        sustain(0.6)
    ms = start.elapsed_time(end)
    ms_max = replicas.max_over_ranks(ms)
    launch_us_ranks = [round(x * 1e3 / args.steps, 3) for x in replicas.gather_over_ranks(ms)]
    bytes_rank = sum(bytes_per[i % N_SETS] for i in range(args.steps))
    value = replicas.whole_job_rate(replicas.sum_over_ranks(bytes_rank), ms_max) / 1e9
    launch_ms = ms / args.steps
    achieved = (bytes_rank / args.steps) / (launch_ms / 1e3) / 1e9

    # ---- e2e through the public API with pinned host buffers ----------------------
    # Every step copies its q, block tables and lengths from pinned host memory and its
    # output back.  A step's three inputs sit in one pinned staging buffer (q | tables |
    # lengths, each region 16-byte aligned) and move with one copy into a device buffer of
    # the same layout, whose views are the call's tensors.  The K steps' public-API calls
    # are captured in one CUDA graph; the copies run on two copy streams into
    # double-buffered device inputs, so step i+1's inputs (and step i-1's output) move
    # while step i's kernel runs.
    def _packed(q, tables, ctx):
        parts = [t.contiguous().view(-1).view(torch.uint8) for t in (q, tables, ctx)]
        return torch.cat(parts)

    q_bytes, t_bytes = sets[0]["q"].numel() * 2, sets[0]["tables"].numel() * 4
    assert q_bytes % 16 == 0 and t_bytes % 16 == 0
    hin = [_packed(s["q"], s["tables"], s["ctx"]).cpu().pin_memory() for s in sets]
    hout = [torch.empty(c["B"], c["H"], c["D"], dtype=torch.float16).pin_memory() for _ in range(N_SETS)]
    din = [torch.empty_like(hin[0], device=dev) for _ in range(2)]
    dq = [d[:q_bytes].view(torch.float16).view(sets[0]["q"].shape) for d in din]
    dt_ = [d[q_bytes:q_bytes + t_bytes].view(torch.int32).view(sets[0]["tables"].shape) for d in din]
    dc = [d[q_bytes + t_bytes:].view(torch.int32) for d in din]
    dout = [torch.empty_like(outs[0]) for _ in range(2)]
    s_h2d, s_d2h = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    K = args.steps
    h2d_done = [torch.cuda.Event() for _ in range(K)]
    k_done = [torch.cuda.Event() for _ in range(K)]
    d2h_done = [torch.cuda.Event() for _ in range(K)]

    def e2e_steps():
        main = torch.cuda.current_stream()
        s_h2d.wait_stream(main)
        s_d2h.wait_stream(main)
        for i in range(K):
            b, j = i % 2, i % N_SETS
            with torch.cuda.stream(s_h2d):
                if i >= 2:
                    s_h2d.wait_event(k_done[i - 2])  # buffer b was read by step i-2
                din[b].copy_(hin[j], non_blocking=True)
                h2d_done[i].record(s_h2d)
            main.wait_event(h2d_done[i])
            if i >= 2:
                main.wait_event(d2h_done[i - 2])  # output buffer b was read back
            ops.paged_decode_attention(dq[b], sets[j]["k_pool"], sets[j]["v_pool"], dt_[b], dc[b], scale=c["scale"],
                                       out=dout[b], workspace=ws)
            k_done[i].record(main)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(k_done[i])
                hout[j].copy_(dout[b], non_blocking=True)
                d2h_done[i].record(s_d2h)
        main.wait_stream(s_h2d)
        main.wait_stream(s_d2h)

    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph, stream=stream):
        e2e_steps()
    with torch.cuda.stream(stream):
        e2e_graph.replay()  # warm
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        e2e_graph.replay()
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms_max = replicas.max_over_ranks(e0.elapsed_time(e1))
    e2e_value = replicas.whole_job_rate(replicas.sum_over_ranks(bytes_rank), e2e_ms_max) / 1e9
    h2d = din[0].numel()
    d2h = dout[0].numel() * 2
    # the read-back outputs are the kernel's: last rotation of host buffers vs the oracle below
    e2e_out_last = hout[(K - 1) % N_SETS].clone()
    del e2e_graph

    # correctness guard on the timed data: one set against the oracle's C port
    ok_err = None
    if rank == 0:
        from oracle import c_oracle
        import numpy as np

        s0 = sets[0]
        ref = c_oracle.paged_decode_attention(s0["q"].cpu().numpy(), s0["k_pool"].cpu().numpy(),
                                              s0["v_pool"].cpu().numpy(), s0["tables"].cpu().numpy(),
                                              s0["ctx"].cpu().numpy(), c["scale"])
        outs[0].fill_(float("nan"))  # an unwritten output cannot pass on stale values
        ops.paged_decode_attention(s0["q"], s0["k_pool"], s0["v_pool"], s0["tables"], s0["ctx"], scale=c["scale"],
                                   out=outs[0], workspace=ws)
        ok_err = float(np.abs(outs[0].float().cpu().numpy() - ref).max())
        jl = (args.steps - 1) % N_SETS  # the e2e leg's read-back outputs are the kernel's
        sl = sets[jl]
        chk = ops.paged_decode_attention(sl["q"], sl["k_pool"], sl["v_pool"], sl["tables"], sl["ctx"], scale=c["scale"],
                                         workspace=ws)
        if not torch.equal(chk.cpu(), e2e_out_last):
            raise RuntimeError("e2e read-back differs from the device-resident call on the same inputs")
        if ok_err > 2e-3:
            raise RuntimeError(f"benchmark output differs from the oracle by {ok_err}")
        if ops.read_error_word(ws) != 0:
            raise RuntimeError("kernel reported a device error during the benchmark")

    del graph
    ref_triton = None
    if rank == 0 and not args.no_ref_triton:
        ref_triton = ref_triton_leg(sets, args.steps, dev)
        if "outputs" in ref_triton:
            # the reference kernel computes the same attention: its outputs agree with ours
            tri = ref_triton.pop("outputs")
            j = (args.steps - 1) % N_SETS
            s_ = sets[j]
            mine = ops.paged_decode_attention(s_["q"], s_["k_pool"], s_["v_pool"], s_["tables"], s_["ctx"],
                                              scale=c["scale"], workspace=ws)
            ref_triton["max_abs_diff_vs_ours"] = float((tri[j].view_as(mine).float() - mine.float()).abs().max())
            ref_triton["frac"] = round(ref_triton["value"] / _peaks()[0], 4)
    serving = {}
    legs = [x for x in args.serving.split(",") if x and x != "none"]
    models = {}
    for name in legs:
        n_req = {"config1": 4, "config4": SERVING["config4"]["n"], "config5": args.config5_requests,
                 "config5_burst": args.config5_burst_requests}[name]
        serving[name] = serving_leg(name, n_req, dev, rank, world, models)
    models.clear()
    if rank == 0 and world == 1 and "config1" in serving and not args.no_cpu_baseline:
        cb = serving_cpu_baseline()
        ours = serving["config1"].pop("tokens")
        ref = cb.pop("tokens")
        agree = sum(a == b for x, y in zip(ours, ref) for a, b in zip(x, y)) / max(1, sum(len(x) for x in ref))
        serving["config1"]["cpu_baseline"] = cb
        serving["config1"]["token_agreement_vs_cpu_oracle"] = round(agree, 4)
    elif "config1" in serving:
        serving["config1"].pop("tokens", None)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, peak_kind = _peaks()
    # DRAM traffic per launch: the ncu capture's dram read+write over algorithmic bytes of
    # the same kernel and shape (profiles/ncu_traffic.json), applied to this batch's bytes.
    traffic = None
    tf = REPO / "profiles" / "ncu_traffic.json"
    if tf.exists():
        ratio = json.loads(tf.read_text()).get("paged_decode_attn_config2", {}).get("traffic_over_algorithmic")
        if ratio:
            traffic = int(ratio * bytes_rank / args.steps)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16 in, f32 arithmetic", "data": "synthetic",
        "config": bench_config(world),
        "timing": "the K steps replayed from one CUDA graph behind one untimed replay, CUDA events on the replay "
                  "stream, barrier + synchronize on both sides, max over ranks",
        "launch_us_per_rank": launch_us_ranks,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} hbm_gbs (copy bandwidth)",
                     "bytes_per_launch": int(bytes_rank / args.steps), "launch_us": round(launch_ms * 1e3, 3)},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "speech_serving.ops.paged_decode_attention (ctypes -> C ABI), pinned host buffers (a step's q, "
                        "tables and lengths staged in one buffer, one copy); the K steps "
                        "captured in one CUDA graph, copies on two copy streams overlapping the previous step's kernel "
                        "(double-buffered device inputs)"},
        "gpu_launches": 2 * args.steps,  # streaming kernel + split merge kernel per step
        "clocks": sampler.summary(),
        "max_abs_err_vs_oracle": ok_err,
        "ref_triton": ref_triton,
        "serving": serving,
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-triton", action="store_true", help="skip timing the reference's Triton kernel")
    ap.add_argument("--serving", default="config1,config4,config5,config5_burst",
                    help="comma-separated serving legs (config1, config4, config5, config5_burst) or none")
    ap.add_argument("--config5-requests", type=int, default=2048,
                    help="config-5 requests per rank (the configuration's 2048-request Poisson stream, 32 s)")
    ap.add_argument("--config5-burst-requests", type=int, default=512,
                    help="requests per rank of the config-5 capacity leg (all arriving at once)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
