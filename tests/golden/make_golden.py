"""Generates the golden fixtures in this directory by running the REFERENCE engine on CPU.

Run in a container where the reference project is importable:
    python tests/golden/make_golden.py --reference <path-to-reference-checkout>

Every fixture is produced by the reference's own code (imported, not restated), with
seeded inputs, and is small enough to commit.  The oracle (oracle/attention_oracle.py)
and the CUDA kernels are pinned against these files by tests/test_oracle_golden.py and
tests/test_kernels_gpu.py.  Nothing at test time imports the reference.

Fixtures:
  paged_attn_ref.npz      op (1)/(5) math: EncoderAttentionBackend.forward
                          (speech_serving/encoder_attention.py:21-71) = paged gather +
                          softmax(q·Kᵀ/√D)·V, on pools/tables from the reference BlockManager
  cross_attn_ref.npz      op (2): DecoderLayer.forward cross-attention with a bool length
                          mask (speech_serving/models.py:167-203)
  kv_write_ref.npz        op (3): per-token paged writes of the reference eager scheduler
                          (speech_serving/phase_aware_scheduler.py:678-690, :1004-1010)
  block_gather_ref.npz    op (5): encoder pool store + gather of the non-direct handoff
                          (speech_serving/phase_aware_scheduler.py:588-624)
  cross_kv_project_ref.npz op (4): PretrainedWhisperModel.encode projections
                          (speech_serving/models.py:554-561) on a random-init WhisperConfig
  config1_tokens.json     BASELINE config 1 end to end: eager scheduler tokens
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn

HERE = Path(__file__).resolve().parent


def _import_reference(path: str):
    sys.path.insert(0, path)
    import speech_serving.models as models  # noqa: F401
    from speech_serving.block_manager import BlockManager
    from speech_serving.dual_cache_manager import DualCacheManager
    from speech_serving.encoder_attention import EncoderAttentionBackend
    from speech_serving.encoder_block_manager import EncoderBlockManager
    from speech_serving.memory_guard import MemoryGuard
    from speech_serving.phase_aware_scheduler import PhaseAwareSpeechScheduler, WHISPER_DEFAULT_PREFIX_TOKENS

    return dict(models=models, BlockManager=BlockManager, DualCacheManager=DualCacheManager,
                EncoderAttentionBackend=EncoderAttentionBackend, EncoderBlockManager=EncoderBlockManager,
                MemoryGuard=MemoryGuard, Scheduler=PhaseAwareSpeechScheduler,
                PREFIX=WHISPER_DEFAULT_PREFIX_TOKENS)


def _h(x: torch.Tensor) -> torch.Tensor:
    """Rounds to the nearest fp16 value, kept as fp32 for the reference's fp32 math."""
    return x.half().float()


# --------------------------------------------------------------------------- op (1)
def make_paged_attn(R) -> None:
    cases = {}
    for name, (H, D, bs, NB, ctxs) in {
        "small": (4, 16, 8, 48, [1, 7, 8, 9, 33, 0, 64]),
        "whisper": (4, 64, 16, 36, [1, 15, 16, 17, 100, 300, 0]),
    }.items():
        torch.manual_seed(1234 + H)
        bm = R["BlockManager"](num_layers=1, num_kv_heads=H, head_dim=D, block_size=bs, num_blocks=NB,
                               dtype=torch.float32, device="cpu")
        # fp16-representable values, so the fp16 kernels see exactly the reference's inputs
        bm.key_pool[0].copy_(_h(torch.randn(NB, bs, H, D) * 0.5))
        bm.value_pool[0].copy_(_h(torch.randn(NB, bs, H, D) * 0.5))
        max_blocks = max(-(-c // bs) for c in ctxs)
        tables = np.zeros((len(ctxs), max_blocks), np.int32)
        for b, c in enumerate(ctxs):
            for j in range(-(-c // bs)):
                tables[b, j] = bm.allocate_block()  # reference LIFO allocation order
        q = _h(torch.randn(len(ctxs), H, D) * 0.5)
        out = np.zeros((len(ctxs), H, D), np.float32)
        for b, c in enumerate(ctxs):
            if c == 0:
                continue  # the Triton reference returns early; output stays zero
            tab = [int(x) for x in tables[b, : -(-c // bs)]]
            o = R["EncoderAttentionBackend"].forward(q[b][None, :, None, :], tab, bm.key_pool[0],
                                                     bm.value_pool[0], c, bs)
            out[b] = o[0, :, 0, :].numpy()
        cases[name] = dict(q=q.half().numpy(), k_pool=bm.key_pool[0].half().numpy(),
                           v_pool=bm.value_pool[0].half().numpy(),
                           block_tables=tables, context_lens=np.array(ctxs, np.int32), out=out)
    np.savez_compressed(HERE / "paged_attn_ref.npz",
                        **{f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()})


# --------------------------------------------------------------------------- op (2)
class _Zero(nn.Module):
    def forward(self, x):
        return torch.zeros_like(x)


def make_cross_attn(R) -> None:
    """Drives the reference DecoderLayer so that its output minus its input is exactly the
    cross-attention result: self-attention and MLP contribute zero, norm2 and the
    cross q/out projections are identities."""
    cases = {}
    for name, (B, H, D, T, valid) in {
        "small": (5, 4, 16, 40, [40, 1, 17, 33, 2]),
        "whisper": (3, 2, 64, 600, [600, 300, 599]),
    }.items():
        torch.manual_seed(77 + D)
        layer = R["models"].DecoderLayer(H * D, H, D, is_decoder=True).eval()
        with torch.no_grad():
            layer.self_attn_out.weight.zero_()
            layer.norm2 = nn.Identity()
            layer.cross_attn_q.weight.copy_(torch.eye(H * D))
            layer.cross_attn_out.weight.copy_(torch.eye(H * D))
            layer.mlp = _Zero()
            q = _h(torch.randn(B, H, D) * 0.5)
            k = _h(torch.randn(B, H, T, D) * 0.5)
            v = _h(torch.randn(B, H, T, D) * 0.5)
            mask = torch.zeros(B, 1, 1, T, dtype=torch.bool)
            for b, n in enumerate(valid):
                mask[b, 0, 0, :n] = True
            x = q.reshape(B, 1, H * D)
            y, _, _ = layer(x, encoder_past_kv=(k, v), encoder_attention_mask=mask)
            out = (y - x).reshape(B, H, D)
        cases[name] = dict(q=q.half().numpy(), k=k.half().numpy(), v=v.half().numpy(),
                           valid_lens=np.array(valid, np.int32),
                           out=out.numpy())
    np.savez_compressed(HERE / "cross_attn_ref.npz",
                        **{f"{c}__{k}": v for c, d in cases.items() for k, v in d.items()})


# --------------------------------------------------------------------------- op (3)
def make_kv_write(R) -> None:
    torch.manual_seed(999)
    H, hid, L, bs, NB = 4, 64, 2, 8, 24
    model = R["models"].WhisperClassSpeechEncoderDecoderModel(2, L, H, hid, 80, 100).eval()
    enc_bm = R["EncoderBlockManager"](L, H, hid // H, bs, 64, dtype=torch.float32, device="cpu")
    dec_bm = R["BlockManager"](L, H, hid // H, bs, NB, dtype=torch.float32, device="cpu")
    sched = R["Scheduler"](model, R["DualCacheManager"](enc_bm, dec_bm), R["MemoryGuard"](), max_batch_size=4,
                           device="cpu")
    captured = {}
    orig = sched._complete_request

    def hook(req, status):
        captured[req.id] = dict(table=list(req.decoder_block_table),
                                kv=[(k.clone(), v.clone()) for k, v in req.cached_decoder_kv],
                                tokens=list(req.generated_tokens))
        return orig(req, status)

    sched._complete_request = hook
    mels = [torch.randn(80, n) for n in (40, 64, 90)]
    for m in mels:
        sched.submit(m, prompt_token_ids=torch.tensor([[1, 2]]), max_new_tokens=12)
    sched.run_until_done()
    ids = sorted(captured)
    T = max(c["kv"][0][0].shape[2] for c in captured.values())
    maxb = max(len(c["table"]) for c in captured.values())
    k_rows = np.zeros((len(ids), L, H, T, hid // H), np.float32)
    v_rows = np.zeros_like(k_rows)
    lens = np.zeros(len(ids), np.int32)
    tables = np.full((len(ids), maxb), -1, np.int32)
    for i, rid in enumerate(ids):
        c = captured[rid]
        t = c["kv"][0][0].shape[2]
        lens[i] = t
        tables[i, : len(c["table"])] = c["table"]
        for l in range(L):
            k_rows[i, l, :, :t] = c["kv"][l][0][0].numpy()
            v_rows[i, l, :, :t] = c["kv"][l][1][0].numpy()
    np.savez_compressed(HERE / "kv_write_ref.npz", k_rows=k_rows, v_rows=v_rows, lens=lens, tables=tables,
                        k_pools=np.stack([p.numpy() for p in dec_bm.key_pool]),
                        v_pools=np.stack([p.numpy() for p in dec_bm.value_pool]), block_size=np.int32(bs))


# --------------------------------------------------------------------------- op (5)
def make_block_gather(R) -> None:
    torch.manual_seed(7)
    H, hid, L, bs = 4, 64, 2, 8
    model = R["models"].WhisperClassSpeechEncoderDecoderModel(L, L, H, hid, 80, 100).eval()
    enc_bm = R["EncoderBlockManager"](L, H, hid // H, bs, 32, dtype=torch.float32, device="cpu")
    dec_bm = R["BlockManager"](L, H, hid // H, bs, 32, dtype=torch.float32, device="cpu")
    sched = R["Scheduler"](model, R["DualCacheManager"](enc_bm, dec_bm), R["MemoryGuard"](), max_batch_size=2,
                           device="cpu", cache_cross_kv=True)
    got = {}
    orig_setup = sched._setup_request_after_encode

    def setup_hook(req, encoder_hidden, encoder_kv_list, full_hash=None, enc_time=0.0):
        got[req.id] = dict(src=[(k.clone(), v.clone()) for k, v in encoder_kv_list])
        orig_setup(req, encoder_hidden, encoder_kv_list, full_hash=full_hash, enc_time=enc_time)
        got[req.id]["table"] = list(req.encoder_block_table)
        got[req.id]["T"] = req.encoder_seq_len
        got[req.id]["gathered"] = [(k.clone(), v.clone()) for k, v in req.cached_encoder_kv]

    sched._setup_request_after_encode = setup_hook
    for n in (40, 70):
        sched.submit(torch.randn(80, n), prompt_token_ids=torch.tensor([[1]]), max_new_tokens=2)
    sched.run_until_done()
    ids = sorted(got)
    Tm = max(g["T"] for g in got.values())
    maxb = max(len(g["table"]) for g in got.values())
    D = hid // H
    src_k = np.zeros((len(ids), L, H, Tm, D), np.float32)
    src_v = np.zeros_like(src_k)
    gat_k = np.zeros_like(src_k)
    gat_v = np.zeros_like(src_k)
    tables = np.full((len(ids), maxb), -1, np.int32)
    lens = np.zeros(len(ids), np.int32)
    for i, rid in enumerate(ids):
        g = got[rid]
        T = g["T"]
        lens[i] = T
        tables[i, : len(g["table"])] = g["table"]
        for l in range(L):
            src_k[i, l, :, :T] = g["src"][l][0][0].numpy()
            src_v[i, l, :, :T] = g["src"][l][1][0].numpy()
            gat_k[i, l, :, :T] = g["gathered"][l][0][0].numpy()
            gat_v[i, l, :, :T] = g["gathered"][l][1][0].numpy()
    np.savez_compressed(HERE / "block_gather_ref.npz", src_k=src_k, src_v=src_v, gathered_k=gat_k,
                        gathered_v=gat_v, tables=tables, lens=lens,
                        k_pools=np.stack([p.numpy() for p in enc_bm.key_pool]),
                        v_pools=np.stack([p.numpy() for p in enc_bm.value_pool]), block_size=np.int32(bs))


# --------------------------------------------------------------------------- op (4)
def make_cross_kv_project(R) -> None:
    from transformers import WhisperConfig, WhisperForConditionalGeneration

    torch.manual_seed(5)
    cfg = WhisperConfig(d_model=64, encoder_layers=2, decoder_layers=2, encoder_attention_heads=4,
                        decoder_attention_heads=4, encoder_ffn_dim=128, decoder_ffn_dim=128, num_mel_bins=80,
                        vocab_size=100, max_source_positions=1500, max_target_positions=448,
                        pad_token_id=0, bos_token_id=1, eos_token_id=2, decoder_start_token_id=3,
                        suppress_tokens=[], begin_suppress_tokens=[])
    hf = WhisperForConditionalGeneration(cfg).eval()

    class Shim:  # the attributes PretrainedWhisperModel.encode reads (models.py:554-561)
        hf_model = hf
        num_heads = 4
        head_dim = 16

    mel = torch.randn(1, 80, 3000).clamp(-1.5, 1.5)
    with torch.no_grad():
        enc_out, kv = R["models"].PretrainedWhisperModel.encode(Shim(), mel)
    rows = 256  # the projection is row-wise; a slice of positions pins it fully
    data = dict(enc_out=enc_out[:, :rows].numpy())
    for l, layer in enumerate(hf.model.decoder.layers):
        a = layer.encoder_attn
        data[f"wk{l}"] = a.k_proj.weight.detach().numpy()
        data[f"wv{l}"] = a.v_proj.weight.detach().numpy()
        data[f"bv{l}"] = a.v_proj.bias.detach().numpy()
        assert a.k_proj.bias is None
        data[f"k{l}"] = kv[l][0][:, :, :rows].numpy()
        data[f"v{l}"] = kv[l][1][:, :, :rows].numpy()
    np.savez_compressed(HERE / "cross_kv_project_ref.npz", **data)


# --------------------------------------------------------------------------- config 1
def config1_inputs():
    """BASELINE config 1 inputs: seeded model and 4 mels 80x3000 N(0,1) clamped."""
    g = torch.Generator().manual_seed(1)
    return [torch.randn(80, 3000, generator=g).clamp(-1.5, 1.5) for _ in range(4)]


def param_fingerprint(model: nn.Module) -> dict:
    return {n: [float(p.double().sum()), float(p.double().abs().sum())] for n, p in model.state_dict().items()}


def make_config1(R) -> None:
    torch.manual_seed(0)
    model = R["models"].WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865).eval()
    fp = param_fingerprint(model)
    mels = config1_inputs()
    enc_bm = R["EncoderBlockManager"](4, 6, 64, 16, 512, dtype=torch.float32, device="cpu")
    dec_bm = R["BlockManager"](4, 6, 64, 16, 64, dtype=torch.float32, device="cpu")
    sched = R["Scheduler"](model, R["DualCacheManager"](enc_bm, dec_bm), R["MemoryGuard"](), max_batch_size=4,
                           device="cpu", eos_token_id=-1, cache_cross_kv=True, batch_encoder=True)
    prompt = torch.tensor([R["PREFIX"]])
    for m in mels:
        sched.submit(m, prompt_token_ids=prompt, max_new_tokens=64, eos_token_id=-1)
    t0 = time.perf_counter()
    done = sorted(sched.run_until_done(), key=lambda r: r.id)
    dt = time.perf_counter() - t0
    out = dict(
        description="BASELINE config 1 run through the reference eager scheduler on CPU (fp32)",
        model="WhisperClassSpeechEncoderDecoderModel(4, 4, 6, 384, 80, 51865), torch.manual_seed(0)",
        mels="g = torch.Generator().manual_seed(1); 4 x torch.randn(80, 3000, generator=g).clamp(-1.5, 1.5)",
        prompt=list(R["PREFIX"]), max_new_tokens=64, eos_token_id=-1,
        tokens=[r.generated_tokens for r in done], wall_s=dt,
        mel_md5=[hashlib.md5(m.numpy().tobytes()).hexdigest() for m in mels],
        param_fingerprint=fp, torch_version=torch.__version__)
    (HERE / "config1_tokens.json").write_text(json.dumps(out, indent=1))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    torch.set_num_threads(8)
    R = _import_reference(a.reference)
    steps = dict(paged=make_paged_attn, cross=make_cross_attn, kv=make_kv_write, gather=make_block_gather,
                 proj=make_cross_kv_project, config1=make_config1)
    for name, fn in steps.items():
        if a.only and name not in a.only.split(","):
            continue
        t0 = time.perf_counter()
        fn(R)
        print(f"{name}: {time.perf_counter() - t0:.1f}s")


if __name__ == "__main__":
    main()
