"""Op (4): the tcgen05 cross-KV projection GEMM, called through the C ABI, against the
golden vectors made by the reference's PretrainedWhisperModel.encode
(speech_serving/models.py:554-561) and against a plain PyTorch fp32 GEMM.

Tolerance: the kernel accumulates in fp32 and rounds once to fp16/bf16, so it is
compared with the fp32 result rounded to the output dtype: max-abs <= 2e-3 for outputs
of magnitude <~ 1 (plus one output ulp where |ref| is larger)."""
import numpy as np
import pytest
import torch

from oracle import attention_oracle as O
from speech_serving import ops

pytestmark = pytest.mark.gpu


def _close(out, ref_f32, dtype):
    ref_r = ref_f32.to(dtype).float()
    ulp = 2.0 ** (-7 if dtype == torch.bfloat16 else -10)  # one output ulp relative to |ref|
    bound = 2e-3 + ulp * ref_f32.abs()
    diff = (out.float() - ref_r).abs()
    return bool((diff <= bound).all()), float(diff.max())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_projection_matches_reference_golden(golden_dir, dtype):
    g = np.load(golden_dir / "cross_kv_project_ref.npz")
    L = len([k for k in g.files if k.startswith("wk")])
    H, D = g["k0"].shape[1], g["k0"].shape[3]
    enc = torch.from_numpy(g["enc_out"]).to(dtype).cuda()
    ws = torch.cat([torch.from_numpy(g[f"{p}{l}"]) for l in range(L) for p in ("wk", "wv")]).to(dtype).cuda()
    bs = torch.cat([torch.zeros(H * D) if p == "k" else torch.from_numpy(g[f"bv{l}"])
                    for l in range(L) for p in ("k", "v")]).to(dtype).cuda()
    B, T, d = enc.shape
    out = torch.full((B, L, 2, H, T, D), float("nan"), dtype=dtype, device="cuda")
    ops.cross_kv_project(enc.contiguous(), ws.contiguous(), bs.contiguous(), out)
    # oracle on the dtype-rounded inputs
    res = O.cross_kv_project(enc.float().cpu().numpy(),
                             [ws[(2 * l) * H * D:(2 * l + 1) * H * D].float().cpu().numpy() for l in range(L)],
                             [ws[(2 * l + 1) * H * D:(2 * l + 2) * H * D].float().cpu().numpy() for l in range(L)],
                             [bs[(2 * l + 1) * H * D:(2 * l + 2) * H * D].float().cpu().numpy() for l in range(L)], H)
    for l in range(L):
        for kv in range(2):
            ok, err = _close(out[:, l, kv].cpu(), torch.from_numpy(res[l][kv]), dtype)
            assert ok, (l, kv, err)
            # and the reference's own fp32 output, within input-rounding distance
            ref = torch.from_numpy(g[f"{'kv'[kv]}{l}"])
            assert float((out[:, l, kv].float().cpu() - ref).abs().max()) < 2e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_projection_whisper_small_shape_vs_torch(dtype):
    """Whisper-small handoff: d_model 768, 12 heads x 64, here 3 layers (N = 4608), two
    requests of 1500 positions scattered into slots 3 and 1 of a 4-slot buffer."""
    torch.manual_seed(0)
    B, T, d, L, H, D, S = 2, 1500, 768, 3, 12, 64, 4
    enc = torch.randn(B, T, d, device="cuda").to(dtype)
    w = (torch.randn(L * 2 * H * D, d, device="cuda") * 0.02).to(dtype)
    bias = (torch.randn(L * 2 * H * D, device="cuda") * 0.1).to(dtype)
    out = torch.full((S, L, 2, H, T, D), 7.0, dtype=dtype, device="cuda")
    slots = torch.tensor([3, 1], dtype=torch.int32, device="cuda")
    ops.cross_kv_project(enc, w, bias, out, slot_ids=slots)
    ref = enc.float().reshape(B * T, d) @ w.float().t() + bias.float()
    ref = ref.view(B, T, L, 2, H, D).permute(0, 2, 3, 4, 1, 5)  # [B, L, 2, H, T, D]
    for i, s in enumerate([3, 1]):
        ok, err = _close(out[s], ref[i], dtype)
        assert ok, err
    assert bool((out[0] == 7.0).all()) and bool((out[2] == 7.0).all())


@pytest.mark.parametrize("d", [128, 1024])
def test_projection_partial_tiles_and_graph_capture(d):
    """N = 1*2*5*64 = 640 (not a multiple of the 256-wide tile), T = 300 < T_out; d_model
    128 runs the one-CTA form, 1024 the CTA-pair form."""
    torch.manual_seed(1)
    B, T, L, H, D, T_out = 3, 300, 1, 5, 64, 320
    dtype = torch.float16
    enc = torch.randn(B, T, d, device="cuda").to(dtype)
    w = (torch.randn(L * 2 * H * D, d, device="cuda") * d ** -0.5).to(dtype)
    out = torch.zeros((B, L, 2, H, T_out, D), dtype=dtype, device="cuda")
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.cross_kv_project(enc, w, None, out)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        ops.cross_kv_project(enc, w, None, out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    ref = (enc.float().reshape(B * T, d) @ w.float().t()).view(B, T, L, 2, H, D).permute(0, 2, 3, 4, 1, 5)
    ok, err = _close(out[:, :, :, :, :T], ref, dtype)
    assert ok, err
    assert not out[:, :, :, :, T:].any()


@pytest.mark.parametrize("B,T,d,L,H", [(1, 100, 256, 1, 4), (1, 200, 1280, 2, 20), (3, 1500, 1280, 1, 20)])
def test_projection_row_tails_and_large_v3_width(B, T, d, L, H):
    """Row counts that leave the second half of a 256-row tile partly or wholly past M
    (M = 100, 200, 4500), and large-v3's d_model (K = 1280: 20 K slices per tile)."""
    torch.manual_seed(B * 7 + T)
    D, dtype = 64, torch.bfloat16
    enc = torch.randn(B, T, d, device="cuda").to(dtype)
    w = (torch.randn(L * 2 * H * D, d, device="cuda") * d ** -0.5).to(dtype)
    bias = (torch.randn(L * 2 * H * D, device="cuda") * 0.1).to(dtype)
    out = torch.full((B, L, 2, H, T, D), float("nan"), dtype=dtype, device="cuda")
    ops.cross_kv_project(enc, w, bias, out)
    ref = (enc.float().reshape(B * T, d) @ w.float().t() + bias.float()).view(B, T, L, 2, H, D)
    ok, err = _close(out, ref.permute(0, 2, 3, 4, 1, 5), dtype)
    assert ok, err
