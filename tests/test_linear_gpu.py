"""The small-batch tcgen05 Linear (spd_linear, through the C ABI) against a plain PyTorch
fp32 computation of the same layer: y = act(x @ w.T + b).

Shapes are the decode step's layers at Whisper-small (d 768) and large-v3 (d 1280)
dimensions: packed q|k|v (three output planes), the d x d projections, the MLP with and
without its GELU, and the vocabulary head (N not a multiple of the 128-feature tile).
Batches of 1, 7, 33 and 64 rows cover the X tile's zero fill.  The cluster split of K
is exercised by the small-N layers (K split 4 or 8 ways) and the unsplit head.

Tolerance: the kernel accumulates in fp32 and rounds once to fp16/bf16, so it is compared
with the fp32 result rounded to the output dtype: max-abs <= 2e-3 plus one output ulp of
|ref| (the projection GEMM's bar)."""
import pytest
import torch
import torch.nn.functional as F

from speech_serving import _native as N
from speech_serving import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(out, ref_f32, dtype):
    ref_r = ref_f32.to(dtype).float()
    ulp = 2.0 ** (-7 if dtype == torch.bfloat16 else -10)
    bound = 2e-3 + ulp * ref_f32.abs()
    diff = (out.float() - ref_r).abs()
    return bool((diff <= bound).all()), float(diff.max())


SHAPES = [  # (N, K, groups, gelu)
    (3 * 768, 768, 3, False),     # Whisper-small q|k|v
    (768, 768, 1, False),         # out-proj / cross q / cross out
    (3072, 768, 1, True),         # fc1 + GELU
    (768, 3072, 1, False),        # fc2
    (3 * 1280, 1280, 3, False),   # large-v3 q|k|v
    (1280, 5120, 1, False),       # large-v3 fc2
    (5120, 1280, 1, True),        # large-v3 fc1 + GELU
    (51866, 1280, 1, False),      # large-v3 head
]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M", [1, 7, 33, 64])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"N{s[0]}_K{s[1]}_g{s[2]}{'_gelu' if s[3] else ''}")
def test_linear_matches_torch_fp32(dtype, M, shape):
    Nf, K, groups, gelu = shape
    g = torch.Generator(device=DEV).manual_seed(Nf * 7 + K + M)
    x = torch.randn(M, K, generator=g, device=DEV).to(dtype)
    w = (torch.randn(Nf, K, generator=g, device=DEV) * K ** -0.5).to(dtype)
    b = (torch.randn(Nf, generator=g, device=DEV) * 0.1).to(dtype)
    ref = x.float() @ w.float().T + b.float()
    if gelu:
        ref = F.gelu(ref)
    out = ops.linear(x, w, b, gelu=gelu, groups=groups)
    got = out if groups == 1 else torch.cat(list(out), dim=1)  # planes back to [M, N]
    ok, err = _close(got, ref, dtype)
    assert ok, err


def test_linear_without_bias_and_repeat_is_bit_identical():
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(64, 768, generator=g, device=DEV).half()
    w = (torch.randn(768, 768, generator=g, device=DEV) * 0.03).half()
    a = ops.linear(x, w)
    b = ops.linear(x, w)
    assert torch.equal(a, b)
    ok, err = _close(a, x.float() @ w.float().T, torch.float16)
    assert ok, err


def test_linear_refuses_unsupported_shapes():
    x = torch.zeros(65, 768, device=DEV, dtype=torch.float16)
    w = torch.zeros(768, 768, device=DEV, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="M <= 64"):
        ops.linear(x, w)
    with pytest.raises(RuntimeError, match="multiple of 64"):
        ops.linear(torch.zeros(4, 100, device=DEV, dtype=torch.float16),
                   torch.zeros(768, 100, device=DEV, dtype=torch.float16))
    with pytest.raises(RuntimeError, match="F16/BF16"):
        ops.linear(torch.zeros(4, 64, device=DEV), torch.zeros(64, 64, device=DEV))
    assert N.load().spd_get_last_error(None, 0) == N.SPD_ERR_UNSUPPORTED
