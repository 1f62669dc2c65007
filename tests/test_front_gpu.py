"""GPU parity of the spectrogram front-end kernels against PyTorch FP32
statements of the reference's formulas (front.py:19-43, 80-87;
kernels/primitives.py:153-187; kernels/native.py:141-163).

BF16 outputs must be within one BF16 ulp of the reference formula (two ulps
plus 2^-7 after SiLU, whose input is already a rounded BF16 value); the masked
rows must be exactly zero.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from trifusion_b200.front import CNNStage  # noqa: E402
from trifusion_b200.kernels import RMSNorm  # noqa: E402
from trifusion_b200.kernels.buffers import front_norm, front_residual, front_stem  # noqa: E402
from trifusion_b200.kernels.native import bands  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16
ULP = 2.0 ** -7


def close_bf16(y, ref, ulps=1, atol=1e-30):
    y, ref = y.float(), ref.float()
    assert torch.all((y - ref).abs() <= ulps * ULP * ref.abs() + atol), (y - ref).abs().max()


def seeded(shape, seed, scale=1.0, dtype=BF):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(DEV)


SHAPES = [(4, 32, 401, 129), (4, 64, 201, 65), (3, 128, 101, 33)]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("silu", [True, False])
def test_front_norm_matches_formula(shape, silu):
    b, c, t, f = shape
    x = seeded(shape, 1, scale=3.0).contiguous(memory_format=torch.channels_last)
    lengths = torch.tensor([t, t // 2, 1, 0][:b], device=DEV)
    norm = RMSNorm(c).to(DEV)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.02 * torch.randn(c, generator=torch.Generator().manual_seed(2)))
    y = front_norm(x, lengths, norm, silu=silu)
    assert y.shape == x.shape and y.dtype == BF
    valid = (torch.arange(t, device=DEV)[None, :] < lengths[:, None])[:, None, :, None]
    rows = x.masked_fill(~valid, 0).permute(0, 2, 3, 1).float()
    ref = (rows * torch.rsqrt(rows.pow(2).mean(-1, keepdim=True) + norm.eps) * norm.weight).to(BF)
    if silu:
        ref = F.silu(ref.float()).to(BF)
    ref = ref.permute(0, 3, 1, 2)
    if silu:
        # The SiLU input is itself a rounded BF16 value: a last-bit difference in
        # rsqrt can move it by one BF16 ulp, which SiLU carries to its output.
        close_bf16(y, ref, ulps=2, atol=ULP)
    else:
        close_bf16(y, ref)
    assert (y.masked_select(~valid.expand_as(y)) == 0).all()


@pytest.mark.parametrize("shape", SHAPES)
def test_front_residual_matches_formula(shape):
    b, c, t, f = shape
    h = seeded(shape, 3).contiguous(memory_format=torch.channels_last)
    skip = seeded(shape, 4).contiguous(memory_format=torch.channels_last)
    lengths = torch.tensor([t, t // 3, 1, 0][:b], device=DEV)
    y = front_residual(h, skip, lengths)
    valid = (torch.arange(t, device=DEV)[None, :] < lengths[:, None])[:, None, :, None]
    ref = F.silu((h + skip).float()).to(BF).masked_fill(~valid, 0)
    close_bf16(y, ref)
    assert (y.masked_select(~valid.expand_as(y)) == 0).all()


@pytest.mark.parametrize("shape", SHAPES + [(2, 16, 7, 8), (2, 16, 7, 9)])
def test_bands_match_adaptive_pool(shape):
    x = seeded(shape, 5).contiguous(memory_format=torch.channels_last)
    y = bands(x)
    ref = F.adaptive_avg_pool2d(x.float(), (shape[2], 8)).permute(0, 2, 3, 1).to(BF)
    assert y.shape == (shape[0], shape[2], 8, shape[1])
    close_bf16(y, ref)


def test_cnn_stage_kernel_path_matches_reference_path():
    torch.manual_seed(0)
    stage = CNNStage(32, 64, 2, "l4").to(DEV).to(memory_format=torch.channels_last)
    ref_stage = CNNStage(32, 64, 2, "reference").to(DEV)
    ref_stage.load_state_dict(stage.state_dict())
    x = seeded((3, 32, 161, 129), 6).float()
    lengths = torch.tensor([161, 90, 7], device=DEV)
    with torch.inference_mode():
        y = stage(x, lengths)
        ref = ref_stage(x, lengths)
    assert y.shape == ref.shape
    torch.testing.assert_close(y.float(), ref.float(), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("shape,lens", [((4, 401, 257), [401, 200, 1, 0]), ((2, 37, 33), [37, 5])])
def test_front_stem_matches_cudnn_stage(shape, lens):
    """The fused first-stage stem against cuDNN's BF16 convolutions followed by the
    front-norm kernel: the skip is one exact product per channel (bit-exact); the
    3x3 sums may round differently from cuDNN's (two BF16 ulps after norm + SiLU)."""
    b, t, f = shape
    torch.manual_seed(3)
    stage = CNNStage(1, 32, 1, "l4").to(DEV)
    with torch.no_grad():
        stage.norm1.weight.copy_(1 + 0.02 * torch.randn(32))
    x = seeded((b, 1, t, f), 4, scale=4.0, dtype=torch.float32)
    lengths = torch.tensor(lens, device=DEV)
    valid = (torch.arange(t, device=DEV)[None, :] < lengths[:, None])[:, None, :, None]
    x = x.masked_fill(~valid, 0)
    with torch.no_grad(), torch.autocast("cuda", dtype=BF):
        h, s = front_stem(x, lengths, stage.conv1, stage.skip, stage.norm1)
        x_cl = x.contiguous(memory_format=torch.channels_last)
        h_ref = front_norm(stage.conv1(x_cl), lengths, stage.norm1, silu=True)
        s_ref = stage.skip(x_cl)
    assert h.shape == h_ref.shape and h.dtype == BF and s.dtype == BF
    assert torch.equal(s.float(), s_ref.float())
    close_bf16(h, h_ref, ulps=2, atol=ULP * 2.0 ** -6)
    assert (h.permute(0, 2, 3, 1)[~valid[:, 0, :, 0]] == 0).all()


@pytest.mark.parametrize("cin,cout,t,f", [(32, 64, 401, 129), (64, 128, 201, 65)])
def test_strided_skip_as_gemm(cin, cout, t, f):
    """The stride-2 stages' 1x1 skip convolution as a gather of the subsampled
    channels-last rows and one BF16 GEMM: equal to cuDNN's convolution up to FP32
    summation order (one BF16 ulp)."""
    from trifusion_b200.front import CNNStage

    torch.manual_seed(3)
    st = CNNStage(cin, cout, 2, "l4").cuda().to(torch.bfloat16).to(memory_format=torch.channels_last)
    x = torch.randn(2, cin, t, f, device="cuda").to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        ref, got = st.skip(x), st._skip_rows(x)
    assert got.shape == ref.shape and got.is_contiguous(memory_format=torch.channels_last)
    torch.testing.assert_close(got.float(), ref.float(), atol=1e-2, rtol=2 ** -7)
