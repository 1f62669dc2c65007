"""GPU parity of the satellite operators (rows A6-A13 around the recurrence).

Each CUDA operator is called through its drop-in Python wrapper (which calls
the C ABI) and compared with the reference's own outputs (golden vectors from
``tests/golden/satellites.npz``) and with the CPU oracle at model sizes.
Index and copy operators must match bit for bit; arithmetic ones within one
BF16 ulp (BF16 outputs) or 2e-6 relative (FP32 outputs).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import mamba_oracle as O

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from trifusion_b200.kernels import gated_branches, gated_concat, reverse_valid, swiglu  # noqa: E402
from trifusion_b200.kernels import native  # noqa: E402
from trifusion_b200.kernels.buffers import Pool4, mamba_controls, mask_buffer, masked_add  # noqa: E402

DEV = "cuda"
BF = torch.bfloat16
GOLDEN = Path(__file__).resolve().parent / "golden" / "satellites.npz"
BF16_ULP = 2.0 ** -7  # relative spacing bound of BF16 values


@pytest.fixture(scope="module")
def sat():
    return dict(np.load(GOLDEN))


def gpu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t.to(dtype) if dtype is not None else t


def host(t):
    return t.float().cpu().numpy()


def within_bf16_ulp(y, ref, ulps=1):
    return np.all(np.abs(y - ref) <= ulps * BF16_ULP * np.abs(ref) + 1e-30)


# ---------------------------------------------------------------- golden vectors

def test_rms_matches_reference_formula(sat):
    y = host(native.rms(gpu(sat["rms_x"], BF), gpu(sat["rms_w"])))
    assert within_bf16_ulp(y, sat["rms_torch"])
    assert (y != sat["rms_torch"]).mean() < 0.01


def test_mean_norm_matches_reference_kernel(sat):
    y = native.mean_norm(gpu(sat["mn_a"], BF), gpu(sat["mn_b"], BF), gpu(sat["mn_w"]))
    assert y.dtype == torch.float32
    np.testing.assert_allclose(host(y), sat["mean_norm_triton"], rtol=2e-6, atol=2e-6)


def test_evidence_norm_matches_reference_kernel(sat):
    y = native.evidence_norm(gpu(sat["ev_x"]), gpu(sat["ev_v"], BF), gpu(sat["ev_g"], BF),
                             gpu(sat["mn_w"]), gpu(sat["ev_mask"]))
    np.testing.assert_allclose(host(y), sat["evidence_norm_triton"], rtol=2e-6, atol=2e-6)


def test_controls_match_reference_kernel(sat):
    # Strided views of one projection row, as the model passes them.
    b, t, h = sat["ctl_a"].shape
    p = torch.zeros(b, t, 3 * h + 5, dtype=BF, device=DEV)
    p[..., :h] = gpu(sat["ctl_a"], BF)
    p[..., h:2 * h] = gpu(sat["ctl_ddt"], BF)
    adt, dt = mamba_controls(p[..., :h], p[..., h:2 * h], gpu(sat["ctl_bias"]), 1e-4)
    np.testing.assert_allclose(host(dt), sat["ctl_dt"], rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(host(adt), sat["ctl_adt"], rtol=2e-6, atol=1e-7)


def test_index_ops_bit_exact(sat):
    x, lengths = gpu(sat["x"], BF), gpu(sat["lengths"])
    mask = torch.arange(x.shape[1], device=DEV)[None, :] < lengths[:, None]
    assert np.array_equal(host(mask_buffer(x, mask)), sat["mask_triton"])
    assert np.array_equal(host(reverse_valid(x, lengths)), sat["reverse_torch"])
    assert np.array_equal(host(native.end_gather(x, lengths)), sat["end_torch"])


def test_swiglu_and_gate_match_reference(sat):
    y = host(swiglu(gpu(sat["sw_x"], BF)))
    assert within_bf16_ulp(y, sat["swiglu_torch"])
    assert (y != sat["swiglu_torch"]).mean() < 0.01
    y = host(gated_concat(gpu(sat["gate_x"], BF), gpu(sat["gate_g"], BF)))
    assert within_bf16_ulp(y, sat["gate_torch"])
    assert (y != sat["gate_torch"]).mean() < 0.01


def test_pool4_bit_exact_with_reference(sat):
    y = host(Pool4.apply(gpu(sat["x"], BF), gpu(sat["lengths"])))
    assert np.array_equal(y, sat["pool_torch"])


def test_masked_mean_matches_reference(sat):
    y = native.masked_mean(gpu(sat["x"], BF), gpu(sat["lengths"]))
    np.testing.assert_allclose(host(y), sat["masked_mean_torch"], rtol=1e-5, atol=1e-6)


# ---------------------------------------------------------------- model sizes

def seeded(shape, seed, scale=1.0, dtype=BF):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


LENGTHS = [200, 137, 1, 0, 64, 199, 3, 200]


@pytest.mark.parametrize("dtype", [BF, torch.float32])
def test_index_ops_model_size(dtype):
    b, t, d = len(LENGTHS), 200, 768
    x = seeded((b, t, d), 1, dtype=dtype)
    lengths = torch.tensor(LENGTHS)
    xd, ld = x.to(DEV), lengths.to(DEV)
    mask = torch.arange(t)[None, :] < lengths[:, None]
    bits = torch.int16 if dtype == BF else torch.int32
    xn = x.view(bits).numpy()
    got = mask_buffer(xd, mask.to(DEV)).cpu()
    assert np.array_equal(got.view(bits).numpy(), O.mask_rows(xn, LENGTHS))
    got = reverse_valid(xd, ld).cpu()
    assert np.array_equal(got.view(bits).numpy(), O.reverse_valid(xn, LENGTHS))
    # Reversing twice restores the valid prefix and keeps the tail zero.
    twice = reverse_valid(reverse_valid(xd, ld), ld)
    assert torch.equal(twice, mask_buffer(xd, mask.to(DEV)))


def test_index_ops_odd_row_sizes_and_views():
    # 3 BF16 per row (6 bytes): no 16/8/4-byte vectors fit; offset base pointer.
    b, t = 4, 33
    base = seeded((b * t * 3 + 1,), 2).to(DEV)
    x = base[1:].view(b, t, 3)  # base pointer 2 bytes past an allocation boundary
    lengths = torch.tensor([33, 0, 17, 1])
    mask = (torch.arange(t)[None, :] < lengths[:, None]).to(DEV)
    ref = O.mask_rows(x.cpu().view(torch.int16).numpy(), lengths.numpy())
    assert np.array_equal(mask_buffer(x, mask).cpu().view(torch.int16).numpy(), ref)
    ref = O.reverse_valid(x.cpu().view(torch.int16).numpy(), lengths.numpy())
    assert np.array_equal(reverse_valid(x, lengths.to(DEV)).cpu().view(torch.int16).numpy(), ref)
    end = native.end_gather(x, lengths.to(DEV)).cpu()
    # length 0 reads index -1 (the last row), as PyTorch indexing does
    assert torch.equal(end, x.cpu()[torch.arange(b), lengths - 1])


@pytest.mark.parametrize("t", [200, 401, 3, 4])
def test_pool4_model_size_bit_exact(t):
    b, d = 8, 384
    x = seeded((b, t, d), 3)
    lengths = torch.tensor([min(v, t) for v in LENGTHS])
    y = Pool4.apply(x.to(DEV), lengths.to(DEV)).cpu().float().numpy()
    assert np.array_equal(y, O.pool4_f32(x.float().numpy(), lengths.numpy()))


@pytest.mark.parametrize("dtype", [BF, torch.float32])
@pytest.mark.parametrize("width", [128, 384, 1024, 36])
def test_rms_model_size(dtype, width):
    x = seeded((16, 101, width), 4, scale=3.0, dtype=dtype)
    w = 1 + 0.02 * torch.randn(width, generator=torch.Generator().manual_seed(5))
    y = native.rms(x.to(DEV), w.to(DEV)).cpu()
    assert y.dtype == dtype
    ref = O.rms(x.float().numpy(), w.numpy(), out_bf16=dtype == BF)
    if dtype == BF:
        assert within_bf16_ulp(y.float().numpy(), ref)
    else:
        np.testing.assert_allclose(y.numpy(), ref, rtol=2e-6, atol=1e-6)


def test_norm_family_model_size():
    b, t, d = 16, 101, 384
    lengths = torch.tensor([101, 50, 1, 0] * 4)
    mask = torch.arange(t)[None, :] < lengths[:, None]
    x = seeded((b, t, d), 6, dtype=torch.float32)
    v, g = seeded((b, t, d), 7), seeded((b, t, d), 8)
    w = 1 + 0.02 * torch.randn(d, generator=torch.Generator().manual_seed(9))
    y = native.evidence_norm(x.to(DEV), v.to(DEV), g.to(DEV), w.to(DEV), mask.to(DEV)).cpu().numpy()
    ref = O.evidence_norm(x.numpy(), v.float().numpy(), g.float().numpy(), w.numpy(), mask.numpy())
    np.testing.assert_allclose(y, ref, rtol=2e-6, atol=2e-6)
    a, c = seeded((b, t, d), 10), seeded((b, t, d), 11)
    y = native.mean_norm(a.to(DEV), c.to(DEV), w.to(DEV)).cpu().numpy()
    np.testing.assert_allclose(y, O.mean_norm(a.float().numpy(), c.float().numpy(), w.numpy()),
                               rtol=2e-6, atol=2e-6)


def test_swiglu_gate_model_size():
    x = seeded((16, 101, 2 * 1536), 12, scale=2.0)
    y = swiglu(x.to(DEV)).cpu().float().numpy()
    assert within_bf16_ulp(y, O.swiglu(x.float().numpy()))
    xg, g = seeded((16, 101, 3 * 384), 13), seeded((16, 101, 3), 14, scale=2.0)
    y = gated_concat(xg.to(DEV), g.to(DEV)).cpu().float().numpy()
    assert within_bf16_ulp(y, O.gated_concat(xg.float().numpy(), g.float().numpy()))
    # FP32 gate against BF16 branches (the model's Linear output under autocast may be either)
    y32 = gated_concat(xg.to(DEV), g.float().to(DEV)).cpu().float().numpy()
    assert np.array_equal(y32, y)


def test_controls_model_layout():
    # [B, T, 1860] in_proj output of a dim-384 block: a and ddt are 12-wide views.
    b, t, h = 16, 200, 12
    p = seeded((b, t, 1860), 15, scale=4.0).to(DEV)
    ddt, a = p[..., 1792:1804], p[..., 1804:1816]
    bias = torch.full((h,), -4.0) + torch.randn(h, generator=torch.Generator().manual_seed(16))
    adt, dt = mamba_controls(a, ddt, bias.to(DEV), 1e-4)
    radt, rdt = O.mamba_controls(a.float().cpu().numpy(), ddt.float().cpu().numpy(), bias.numpy())
    np.testing.assert_allclose(dt.cpu().numpy(), rdt, rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(adt.cpu().numpy(), radt, rtol=2e-6, atol=1e-7)


def test_masked_mean_and_end_gather_model_size():
    b, t, d = 16, 101, 384
    lengths = torch.tensor([101, 50, 1, 7] * 4)
    x = seeded((b, t, d), 17)
    y = native.masked_mean(x.to(DEV), lengths.to(DEV)).cpu().numpy()
    np.testing.assert_allclose(y, O.masked_mean(x.float().numpy(), lengths.numpy()), rtol=1e-5, atol=1e-6)
    e = native.end_gather(x.to(DEV), lengths.to(DEV)).cpu()
    assert torch.equal(e, x[torch.arange(b), lengths - 1])


def test_empty_inputs():
    x = torch.zeros(0, 5, 8, dtype=BF, device=DEV)
    lengths = torch.zeros(0, dtype=torch.int64, device=DEV)
    assert reverse_valid(x, lengths).shape == x.shape
    assert Pool4.apply(x, lengths).shape == (0, 2, 8)
    assert native.rms(torch.zeros(0, 128, device=DEV), torch.ones(128, device=DEV)).shape == (0, 128)
    assert swiglu(torch.zeros(0, 16, dtype=BF, device=DEV)).shape == (0, 8)


def test_capture_in_cuda_graph_matches_eager():
    b, t, d = 4, 64, 384
    x = seeded((b, t, d), 18).to(DEV)
    lengths = torch.tensor([64, 30, 1, 0], device=DEV)
    w = torch.ones(d, device=DEV)

    def step():
        r = reverse_valid(x, lengths)
        return native.mean_norm(r, x, w), Pool4.apply(r, lengths), swiglu(torch.cat((x, r), -1))

    eager = step()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = step()
    graph.replay()
    torch.cuda.synchronize()
    for a, c in zip(eager, captured):
        assert torch.equal(a, c)


@pytest.mark.parametrize("dtype", [BF, torch.float32])
@pytest.mark.parametrize("taps,width", [(7, 384), (3, 1152)])
def test_depthwise_masked_matches_conv1d(dtype, taps, width):
    from trifusion_b200.kernels.buffers import depthwise_masked

    b, t = 4, 101
    x = seeded((b, t, width), 21, dtype=dtype).to(DEV)
    torch.manual_seed(22)
    conv = torch.nn.Conv1d(width, width, taps, padding=taps // 2, groups=width).to(DEV).to(BF)
    lengths = torch.tensor([101, 50, 1, 0], device=DEV)
    y = depthwise_masked(x, conv, lengths)
    assert y.dtype == BF and y.shape == (b, t, width)
    # The reference rounds the input to BF16 (the autocast type) and sums in FP32.
    ref = torch.nn.functional.conv1d(x.to(BF).float().transpose(1, 2), conv.weight.float(), conv.bias.float(),
                                     padding=taps // 2, groups=width).transpose(1, 2)
    valid = (torch.arange(t, device=DEV)[None, :] < lengths[:, None])[..., None]
    ref = torch.where(valid, ref, torch.zeros((), device=DEV)).to(BF)
    y32, r32 = y.float(), ref.float()
    assert torch.all((y32 - r32).abs() <= BF16_ULP * r32.abs() + 1e-5), (y32 - r32).abs().max()
    assert (y.masked_select(~valid.expand_as(y)) == 0).all()


@pytest.mark.parametrize("taps,width", [(7, 384), (3, 64)])
def test_glu_depthwise_equals_glu_then_depthwise(taps, width):
    """The GLU formed inside the depthwise pass equals PyTorch's glu followed by the
    depthwise kernel, bit for bit (model.py:122-124)."""
    from trifusion_b200.kernels.buffers import depthwise_masked, glu_depthwise

    b, t = 3, 77
    u = (seeded((b, t, 2 * width), 31) * 3).to(BF).to(DEV)
    torch.manual_seed(32)
    conv = torch.nn.Conv1d(width, width, taps, padding=taps // 2, groups=width).to(DEV).to(BF)
    lengths = torch.tensor([77, 40, 0], device=DEV)
    fused = glu_depthwise(u, conv, lengths)
    assert torch.equal(fused, depthwise_masked(torch.nn.functional.glu(u, dim=-1), conv, lengths))


def test_rotary_qkv_bit_exact_with_formula():
    from trifusion_b200.kernels.buffers import RotaryQKV
    from trifusion_b200.masking import rotary_table
    from trifusion_b200.model import rope

    b, t, heads, d = 4, 26, 6, 64
    x = seeded((b, t, 3 * heads * d), 23, scale=2.0).to(DEV)
    cos, sin = rotary_table(t, d, DEV)
    y = RotaryQKV.apply(x, cos, sin, heads, torch.float32)
    q, k, v = x.view(b, t, 3, heads, d).permute(2, 0, 3, 1, 4).unbind(0)
    assert torch.equal(y[0], rope(q, cos, sin).float())
    assert torch.equal(y[1], rope(k, cos, sin).float())
    assert torch.equal(y[2], v.float())
    assert torch.equal(RotaryQKV.apply(x, cos, sin, heads), y.to(BF))


def test_interpolate_bit_exact_with_formula():
    from trifusion_b200.kernels.native import interpolate
    from trifusion_b200.masking import Grids

    lengths = torch.tensor([101, 57, 1, 9], device=DEV)
    grids = Grids.make(lengths, 101, 64)
    low = seeded((4, 26, 384), 24).to(DEV)
    y = interpolate(low, grids)
    ref = Grids.make(lengths, 101, 64, native_kernels=False).interpolate(low)
    assert torch.equal(y, ref)


@pytest.mark.parametrize("b_dtype", [torch.bfloat16, torch.float32])
def test_masked_add_is_exact(b_dtype):
    """mask(a + b) in one pass equals PyTorch's FP32 add (b promoted) then the row mask, bit for bit."""
    g = torch.Generator().manual_seed(5)
    a = torch.randn(4, 37, 384, generator=g).to(DEV)
    bb = torch.randn(4, 37, 384, generator=g).to(b_dtype).to(DEV)
    lengths = torch.tensor([37, 20, 1, 0], device=DEV)
    mask = torch.arange(37, device=DEV)[None, :] < lengths[:, None]
    y = masked_add(a, bb, mask)
    ref = torch.where(mask[..., None], a + bb, torch.zeros((), device=DEV))
    assert y.dtype == torch.float32 and torch.equal(y, ref)


def test_bf16_outputs_equal_cast_fp32_outputs():
    """The BF16-output forms (norms feeding a projection, depthwise plus its input) equal
    the FP32 forms followed by the autocast cast, bit for bit."""
    from trifusion_b200.kernels.buffers import depthwise_masked

    g = torch.Generator().manual_seed(9)
    x = (torch.randn(3, 41, 384, generator=g) * 2).to(DEV)
    w = (1 + 0.05 * torch.randn(384, generator=g)).to(DEV)
    assert torch.equal(native.rms(x, w, 1e-5, out_dtype=torch.bfloat16), native.rms(x, w, 1e-5).to(torch.bfloat16))
    value = torch.randn(3, 41, 384, generator=g).to(torch.bfloat16).to(DEV)
    gate = torch.randn(3, 41, 384, generator=g).to(torch.bfloat16).to(DEV)
    lengths = torch.tensor([41, 17, 0], device=DEV)
    mask = torch.arange(41, device=DEV)[None, :] < lengths[:, None]
    e32 = native.evidence_norm(x, value, gate, w, mask, 1e-5)
    e16 = native.evidence_norm(x, value, gate, w, mask, 1e-5, out_dtype=torch.bfloat16)
    assert e16.dtype == torch.bfloat16 and torch.equal(e16, e32.to(torch.bfloat16))
    conv = torch.nn.Conv1d(384, 384, 3, padding=1, groups=384).to(DEV)
    xm = torch.where(mask[..., None], x, 0.0)
    fused = depthwise_masked(xm, conv, lengths, residual=True)
    assert torch.equal(fused, (xm + depthwise_masked(xm, conv, lengths).float()).to(torch.bfloat16))


def test_pool4_bf16_and_rms_silu_exact():
    """Pool4 into BF16 equals the FP32 means cast once; rms_silu equals PyTorch's silu
    applied to the norm's BF16 output, bit for bit."""
    import torch.nn.functional as F

    g = torch.Generator().manual_seed(13)
    x = (torch.randn(4, 101, 384, generator=g) * 1.5).to(DEV)
    lengths = torch.tensor([101, 57, 3, 0], device=DEV)
    assert torch.equal(Pool4.apply(x, lengths, torch.bfloat16), Pool4.apply(x, lengths).to(torch.bfloat16))
    h = (torch.randn(4, 101, 384, generator=g) * 3).to(torch.bfloat16).to(DEV)
    w = (1 + 0.05 * torch.randn(384, generator=g)).to(DEV)
    assert torch.equal(native.rms_silu(h, w, 1e-5), F.silu(native.rms(h, w, 1e-5)))


def test_add_rms_exact():
    """x + a and its RMSNorm in one pass equal PyTorch's FP32 add then the norm kernel, bit for bit."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn(3, 57, 384, generator=g).to(DEV)
    a = torch.randn(3, 57, 384, generator=g).to(torch.bfloat16).to(DEV)
    w = (1 + 0.05 * torch.randn(384, generator=g)).to(DEV)
    total, y = native.add_rms(x, a, w, 1e-5)
    ref_total = x + a
    assert torch.equal(total, ref_total)
    assert torch.equal(y, native.rms(ref_total, w, 1e-5, out_dtype=torch.bfloat16))


@pytest.mark.parametrize("width", [384, 30])
def test_norms_into_concatenated_rows_and_branch_gate_exact(width):
    """The block's concatenations written in place: cn/an norms into slices of e_down's
    and the gate's input rows, mean_norm's BF16 copy, and the branch gate read from the
    three pieces, each equal bit for bit to the torch.cat forms (width 30: scalar path)."""
    g = torch.Generator().manual_seed(23)
    b, t, d = 2, 75, width
    lc = torch.randn(b, t, d, generator=g).to(torch.bfloat16).to(DEV)
    at = torch.randn(b, t, d, generator=g).to(torch.bfloat16).to(DEV)
    mf = torch.randn(b, t, d, generator=g).to(torch.bfloat16).to(DEV)
    mb = torch.randn(b, t, d, generator=g).to(torch.bfloat16).to(DEV)
    wc, wa, wm = [(1 + 0.05 * torch.randn(d, generator=g)).to(DEV) for _ in range(3)]
    gate = torch.randn(b, t, 3, generator=g).to(torch.bfloat16).to(DEV)
    e_in = torch.full((b, t, 2 * d), float("nan"), dtype=torch.bfloat16, device=DEV)
    s16 = torch.full((b, t, 3 * d), float("nan"), dtype=torch.bfloat16, device=DEV)
    cn = native.rms_into(lc, wc, 1e-5, e_in[..., :d], s16[..., :d])
    an = native.rms_into(at, wa, 1e-5, e_in[..., d:], s16[..., 2 * d:])
    mn = native.mean_norm(mf, mb, wm, 1e-5, copy_to=s16[..., d:2 * d])
    rc, ra = native.rms(lc, wc, 1e-5), native.rms(at, wa, 1e-5)
    rm = native.mean_norm(mf, mb, wm, 1e-5)
    assert torch.equal(mn, rm)
    assert torch.equal(e_in, torch.cat((rc, ra), -1))
    s = torch.cat((rc, rm, ra), -1)
    assert torch.equal(s16, s.to(torch.bfloat16))
    assert torch.equal(gated_branches(cn, mn, an, gate), gated_concat(s, gate))
    f32 = torch.empty(b, t, 2 * d, device=DEV)
    native.rms_into(lc, wc, 1e-5, f32[..., d:])
    assert torch.equal(f32[..., d:], native.rms(lc, wc, 1e-5, out_dtype=torch.float32))


def test_gate_projection_and_branch_gate_in_one_pass():
    """The gate's three-output projection computed per row (FP32 sums) is within one
    BF16 ulp of the FP32 projection rounded once, and the gated row equals the branch
    gate applied with those gate values, bit for bit. (cuBLAS's BF16 GEMM for N = 3
    may reduce split-K partial sums in BF16, PyTorch's default
    allow_bf16_reduced_precision_reduction, so it is compared more loosely.)"""
    from trifusion_b200.kernels import gate_branches

    g = torch.Generator().manual_seed(29)
    b, t, d = 3, 91, 384
    s16 = torch.randn(b, t, 3 * d, generator=g).to(torch.bfloat16).to(DEV)
    mn = torch.randn(b, t, d, generator=g).to(DEV)
    w = (0.05 * torch.randn(3, 3 * d, generator=g)).to(torch.bfloat16).to(DEV)
    bias = torch.randn(3, generator=g).to(torch.bfloat16).to(DEV)
    gate = torch.empty(b, t, 3, dtype=torch.bfloat16, device=DEV)
    v = gate_branches(s16, mn, w, bias, gate_out=gate)
    ref = torch.nn.functional.linear(s16.float(), w.float(), bias.float()).to(torch.bfloat16)
    ulp = torch.finfo(torch.bfloat16).eps * ref.float().abs().clamp_min(2.0 ** -126)
    assert ((gate.float() - ref.float()).abs() <= ulp * 1.01 + 1e-5).all()  # 1 ulp; near-cancelling sums aside
    assert torch.equal(v, gated_branches(s16[..., :d], mn, s16[..., 2 * d:], gate))
    # without gate_out and bias, on a slice of a wider row buffer
    wide = torch.zeros(b, t, 3 * d + 8, dtype=torch.bfloat16, device=DEV)
    wide[..., 4:4 + 3 * d] = s16
    gate2 = torch.empty_like(gate)
    v2 = gate_branches(wide[..., 4:4 + 3 * d], mn, w, gate_out=gate2)
    ref2 = torch.nn.functional.linear(s16.float(), w.float()).to(torch.bfloat16)
    ulp2 = torch.finfo(torch.bfloat16).eps * ref2.float().abs().clamp_min(2.0 ** -126)
    assert ((gate2.float() - ref2.float()).abs() <= ulp2 * 1.01 + 1e-5).all()
    assert torch.equal(v2, gated_branches(s16[..., :d], mn, s16[..., 2 * d:], gate2))


def test_stacked_in_proj_matches_separate_projections():
    """Both directions' in_proj as one GEMM over zero-padded, stacked weights: the
    views equal the separate projections to BF16 rounding, and their rows are
    16-byte aligned."""
    from types import SimpleNamespace

    from trifusion_b200.mamba import projections

    g = torch.Generator().manual_seed(31)
    mods = [SimpleNamespace(in_proj=torch.nn.Linear(384, 1860, bias=False).to(DEV)) for _ in range(2)]
    u = torch.randn(4, 77, 384, generator=g).to(torch.bfloat16).to(DEV)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        pf, pb = projections(mods, u)
        rf, rb = mods[0].in_proj(u), mods[1].in_proj(u)
    assert pf.shape == rf.shape and pf.stride(-2) == 2 * 1864 and pf.stride(-2) * 2 % 16 == 0
    for got, ref in ((pf, rf), (pb, rb)):
        assert got.dtype == ref.dtype == torch.bfloat16
        torch.testing.assert_close(got.float(), ref.float(), atol=2e-2, rtol=1e-2)


def _query_read_f64(q, kv, lengths, keys_per_length):
    """FP64 restatement of decoder.py:26-30 on the same BF16 operands."""
    qd, kvd = q.double().cpu(), kv.double().cpu()
    b, t, _ = kvd.shape
    k = kvd[..., :256].view(b, t, 8, 32).permute(0, 2, 1, 3)
    v = kvd[..., 256:512].view(b, t, 8, 32).permute(0, 2, 1, 3)
    qh = qd.view(10, 8, 32).transpose(0, 1)
    s = torch.einsum("hid,bhjd->bhij", qh, k) / 32 ** 0.5
    valid = torch.arange(t)[None, :] < (lengths.cpu() * keys_per_length)[:, None]
    s = s.masked_fill(~valid[:, None, None, :], float("-inf"))
    h = torch.einsum("bhij,bhjd->bhid", s.softmax(-1), v)
    return h.transpose(1, 2).reshape(b, 10, 256)


@pytest.mark.parametrize("batch,time,kpl,lens", [(3, 200, 1, [200, 57, 1]), (2, 1608, 8, [201, 13]),
                                                  (2, 700, 1, [700, 256])])
def test_query_read_matches_float64_attention(batch, time, kpl, lens):
    """Split-key decoder attention: within one BF16 ulp of the FP64 softmax attention
    on the same BF16 operands, masked by lengths (8 keys per frame for the fine read),
    from contiguous and from pitched projection rows."""
    g = torch.Generator().manual_seed(37)
    q = (0.5 * torch.randn(10, 256, generator=g)).to(torch.bfloat16).to(DEV)
    wide = torch.randn(batch, time, 520, generator=g).to(torch.bfloat16).to(DEV)
    lengths = torch.tensor(lens, device=DEV)
    for kv in (wide[..., :512].contiguous(), wide[..., 8:520]):
        y = native.query_read(q, kv, lengths, kpl)
        ref = _query_read_f64(q, kv, lengths, kpl)
        err = (y.double().cpu() - ref).abs()
        assert (err <= 2.0 ** -7 * ref.abs() + 1e-6).all(), float(err.max())


@pytest.mark.parametrize("batch,low_time,lens", [(3, 50, [50, 17, 1]), (2, 130, [130, 33])])
def test_pooled_attention_matches_float64(batch, low_time, lens):
    """Rotary + FP32 masked attention over the pooled rows in one kernel: within one
    BF16 ulp of FP64 attention on the rotated BF16 q/k (the rotary kernel's output,
    itself bit-exact with the reference formula), keys masked by the lengths."""
    from trifusion_b200.kernels.buffers import RotaryQKV
    from trifusion_b200.masking import rotary_table

    heads = 6
    g = torch.Generator().manual_seed(41)
    qkv = torch.randn(batch, low_time, 3 * heads * 64, generator=g).to(torch.bfloat16).to(DEV)
    cos, sin = rotary_table(low_time, 64, DEV)
    lengths = torch.tensor(lens, device=DEV)
    y = native.pooled_attention(qkv, cos, sin, lengths, heads)
    q, k, v = RotaryQKV.apply(qkv, cos, sin, heads, torch.float32).double().cpu().unbind(0)
    s = q @ k.transpose(-1, -2) / 8.0
    valid = torch.arange(low_time)[None, :] < lengths.cpu()[:, None]
    s = s.masked_fill(~valid[:, None, None, :], float("-inf"))
    ref = (s.softmax(-1) @ v).transpose(1, 2).reshape(batch, low_time, heads * 64)
    err = (y.double().cpu() - ref).abs()
    assert (err <= 2.0 ** -7 * ref.abs() + 1e-6).all(), float(err.max())


def test_evidence_norm_reads_stacked_halves_in_place():
    """value/gate as the two halves of one stacked projection row: equal bit for bit
    to the same values passed as separate contiguous tensors; the stacked GEMM equals
    the two projections to BF16 rounding."""
    from trifusion_b200.kernels.buffers import stacked_linear

    g = torch.Generator().manual_seed(43)
    b, t, d, r = 3, 70, 384, 48
    x = torch.randn(b, t, d, generator=g).to(DEV)
    z = torch.randn(b, t, r, generator=g).to(torch.bfloat16).to(DEV)
    ev_v, ev_g = torch.nn.Linear(r, d).to(DEV), torch.nn.Linear(r, d).to(DEV)
    w = (1 + 0.05 * torch.randn(d, generator=g)).to(DEV)
    mask = torch.arange(t, device=DEV)[None, :] < torch.tensor([70, 31, 1], device=DEV)[:, None]
    wst, bst, pitch = stacked_linear([ev_v, ev_g], torch.bfloat16)
    assert pitch == d and wst.shape == (2 * d, r) and bst.shape == (2 * d,)
    ev = torch.nn.functional.linear(z, wst, bst)
    for out_dtype in (torch.float32, torch.bfloat16):
        got = native.evidence_norm(x, ev[..., :d], ev[..., d:], w, mask, 1e-5, out_dtype=out_dtype)
        ref = native.evidence_norm(x, ev[..., :d].contiguous(), ev[..., d:].contiguous(), w, mask, 1e-5,
                                   out_dtype=out_dtype)
        assert torch.equal(got, ref)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        sv, sg = ev_v(z), ev_g(z)
    torch.testing.assert_close(ev[..., :d].float(), sv.float(), atol=1e-2, rtol=2 ** -7)
    torch.testing.assert_close(ev[..., d:].float(), sg.float(), atol=1e-2, rtol=2 ** -7)
