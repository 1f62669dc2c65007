"""GPU checks of the multi-direction recurrence launch (tf_mamba_recurrence_multi_fwd):

* controls computed inside the launch from the projection views (prologue
  fusion) equal the controls kernel followed by the recurrence, bit for bit;
* a reversed direction equals reversing the valid prefix of the projection
  rows, running forward, and reversing the output back, bit for bit (short rows
  that fold every predecessor and long rows that use the look-back);
* both directions in one launch equal two separate launches, bit for bit;
* the reversed direction against the CPU oracle, at the recurrence tolerance.
"""

import pytest
import torch

from oracle import mamba_oracle as O
from parity import assert_recurrence_close, oracle_out

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from trifusion_b200 import fused_recurrence  # noqa: E402
from trifusion_b200.kernels.buffers import mamba_controls  # noqa: E402
from trifusion_b200.mamba_fused import fused_recurrence_multi  # noqa: E402
from trifusion_b200.synthetic import norm_weight  # noqa: E402

DEV = "cuda"
H, N, R = 12, 128, 32
WIDTH = 2 * 768 + 2 * N + 3 * H + R  # the in_proj row of a dim-384 block: 1860


def projection(b, t, seed):
    """A [B, T, 1860] BF16 projection with the model's value scales per field."""
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(b, t, WIDTH, generator=g)
    p[..., 1536:1792] *= 1.0                     # k, q (normalised in the launch)
    p[..., 1792:1804] = p[..., 1792:1804] * 0.5  # ddt (dt = softplus(ddt - 4 + ...))
    p[..., 1804:1816] *= 2.0                     # a
    return p.to(torch.bfloat16).to(DEV)


def split(p, b, t):
    z, v, k, q, ddt, a, trap, angles = p.split([768, 768, N, N, H, H, H, R], -1)
    heads = (b, t, H, 64)
    return dict(q=q.reshape(b, t, 1, N), k=k.reshape(b, t, 1, N), v=v.reshape(heads), z=z.reshape(heads),
                trap=trap.transpose(1, 2), angles=angles.unsqueeze(2).expand(b, t, H, R), a=a, ddt=ddt)


def params(seed):
    g = torch.Generator().manual_seed(seed)
    return dict(qb=(1 + 0.1 * torch.randn(H, N, generator=g)).to(DEV),
                kb=(1 + 0.1 * torch.randn(H, N, generator=g)).to(DEV),
                d=torch.randn(H, generator=g).to(DEV),
                dt_bias=(-4 + 0.3 * torch.randn(H, generator=g)).to(DEV),
                q_norm=norm_weight(N, seed + 1).to(DEV), k_norm=norm_weight(N, seed + 2).to(DEV))


def direction(p, b, t, prm, reverse=False):
    s = split(p, b, t)
    return dict(q=s["q"], k=s["k"], v=s["v"], z=s["z"], trap=s["trap"], angles=s["angles"], qb=prm["qb"],
                kb=prm["kb"], d=prm["d"], a_raw=s["a"], ddt_raw=s["ddt"], dt_bias=prm["dt_bias"],
                a_floor=1e-4, q_norm=prm["q_norm"], k_norm=prm["k_norm"], reverse=reverse)


def reverse_rows(x, lengths):
    """Reverse every row's valid prefix along dim 1; rows past the length stay."""
    b, t = x.shape[:2]
    pos = torch.arange(t, device=x.device)[None, :]
    idx = torch.where(pos < lengths[:, None], lengths[:, None] - 1 - pos, pos)
    return torch.take_along_dim(x, idx.view(b, t, *([1] * (x.dim() - 2))), dim=1)


CASES = [(16, 200, [200, 137, 1, 0, 64, 199, 3, 128, 65, 200, 150, 77, 190, 13, 100, 180]),
         (3, 700, [700, 513, 64])]


@pytest.mark.parametrize("b,t,lens", CASES)
def test_controls_inside_the_launch_equal_the_controls_kernel(b, t, lens):
    p = projection(b, t, 1)
    prm = params(2)
    lengths = torch.tensor(lens, device=DEV)
    fused = fused_recurrence_multi([direction(p, b, t, prm)], lengths=lengths)[0]
    s = split(p, b, t)
    adt, dt = mamba_controls(s["a"], s["ddt"], prm["dt_bias"], 1e-4)
    ref = fused_recurrence(s["q"], s["k"], s["v"], adt, dt, s["trap"], prm["qb"], prm["kb"], s["angles"],
                           prm["d"], s["z"], q_norm=prm["q_norm"], k_norm=prm["k_norm"], lengths=lengths)
    assert torch.equal(fused, ref)


@pytest.mark.parametrize("b,t,lens", CASES)
def test_reversed_direction_equals_reversed_rows(b, t, lens):
    p = projection(b, t, 3)
    prm = params(4)
    lengths = torch.tensor(lens, device=DEV)
    rev = fused_recurrence_multi([direction(p, b, t, prm, reverse=True)], lengths=lengths)[0]
    fwd_of_reversed = fused_recurrence_multi([direction(reverse_rows(p, lengths), b, t, prm)], lengths=lengths)[0]
    assert torch.equal(rev, reverse_rows(fwd_of_reversed, lengths))
    # rows at or past each length are zero
    pad = torch.arange(t, device=DEV)[None, :] >= lengths[:, None]
    assert (rev[pad] == 0).all()


@pytest.mark.parametrize("b,t,lens", CASES)
def test_pair_launch_equals_two_launches(b, t, lens):
    pf, pb = projection(b, t, 5), projection(b, t, 6)
    prf, prb = params(7), params(8)
    lengths = torch.tensor(lens, device=DEV)
    yf, yb = fused_recurrence_multi([direction(pf, b, t, prf), direction(pb, b, t, prb, reverse=True)],
                                    lengths=lengths)
    sf = fused_recurrence_multi([direction(pf, b, t, prf)], lengths=lengths)[0]
    sb = fused_recurrence_multi([direction(pb, b, t, prb, reverse=True)], lengths=lengths)[0]
    assert torch.equal(yf, sf) and torch.equal(yb, sb)


def test_reversed_direction_against_oracle():
    b, t = 2, 150
    lengths = torch.tensor([150, 97], device=DEV)
    p = projection(b, t, 9)
    prm = params(10)
    rev = fused_recurrence_multi([direction(p, b, t, prm, reverse=True)], lengths=lengths)[0]
    # Oracle: the reversed rows, controls and norms in PyTorch FP32, the FP64 recurrence.
    pr = reverse_rows(p, lengths)
    s = split(pr, b, t)
    a, ddt = s["a"].float(), s["ddt"].float()
    control = -(a.clamp(min=0) + 1 / (1 - a.clamp(max=0))).clamp(min=1e-4)
    dt = torch.nn.functional.softplus(ddt + prm["dt_bias"])
    adt, dt = (control * dt).transpose(1, 2), dt.transpose(1, 2)

    def rms(x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5) * w).to(torch.bfloat16)

    args = (rms(s["q"], prm["q_norm"]), rms(s["k"], prm["k_norm"]), s["v"], adt, dt, s["trap"], prm["qb"],
            prm["kb"], s["angles"], prm["d"], s["z"])
    ref = torch.as_tensor(oracle_out(args))
    pad = torch.arange(t)[None, :] >= lengths.cpu()[:, None]
    ref[pad] = 0
    assert_recurrence_close(reverse_rows(rev, lengths).float().cpu(), ref, "reversed direction")


def test_reversed_direction_contiguous_inputs():
    """Contiguous 16-byte-aligned inputs (rows staged by bulk copies): the reversed
    direction equals the forward direction on reversed rows, bit for bit."""
    from trifusion_b200.synthetic import recurrence_inputs

    b, t = 4, 300
    lengths = torch.tensor([300, 170, 64, 1], device=DEV)
    names = ("q", "k", "v", "adt", "dt", "trap", "qb", "kb", "angles", "d", "z")
    args = dict(zip(names, recurrence_inputs(b, t, H, kind="baseline", seed=11, device=DEV)))
    prm = params(12)
    rev = fused_recurrence_multi([dict(args, q_norm=prm["q_norm"], k_norm=prm["k_norm"], reverse=True)],
                                 lengths=lengths)[0]
    flipped = dict(args)
    for name in ("q", "k", "v", "z", "angles"):
        flipped[name] = reverse_rows(args[name], lengths).contiguous()
    for name in ("adt", "dt", "trap"):  # [B, H, T]: reverse along the last axis
        flipped[name] = reverse_rows(args[name].transpose(1, 2), lengths).transpose(1, 2).contiguous()
    fwd = fused_recurrence_multi([dict(flipped, q_norm=prm["q_norm"], k_norm=prm["k_norm"])], lengths=lengths)[0]
    assert torch.equal(rev, reverse_rows(fwd, lengths))


def test_pair_rows_side_by_side_and_paired_mean():
    """Both directions written into one [B, T, 2 * 768] row buffer through the output
    strides equal the separate outputs bit for bit, and the one-GEMM mean of the two
    out projections is within BF16 rounding of the mean of the two projections."""
    from types import SimpleNamespace

    from trifusion_b200.mamba import Mamba3Inference, bidirectional_pair, bidirectional_rows, paired_mean

    torch.manual_seed(11)
    cfg = SimpleNamespace(dim=384, state_dim=128, backend="l4")
    fwd, bwd = Mamba3Inference(cfg).cuda(), Mamba3Inference(cfg).cuda()
    for m in (fwd, bwd):
        m.fused_recurrence = True
    u = (0.5 * torch.randn(3, 150, 384, device="cuda")).to(torch.bfloat16)
    lengths = torch.tensor([150, 77, 9], device="cuda")
    with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16):
        y = bidirectional_rows(fwd, bwd, u, lengths)
        from trifusion_b200.mamba import projections
        from trifusion_b200.mamba_fused import fused_recurrence_multi

        pf, pb = projections([fwd, bwd], u)
        yf, yb = fused_recurrence_multi([fwd._direction(pf, 3, 150), bwd._direction(pb, 3, 150, reverse=True)],
                                        lengths=lengths, eps=fwd.C_norm.eps)
        avg = paired_mean(fwd, bwd, y)
        mf, mb = bidirectional_pair(fwd, bwd, u, lengths)
    assert torch.equal(y[..., :768], yf.reshape(3, 150, 768))
    assert torch.equal(y[..., 768:], yb.reshape(3, 150, 768))
    ref = (mf.float() + mb.float()) * 0.5
    torch.testing.assert_close(avg.float(), ref, atol=2e-2, rtol=2 ** -6)
    with pytest.raises(ValueError):
        d = fwd._direction(pf, 3, 150)
        d["out"] = torch.empty(3, 150, 12, 32, dtype=torch.bfloat16, device="cuda")
        fused_recurrence_multi([d], lengths=lengths)


def _aligned_views(p, pitch, offset):
    """The projection's values in a wider buffer: rows `pitch` elements apart, starting
    `offset` elements in (pitch 1864, offset 0: 16-byte rows; 1868, 4: 8-byte rows)."""
    b, t, w = p.shape
    buf = torch.zeros(b, t, pitch, dtype=p.dtype, device=p.device)
    buf[..., offset:offset + w] = p
    return buf[..., offset:offset + w]


@pytest.mark.parametrize("mode", ["forward", "reversed", "pair"])
def test_tma_staging_equals_cp_async_staging(mode):
    """Rows of more than 8 chunks with 16-byte rows are staged by TMA boxes; the same
    values in 8-byte-aligned rows by per-thread cp.async. Same arithmetic: equal bits."""
    b, t = 3, 700
    lengths = torch.tensor([700, 451, 64], device=DEV)
    p = projection(b, t, 21)
    prm = params(22)
    outs = []
    for pitch, offset in ((1864, 0), (1868, 4)):
        pv = _aligned_views(p, pitch, offset)
        dirs = {"forward": [direction(pv, b, t, prm)], "reversed": [direction(pv, b, t, prm, reverse=True)],
                "pair": [direction(pv, b, t, prm), direction(pv, b, t, prm, reverse=True)]}[mode]
        outs.append(fused_recurrence_multi(dirs, lengths=lengths))
    for x, y in zip(*outs):
        assert torch.equal(x, y)


def test_tma_staged_long_rows_against_oracle():
    from trifusion_b200.synthetic import recurrence_inputs

    b, t = 2, 1100
    lengths = torch.tensor([1100, 777], device=DEV)
    args = recurrence_inputs(b, t, 4, kind="baseline", seed=31, device=DEV)
    out = fused_recurrence(*args, lengths=lengths)
    ref = O.mask_rows(oracle_out(args), lengths.cpu().numpy())
    assert_recurrence_close(out, ref, "TMA-staged long rows")
