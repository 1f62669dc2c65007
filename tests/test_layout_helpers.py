"""Host-side layout helpers of the block and decoder kernels (CPU only).

* row pitch of views that are slices of wider row buffers (what the pitched norm,
  branch-gate and query-read entry points are given);
* stacked projection weights: zero-padded to aligned row slices, cached until a
  parameter changes, superseded copies kept alive for captured graphs;
* the pair's one-GEMM mean of two out projections;
* the decoder's query read given lengths instead of a mask.
"""

import pytest
import torch

from trifusion_b200.kernels.native import _row_pitch


def test_row_pitch_of_slices_and_rejections():
    buf = torch.empty(4, 5, 24)
    assert _row_pitch(buf[..., :8], 8, "t") == 24
    assert _row_pitch(buf[..., 16:], 8, "t") == 24
    assert _row_pitch(torch.empty(4, 5, 8), 8, "t") == 8
    assert _row_pitch(torch.empty(4, 1, 24)[..., 8:16], 8, "t") == 24  # unit dims carry no stride
    assert _row_pitch(torch.empty(1, 1, 24)[..., 8:16], 8, "t") == 8
    with pytest.raises(ValueError):
        _row_pitch(buf.transpose(0, 1)[..., :8], 8, "t")  # rows not evenly spaced
    with pytest.raises(ValueError):
        _row_pitch(buf[..., ::2][..., :8], 8, "t")  # last dim not contiguous
    with pytest.raises(ValueError):
        _row_pitch(buf[..., :8], 6, "t")  # width mismatch


def test_stacked_linear_pads_caches_and_retires():
    from trifusion_b200.kernels import buffers as B

    torch.manual_seed(0)
    a, b = torch.nn.Linear(16, 13), torch.nn.Linear(16, 13)
    w, bias, pitch = B.stacked_linear([a, b], torch.float32, multiple=8)
    assert pitch == 16 and w.shape == (32, 16) and bias.shape == (32,)
    assert torch.equal(w[:13], a.weight.detach()) and torch.equal(w[16:29], b.weight.detach())
    assert not w[13:16].any() and not w[29:].any() and not bias[13:16].any()
    x = torch.randn(7, 16)
    y = torch.nn.functional.linear(x, w, bias)
    torch.testing.assert_close(y[:, :13], a(x).detach())
    torch.testing.assert_close(y[:, 16:29], b(x).detach())
    assert B.stacked_linear([a, b], torch.float32, multiple=8)[0] is w  # cached
    key = next(k for k, e in B._STACKED._entries.items() if e[1][0] is w)
    with torch.no_grad():
        a.weight.add_(1.0)  # version counter moves: a new stacked copy, the old one kept
    w2, _, _ = B.stacked_linear([a, b], torch.float32, multiple=8)
    assert w2 is not w and B._STACKED._entries[key][2][-1][0] is w
    assert torch.equal(w2[:13], a.weight.detach())
    with pytest.raises(ValueError):
        B.stacked_linear([a, torch.nn.Linear(16, 12)], torch.float32)


def test_param_caches_drop_entries_of_freed_parameters():
    """Loading and freeing layers leaves no cached copies behind: an entry (with the
    copies it superseded) goes when one of its parameters is garbage-collected."""
    import gc

    from trifusion_b200.kernels import buffers as B

    before = len(B._STACKED), len(B._BF16_PARAMS)
    for _ in range(5):
        a, b = torch.nn.Linear(16, 13), torch.nn.Linear(16, 13)
        B.stacked_linear([a, b], torch.float32, multiple=8)
        with torch.no_grad():
            a.weight.add_(1.0)
        B.stacked_linear([a, b], torch.float32, multiple=8)
        B._param_bf16(a.weight, (13, 16))
        assert len(B._STACKED) == before[0] + 1 and len(B._BF16_PARAMS) == before[1] + 1
        del a, b
        gc.collect()
        assert (len(B._STACKED), len(B._BF16_PARAMS)) == before


def test_paired_mean_is_the_mean_of_both_projections():
    from types import SimpleNamespace

    from trifusion_b200.mamba import paired_mean

    torch.manual_seed(1)
    f = SimpleNamespace(out_proj=torch.nn.Linear(32, 12, bias=False))
    b = SimpleNamespace(out_proj=torch.nn.Linear(32, 12, bias=False))
    y = torch.randn(3, 5, 64, dtype=torch.float64).float()
    got = paired_mean(f, b, y)
    ref = (f.out_proj(y[..., :32]) + b.out_proj(y[..., 32:])).detach() * 0.5
    torch.testing.assert_close(got, ref, atol=1e-6, rtol=1e-6)


def test_query_read_lengths_equal_the_expanded_mask_on_cpu():
    """On the CPU (no kernel) the lengths form builds the same mask the reference
    expands: key t * 8 + band valid when t < length."""
    from trifusion_b200.decoder import QueryRead
    from trifusion_b200.masking import time_mask

    torch.manual_seed(2)
    qr = QueryRead(64)
    b, t = 2, 9
    x = torch.randn(b, t * 8, 64)
    query = torch.randn(10, 256) * 0.02
    lengths = torch.tensor([9, 4])
    mask = time_mask(lengths, t)[:, :, None].expand(b, t, 8).reshape(b, -1)
    with torch.inference_mode():
        ref = qr(query, x, mask)
        got = qr(query, x, None, lengths, keys_per_length=8)
    for r, g in zip(ref, got):
        assert torch.equal(r, g)


def test_weight_caches_match_only_the_same_live_parameter():
    """A cache entry hits only for the very parameter object it was made from: another
    tensor with the same address and version counter (here a view, as a new model's
    parameter can be after the old one is freed) is a miss, and so is a freed one."""
    from trifusion_b200.kernels import buffers as B

    p = torch.nn.Parameter(torch.randn(6, 4))
    stamp = B._stamp((p,))
    assert B._stamp_matches(stamp, (p,))
    alias = p.view(6, 4)  # same storage, same version counter, another object
    assert alias.data_ptr() == p.data_ptr() and alias._version == p._version
    assert not B._stamp_matches(stamp, (alias,))
    with torch.no_grad():
        p.mul_(2.0)
    assert not B._stamp_matches(stamp, (p,))  # version moved
    q = torch.nn.Parameter(torch.randn(6, 4))
    first = B._param_bf16(q, (6, 4))
    assert B._param_bf16(q, (6, 4)) is first
    torch.testing.assert_close(first.float(), q.detach(), atol=1e-2, rtol=1e-2)
