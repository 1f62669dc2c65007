"""CUDA parity of the fused recurrence against the reference (GPU only).

Mirrors the reference's parity suite (tests/test_recurrence.py): the 7 shapes
(T < C, C-1, C, C+1, multi-chunk, long), strided V/Z/angle views, and the
independent FP64 per-step formula; plus the benchmark configurations at full
size, Hq > 1, per-head angles, BF16 trap, misaligned views and empty inputs.
"""

import numpy as np
import pytest
import torch

from oracle import mamba_oracle as O
from golden_io import compare_packed, load_case, recurrence_cases
from parity import ATOL, RTOL, assert_recurrence_close, oracle_out, to_np
from trifusion_b200.synthetic import recurrence_inputs, lengths_uniform, norm_weight

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from trifusion_b200 import fused_mamba, fused_recurrence  # noqa: E402

DEV = "cuda"


@pytest.mark.parametrize("name", recurrence_cases())
def test_matches_reference_golden(name):
    """Against outputs of the reference's own kernels (FP32 path)."""
    shape, kw, data = load_case(name)
    args = recurrence_inputs(*shape, **kw, device=DEV)
    out = fused_mamba(*args)
    torch.cuda.synchronize()
    assert out.is_contiguous() and out.dtype == torch.bfloat16
    if "out" in data:
        assert_recurrence_close(out, data["out"], name)
    else:
        err, scale, rel = compare_packed(out.float().cpu().numpy(), data)
        assert rel < 0.006 and err < ATOL + RTOL * scale, (name, err, rel)


@pytest.mark.parametrize("batch,time,heads", [(1, 1, 4), (2, 26, 4), (1, 63, 32), (1, 64, 32),
                                              (2, 65, 4), (1, 255, 32), (1, 1501, 32)])
def test_reference_shapes_against_oracle(batch, time, heads):
    args = recurrence_inputs(batch, time, heads, kind="reftest", device=DEV)
    out = fused_mamba(*args)
    assert_recurrence_close(out, oracle_out(args), f"{batch}x{time}x{heads}")


def test_against_independent_float64_formula():
    """tests/test_recurrence.py:50-86: relative L2 < 0.012 vs the FP64 formula."""
    args = recurrence_inputs(1, 17, 4, kind="reftest", device=DEV)
    ref = O.fused_mamba_stepwise_f64(*to_np(args))
    out = fused_mamba(*args).double().cpu().numpy()
    assert np.linalg.norm(out - ref) / np.linalg.norm(ref) < 0.012


@pytest.mark.parametrize("batch,time", [(16, 200), (2, 3600), (2, 200)])
def test_benchmark_configs_full_size(batch, time):
    args = recurrence_inputs(batch, time, 12, kind="baseline", device=DEV)
    out = fused_mamba(*args)
    assert_recurrence_close(out, oracle_out(args), f"cfg B={batch} T={time}")


@pytest.mark.parametrize("groups", [2, 4])
def test_shared_qk_groups(groups):
    args = recurrence_inputs(2, 130, 8, groups=groups, kind="reftest", device=DEV)
    assert_recurrence_close(fused_mamba(*args), oracle_out(args), f"Hq={groups}")


def test_per_head_angles_and_bf16_trap():
    args = recurrence_inputs(2, 100, 6, kind="baseline", distinct_angles=True,
                             trap_dtype=torch.bfloat16, device=DEV)
    assert args[5].dtype == torch.bfloat16
    assert_recurrence_close(fused_mamba(*args), oracle_out(args), "distinct angles, bf16 trap")


def test_projection_views_like_the_model():
    """v, z, trap and angles as strided views of one in_proj output row
    (mamba.py:43-55,66,73-81): dim 384 gives a 1860-wide row (3720 B)."""
    b, t, h = 3, 150, 12
    g = torch.Generator().manual_seed(5)
    p = torch.randn(b, t, 1860, generator=g).to(torch.bfloat16).to(DEV)
    z, v, k, q, ddt, a, trap, ang = p.split([768, 768, 128, 128, h, h, h, 32], -1)
    ref_args = recurrence_inputs(b, t, h, kind="baseline", device=DEV)
    adt, dt = ref_args[3], ref_args[4]
    qb, kb, d = ref_args[6], ref_args[7], ref_args[9]
    args = (q.reshape(b, t, 1, 128), k.reshape(b, t, 1, 128), v.reshape(b, t, h, 64), adt, dt,
            trap.transpose(1, 2), qb, kb, ang.unsqueeze(2).expand(b, t, h, 32), d,
            z.reshape(b, t, h, 64))
    assert args[2].stride() == (t * 1860, 1860, 64, 1)
    out = fused_mamba(*args)
    assert_recurrence_close(out, oracle_out(args), "projection views")


def test_misaligned_views_take_the_scalar_path():
    """Odd element offsets (2-byte aligned rows): held to the oracle, and equal bit
    for bit to the 16-byte path on the same values."""
    b, t, h = 2, 70, 4
    base = recurrence_inputs(b, t, h, kind="reftest", device=DEV)
    q, k, v, adt, dt, trap, qb, kb, angles, d, z = base
    buf = torch.zeros(b, t, h * 64 * 2 + 3, dtype=torch.bfloat16, device=DEV)
    buf[:, :, 1:1 + h * 64] = v.reshape(b, t, -1)
    buf[:, :, 2 + h * 64: 2 + 2 * h * 64] = z.reshape(b, t, -1)
    v2 = buf[:, :, 1:1 + h * 64].reshape(b, t, h, 64)
    z2 = buf[:, :, 2 + h * 64: 2 + 2 * h * 64].reshape(b, t, h, 64)
    assert v2.data_ptr() % 4 == 2
    out = fused_mamba(q, k, v2, adt, dt, trap, qb, kb, angles, d, z2)
    assert_recurrence_close(out, oracle_out(base), "2-byte aligned views")
    ref = fused_mamba(*base)
    torch.testing.assert_close(out, ref, atol=0, rtol=0)


def test_empty_and_single_step():
    args = recurrence_inputs(2, 0 + 1, 3, kind="reftest", device=DEV)
    assert_recurrence_close(fused_mamba(*args), oracle_out(args), "T=1")
    e = recurrence_inputs(2, 5, 3, kind="reftest", device=DEV)
    e = [x[:, :0] if i in (0, 1, 2, 8, 10) else (x[:, :, :0] if i in (3, 4, 5) else x)
         for i, x in enumerate(e)]
    out = fused_mamba(*e)
    assert out.shape == (2, 0, 3, 64)


def test_deterministic_and_graph_capturable():
    args = recurrence_inputs(4, 200, 12, kind="baseline", device=DEV)
    a = fused_mamba(*args)
    b = fused_mamba(*args)
    assert torch.equal(a, b)
    out = torch.empty_like(a)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fused_mamba(*args)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        y = fused_mamba(*args)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, a)


@pytest.mark.parametrize("batch,time", [(16, 200), (2, 3600)])
def test_fused_norm_and_length_mask(batch, time):
    """RMSNorm prologue + recurrence + length mask in one launch, against the
    oracle's rms -> fused_mamba -> mask_rows sequence."""
    args = list(recurrence_inputs(batch, time, 12, kind="baseline", device=DEV))
    if batch == 16:
        lengths = lengths_uniform(batch, 120, 200)
    else:
        lengths = torch.tensor([3600, 2871])
    qw, kw = norm_weight(128, 1), norm_weight(128, 2)
    out = fused_recurrence(*args, q_norm=qw.to(DEV), k_norm=kw.to(DEV), lengths=lengths.to(DEV))
    npa = to_np(args)
    npa[0] = O.rms(npa[0], qw.numpy())
    npa[1] = O.rms(npa[1], kw.numpy())
    ref = O.mask_rows(O.fused_mamba(*npa), lengths.numpy())
    assert_recurrence_close(out, ref, "norm+mask")
    mask = torch.arange(time)[None, :] >= lengths[:, None]
    assert (out.cpu()[mask] == 0).all()


def test_length_edge_cases():
    args = list(recurrence_inputs(4, 130, 3, kind="reftest", device=DEV))
    lengths = torch.tensor([0, 1, 64, 130])
    out = fused_recurrence(*args, lengths=lengths.to(DEV))
    ref = O.mask_rows(oracle_out(args), lengths.numpy())
    assert_recurrence_close(out, ref, "length edges")


@pytest.mark.parametrize("batch,time,heads", [(260, 70, 1), (1, 64 * 513 + 5, 1)])
def test_launches_beyond_the_ticket_map(batch, time, heads):
    """Launches with more rows (260 > 256) or more chunks per row (514 > 512) than the
    kernel's ticket map holds hand out every unit and skip the empty ones; both
    against the oracle, with empty and partial rows."""
    args = list(recurrence_inputs(batch, time, heads, kind="reftest", device=DEV))
    if batch > 1:
        lengths = lengths_uniform(batch, 0, time, seed=5)
        lengths[:3] = torch.tensor([0, time, 1])
    else:
        lengths = torch.tensor([time - 100])
    out = fused_recurrence(*args, lengths=lengths.to(DEV))
    ref = O.mask_rows(oracle_out(args), lengths.numpy())
    assert_recurrence_close(out, ref, f"beyond the ticket map {batch}x{time}")


def test_padding_rows_zeroed_into_a_dirty_buffer():
    """Chunks wholly past a row's length are zeroed apart from the ticketed
    units; the caller's output buffer starts full of NaN, and most chunks of the
    shorter rows are empty (look-back rows: T = 1000 is 16 chunks)."""
    b, t, h = 8, 1000, 4
    args = list(recurrence_inputs(b, t, h, kind="reftest", device=DEV))
    lengths = torch.tensor([0, 1, 5, 64, 65, 300, 999, 1000])
    out = torch.full((b, t, h, 64), float("nan"), dtype=torch.bfloat16, device=DEV)
    for _ in range(2):
        fused_recurrence(*args, lengths=lengths.to(DEV), out=out)
    ref = O.mask_rows(oracle_out(args), lengths.numpy())
    assert_recurrence_close(out, ref, "dirty buffer")
    mask = torch.arange(t)[None, :] >= lengths[:, None]
    assert (out.cpu()[mask] == 0).all()


@pytest.mark.parametrize("batch,time,heads", [(2, 65, 4), (1, 255, 32), (1, 1501, 32)])
def test_agrees_with_reference_bf16_arithmetic(batch, time, heads):
    """Against the reference fused kernel's own BF16 rounding points, with the
    bound the reference holds its two BF16 kernels to (test_recurrence.py:45-47)."""
    args = recurrence_inputs(batch, time, heads, kind="reftest", device=DEV)
    ref = torch.from_numpy(oracle_out(args, bf16=True)).float()
    out = fused_mamba(*args).float().cpu()
    rel = (out - ref).norm() / ref.norm()
    assert rel < 0.006, float(rel)
    torch.testing.assert_close(out, ref, atol=0.04, rtol=0.02)


def test_captured_graph_survives_workspace_growth():
    """A CUDA graph captured with the cached recurrence workspace still replays correctly
    after a larger call has outgrown that workspace and the allocator has released its
    cache: the outgrown buffer stays allocated (an engine serving many batch shapes
    captures its graphs in increasing size)."""
    from trifusion_b200 import _lib

    small = recurrence_inputs(2, 130, 4, kind="reftest", device=DEV)
    ref = fused_mamba(*small)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fused_mamba(*small)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = fused_mamba(*small)
    before = _lib._workspaces[torch.cuda.current_device()]
    lib = _lib.lib()
    t = 4096
    while lib.tf_recurrence_workspace_size(4, t, 12) <= before.numel():
        t *= 2
    big = recurrence_inputs(4, t, 12, kind="baseline", device=DEV)
    fused_mamba(*big)
    assert _lib._workspaces[torch.cuda.current_device()].data_ptr() != before.data_ptr()
    del before, big
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
