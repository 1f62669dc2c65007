"""Pin the CPU oracle against golden vectors produced by the reference itself.

The goldens come from the reference's Triton kernels (run through the Triton
interpreter on FP32 inputs) and its PyTorch formulas; see
tests/golden/make_golden.py. These tests need no GPU.
"""

import numpy as np
import pytest
import torch

from oracle import mamba_oracle as O
from trifusion_b200.synthetic import recurrence_inputs
from golden_io import compare_packed, input_checksum, load_case, recurrence_cases, GOLDEN


def _np(args):
    return [a.float().numpy() for a in args]


@pytest.mark.parametrize("name", recurrence_cases())
def test_generator_reproduces_golden_inputs(name):
    shape, kw, data = load_case(name)
    args = recurrence_inputs(*shape, **kw)
    assert input_checksum(_np(args)) == pytest.approx(float(data["input_checksum"]), rel=1e-12, abs=1e-9)


@pytest.mark.parametrize("name", recurrence_cases())
def test_oracle_matches_reference_fp32_path(name):
    shape, kw, data = load_case(name)
    if shape[1] > 600:
        pytest.skip("long case covered by test_oracle_long_case")
    out = O.fused_mamba(*_np(recurrence_inputs(*shape, **kw)))
    err, scale, rel = compare_packed(out, data)
    assert rel < 2e-6, (rel, err, scale)
    assert err < 2e-5 * max(scale, 1.0)


def test_oracle_long_case():
    shape, kw, data = load_case("rec_reftest_1x1501x2")
    out = O.fused_mamba(*_np(recurrence_inputs(*shape, **kw)))
    err, scale, rel = compare_packed(out, data)
    assert rel < 5e-6, (rel, err, scale)


def test_oracle_angle_scan_matches_reference():
    for name in recurrence_cases():
        shape, kw, data = load_case(name)
        if "phase" not in data:
            continue
        q, k, v, adt, dt, trap, qb, kb, angles, d, z = _np(recurrence_inputs(*shape, **kw))
        ph = O.angle_phase(angles, dt)
        # Phases near 0/2pi may wrap differently by one ulp; compare on the circle.
        diff = np.angle(np.exp(1j * (ph - data["phase"])))
        assert np.abs(diff).max() < 1e-5, name


@pytest.mark.parametrize("name", ["rec_reftest_2x26x4", "rec_groups2_2x100x4", "rec_distinct_1x90x3",
                                  "rec_baseline_cfg0"])
def test_chunked_oracle_matches_independent_f64_formula(name):
    """The reference's own FP64 per-step formula (tests/test_recurrence.py:54-85)."""
    shape, kw, _ = load_case(name)
    args = _np(recurrence_inputs(*shape, **kw))
    a = O.fused_mamba(*args)
    b = O.fused_mamba_stepwise_f64(*args)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-9


def test_bf16_oracle_is_close_to_fp32_path():
    shape, kw, data = load_case("rec_reftest_2x65x4")
    args = _np(recurrence_inputs(*shape, **kw))
    a = O.fused_mamba(*args, bf16=True)
    err, scale, rel = compare_packed(a, data)
    # The reference's own bound between its BF16 kernels (test_recurrence.py:45-47).
    assert rel < 0.006


def test_bf16_round_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.bf16_round(x), ref)


def test_shape_gate_message():
    args = _np(recurrence_inputs(1, 4, 2))
    args[0] = args[0][..., :64]
    with pytest.raises(ValueError, match="L4 recurrence requires state=128, head=64, rotary=32"):
        O.fused_mamba(*args)


# ---- satellites -------------------------------------------------------------

@pytest.fixture(scope="module")
def sat():
    return dict(np.load(GOLDEN / "satellites.npz"))


def _within_one_bf16_ulp(a, b):
    """The Triton interpreter truncates when it stores into a BF16 tensor, so
    its BF16 outputs can sit one BF16 ulp toward zero from a rounded result."""
    return np.all(np.abs(a - b) <= np.abs(b) * 2.0 ** -7 + 1e-30)


def test_rms_oracle(sat):
    y = O.rms(sat["rms_x"], sat["rms_w"])
    # The reference PyTorch formula is the bit-level golden; allow a rare
    # one-ulp difference where FP32 statistics land on a BF16 rounding tie.
    assert _within_one_bf16_ulp(y, sat["rms_torch"])
    assert (y != sat["rms_torch"]).mean() < 0.01
    assert _within_one_bf16_ulp(sat["rms_triton"], y)


def test_mean_norm_oracle(sat):
    y = O.mean_norm(sat["mn_a"], sat["mn_b"], sat["mn_w"])
    np.testing.assert_allclose(y, sat["mean_norm_triton"], rtol=2e-6, atol=2e-6)


def test_controls_oracle(sat):
    adt, dt = O.mamba_controls(sat["ctl_a"], sat["ctl_ddt"], sat["ctl_bias"])
    np.testing.assert_allclose(dt, sat["ctl_dt"], rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(adt, sat["ctl_adt"], rtol=2e-6, atol=1e-7)


def test_index_ops_bit_exact(sat):
    x, lengths = sat["x"], sat["lengths"]
    assert np.array_equal(O.mask_rows(x, lengths), sat["mask_triton"])
    assert np.array_equal(O.reverse_valid(x, lengths), sat["reverse_triton"])
    assert np.array_equal(O.reverse_valid(x, lengths), sat["reverse_torch"])
    assert np.array_equal(O.end_gather(x, lengths), sat["end_torch"])


def test_swiglu_gate_oracle(sat):
    for name, fn, args in [("swiglu", O.swiglu, (sat["sw_x"],)),
                           ("gate", O.gated_concat, (sat["gate_x"], sat["gate_g"]))]:
        y = fn(*args)
        ref = sat[f"{name}_torch"]
        assert np.abs(y - ref).max() <= 2 ** -7 * np.abs(ref).max()
        assert (y != ref).mean() < 0.01
        assert _within_one_bf16_ulp(sat[f"{name}_triton"], y)


def test_pool_oracle(sat):
    x, lengths = sat["x"], sat["lengths"]
    y = O.pool4(x, lengths)
    assert np.abs(y - sat["pool_torch"]).max() <= 2 ** -7 * np.abs(sat["pool_torch"]).max()
    assert (y != sat["pool_torch"]).mean() < 0.01
    assert _within_one_bf16_ulp(sat["pool_triton"], y)
    counts = O.pool4_counts(lengths, x.shape[1])
    assert counts.min() >= 1 and counts.max() <= 4


def test_masked_mean_oracle(sat):
    y = O.masked_mean(sat["x"], sat["lengths"])
    np.testing.assert_allclose(y, sat["masked_mean_torch"], rtol=1e-5, atol=1e-6)


def test_pool4_f32_is_the_reference_arithmetic(sat):
    # The FP32 sequential statement equals the PyTorch formula bit for bit, and
    # truncating it to BF16 reproduces the interpreter's stored output exactly.
    x, lengths = sat["x"], sat["lengths"]
    assert np.array_equal(O.pool4_f32(x, lengths), sat["pool_torch"])
    raw = O.pool4_f32(x, lengths, out_bf16=False)
    truncated = (raw.view(np.uint32) & 0xFFFF0000).view(np.float32)
    assert np.array_equal(truncated, sat["pool_triton"])


def test_evidence_norm_oracle(sat):
    y = O.evidence_norm(sat["ev_x"], sat["ev_v"], sat["ev_g"], sat["mn_w"], sat["ev_mask"])
    np.testing.assert_allclose(y, sat["evidence_norm_triton"], rtol=2e-6, atol=2e-6)
    assert (sat["evidence_norm_triton"][~sat["ev_mask"]] == 0).all()
