"""Shared helpers for the CUDA-vs-oracle parity tests."""

import numpy as np
import torch

from oracle import mamba_oracle as O

# Tolerance the CUDA recurrence is held to against the reference's FP32 path:
# |cuda - ref| <= ATOL + RTOL * |ref| elementwise.
ATOL = 1e-2
RTOL = 1e-2
# The reference's own bound between its BF16 kernels (tests/test_recurrence.py:45-46).
REL_L2 = 0.006


def to_np(args):
    return [a.detach().float().cpu().numpy() for a in args]


def assert_recurrence_close(actual, ref, what=""):
    a = actual.detach().float().cpu().numpy().astype(np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert np.isfinite(a).all(), f"{what}: non-finite output"
    err = np.abs(a - r)
    bound = ATOL + RTOL * np.abs(r)
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), (
        f"{what}: max excess {float((err - bound).max()):.3e} at {worst}: "
        f"got {a[worst]:.5f} ref {r[worst]:.5f}; max abs err {err.max():.3e}")
    rel = np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-30)
    assert rel < REL_L2, f"{what}: relative L2 {rel:.3e}"
    return float(err.max()), float(rel)


def oracle_out(args, **kw):
    return O.fused_mamba(*to_np(args), **kw)
