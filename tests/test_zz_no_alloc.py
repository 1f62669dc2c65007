"""The recurrence entry point that allocates nothing (GPU only).

`tf_mamba_recurrence_fwd_static` serves callers that cannot allocate device
memory — plugin hosts that own all GPU memory through their own pool, and
services that forbid cudaMalloc after start-up — by running on a 64 MiB
workspace array that lives inside the library. This file is named to be
collected last, so that a run stopping at the first failure has already run
every other test; it passes alone in a fresh process (where its first call
sets up the array's device address) and after the other tests.
"""

import ctypes

import pytest
import torch

from trifusion_b200 import _lib
from trifusion_b200.synthetic import lengths_uniform, norm_weight, recurrence_inputs

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from trifusion_b200 import fused_recurrence  # noqa: E402
from trifusion_b200.mamba_fused import _strides  # noqa: E402

DEV = "cuda"


def _call_static(args, qw, kw, lengths, out):
    q, k, v, adt, dt, trap, qb, kb, angles, d, z = args
    b, t, h, _ = v.shape
    lib = _lib.lib()
    status = lib.tf_mamba_recurrence_fwd_static(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), adt.data_ptr(), dt.data_ptr(), trap.data_ptr(),
        _lib.TF_F32, qb.data_ptr(), kb.data_ptr(), angles.data_ptr(), d.data_ptr(), z.data_ptr(),
        out.data_ptr(), _strides(q, k, v, adt, dt, trap, angles, z, out), b, t, h, q.shape[2],
        qw.data_ptr(), kw.data_ptr(), ctypes.c_float(1e-5), lengths.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    return status


def _check(b, t, h, seed, qw, kw, lo):
    args = recurrence_inputs(b, t, h, kind="baseline", seed=seed, device=DEV)
    lengths = lengths_uniform(b, lo, t, seed=seed).to(DEV)
    ref = fused_recurrence(*args, q_norm=qw, k_norm=kw, lengths=lengths)
    out = torch.full_like(ref, float("nan"))
    assert _call_static(args, qw, kw, lengths, out) == _lib.TF_OK
    torch.cuda.synchronize()
    # The kernel is deterministic: both entries give the same bits.
    assert torch.equal(out, ref)


def test_static_workspace_entry_matches_the_workspace_entry_twice():
    qw, kw = norm_weight(128, 1).to(DEV), norm_weight(128, 2).to(DEV)
    for call in range(2):  # the second call runs on what the first left in the array
        _check(16, 200, 12, call, qw, kw, 120)
    assert _lib.lib().tf_device_error(1) == 0


def test_static_workspace_after_a_larger_problem_of_another_shape():
    """Every call clears the array's header (launch epoch, ticket and done counters)
    and the flags of the chunks it will use, so a call never depends on what an earlier
    call left there: here a long problem of one shape fills much of the array before a
    short one of another batch size and head count runs on it."""
    qw, kw = norm_weight(128, 1).to(DEV), norm_weight(128, 2).to(DEV)
    _check(1, 1000, 12, 5, qw, kw, 700)
    _check(5, 130, 7, 6, qw, kw, 1)
    assert _lib.lib().tf_device_error(1) == 0


def test_static_workspace_rejects_problems_beyond_its_capacity():
    # B=2, T=3600, H=12 needs ~68 MB of workspace, more than the 64 MiB array.
    args = recurrence_inputs(2, 3600, 12, kind="baseline", device=DEV)
    qw, kw = norm_weight(128, 1).to(DEV), norm_weight(128, 2).to(DEV)
    lengths = torch.tensor([3600, 2871], device=DEV)
    need = _lib.lib().tf_recurrence_workspace_size(2, 3600, 12)
    assert need > 64 * 2 ** 20
    out = torch.zeros(2, 3600, 12, 64, dtype=torch.bfloat16, device=DEV)
    assert _call_static(args, qw, kw, lengths, out) == _lib.TF_ERR_SIZE
    torch.cuda.synchronize()
    assert (out == 0).all()  # nothing was launched
