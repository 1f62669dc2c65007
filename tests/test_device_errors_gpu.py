"""Device-side timeouts reach the caller as exceptions (GPU only).

Every wait in the recurrence kernel is bounded. When one gives up, the kernel
records an error and finishes (its outputs are then invalid) instead of hanging;
the host sees the error through a host-mapped word, without a synchronisation,
and the next public call raises ``RuntimeError``. These tests make a wait run
out without faulting anything: the workspace's ticket counter is started at 1,
so chunk 0 of the row is never processed and its flag is never raised, and the
limit of waits on other CTAs' flags is lowered to a few nanoseconds. The CUDA
context stays usable afterwards.
"""

import pytest
import torch

from trifusion_b200 import _lib
from trifusion_b200.synthetic import recurrence_inputs

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

import trifusion_b200  # noqa: E402
from trifusion_b200 import fused_mamba  # noqa: E402

DEV = "cuda"
TICKET_OFFSET = 128  # byte offset of the ticket counter in the workspace header


def _skip_first_unit(b, t, h):
    lib = _lib.lib()
    ws = _lib.workspace(torch.device(DEV, torch.cuda.current_device()), lib.tf_recurrence_workspace_size(b, t, h))
    ws[TICKET_OFFSET:TICKET_OFFSET + 4].view(torch.int32).fill_(1)


@pytest.mark.parametrize("chunks", [4, 20])  # parallel flag waits; look-back (rows over 8 chunks)
def test_flag_wait_timeout_raises_on_the_next_call(chunks):
    t = 64 * chunks
    args = recurrence_inputs(1, t, 1, kind="baseline", seed=3, device=DEV)
    ref = fused_mamba(*args)
    torch.cuda.synchronize()
    assert _lib.lib().tf_device_error(1) == 0
    _skip_first_unit(1, t, 1)
    _lib.set_flag_wait_ns(5)
    try:
        fused_mamba(*args)
        torch.cuda.synchronize()
    finally:
        _lib.set_flag_wait_ns(0)
    assert _lib.lib().tf_device_error_pending() == 1
    with pytest.raises(RuntimeError, match="bounded waits"):
        fused_mamba(*args)
    # Raised once; the context and the workspace are usable again.
    assert _lib.lib().tf_device_error(0) == 0
    again = fused_mamba(*args)
    torch.cuda.synchronize()
    assert torch.equal(again, ref)


def test_check_device_error_is_exported():
    assert trifusion_b200.check_device_error is _lib.check_device_error
    trifusion_b200.check_device_error()  # nothing pending
