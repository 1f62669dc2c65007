"""C-ABI library checks that need no GPU: it loads, exports every symbol the
public header declares, and rejects bad arguments before touching a device."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

from trifusion_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "trifusion_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tf_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_symbols()
    assert "tf_fused_mamba_fwd" in names and len(names) >= 5
    for name in names:
        assert hasattr(lib, name), name
    # The ctypes table covers the header exactly.
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_ctypes_table_matches_header_arity():
    """Every ctypes argument list has as many entries as the header's prototype."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, params in re.findall(r"\b(tf_[a-z0-9_]+)\s*\(([^;{]*?)\)\s*;", text):
        params = params.strip()
        count = 0 if params in ("", "void") else params.count(",") + 1
        assert len(_lib.SIGNATURES[name]) == count, (name, len(_lib.SIGNATURES[name]), count)


def test_status_strings_and_version():
    lib = _lib.lib()
    assert lib.tf_status_string(0) == b"ok"
    assert lib.tf_status_string(1).decode() == _lib.SHAPE_MESSAGE
    assert lib.tf_version() >= 100


def test_invalid_arguments_rejected_without_a_device():
    lib = _lib.lib()
    strides = _lib.int64_array([0] * 33)
    # Null strides, bad dtype, groups not dividing heads: validated on the host.
    assert lib.tf_fused_mamba_fwd(*([None] * 6), 0, *([None] * 6), None, 1, 1, 4, 1, None, 0, None) == _lib.TF_ERR_ARG
    assert lib.tf_fused_mamba_fwd(*([None] * 6), 7, *([None] * 6), strides, 1, 1, 4, 1, None, 0, None) == _lib.TF_ERR_ARG
    assert lib.tf_fused_mamba_fwd(*([None] * 6), 0, *([None] * 6), strides, 1, 1, 4, 3, None, 0, None) == _lib.TF_ERR_ARG
    # Empty problems are a no-op success.
    assert lib.tf_fused_mamba_fwd(*([None] * 6), 0, *([None] * 6), strides, 0, 5, 4, 1, None, 0, None) == _lib.TF_OK
    # Workspace size query: grows with the number of 64-step chunk units.
    assert lib.tf_recurrence_workspace_size(0, 5, 4) == 0
    assert lib.tf_recurrence_workspace_size(16, 200, 12) > lib.tf_recurrence_workspace_size(16, 64, 12) > 0
    with pytest.raises(ValueError):
        _lib.check(_lib.TF_ERR_ARG)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.TF_ERR_LAUNCH)


def test_python_shape_gate_matches_reference_message():
    from trifusion_b200 import fused_mamba
    from trifusion_b200.synthetic import recurrence_inputs
    args = list(recurrence_inputs(1, 4, 2))
    args[0] = args[0][..., :64].contiguous()
    with pytest.raises(ValueError, match=r"^L4 recurrence requires state=128, head=64, rotary=32$"):
        fused_mamba(*args)


def test_cpu_tensors_fail_loudly_no_fallback():
    from trifusion_b200 import fused_mamba
    from trifusion_b200.synthetic import recurrence_inputs
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        fused_mamba(*recurrence_inputs(1, 4, 2))


def test_lazy_import_keeps_torch_out():
    import subprocess
    import sys
    root = Path(__file__).resolve().parent.parent / "trifusion-fp-kernel_b200"
    code = ("import sys; sys.path.insert(0, %r); import trifusion_b200 as t; "
            "assert 'torch' not in sys.modules; assert t.__version__ == '0.1.0'; "
            "assert {'configure_runtime','load_student','InferenceEngine','fused_mamba'} <= set(dir(t))"
            % str(root))
    subprocess.run([sys.executable, "-c", code], check=True)


def test_satellite_entry_points_validate_on_the_host():
    lib = _lib.lib()
    # Bad dtype codes and negative sizes are argument errors; empty work is a no-op.
    assert lib.tf_rms_fwd(None, 7, None, None, 4, 128, 1e-5, None) == _lib.TF_ERR_ARG
    assert lib.tf_rms_fwd(None, _lib.TF_BF16, None, None, 0, 128, 1e-5, None) == _lib.TF_OK
    assert lib.tf_mean_norm_fwd(None, None, _lib.TF_BF16, None, None, 4, 0, 1e-5, None) == _lib.TF_ERR_ARG
    assert lib.tf_evidence_norm_fwd(None, 0, None, None, 3, None, None, None, 1, 8, 1e-5, None) == _lib.TF_ERR_ARG
    assert lib.tf_swiglu_fwd(None, _lib.TF_BF16, None, -1, 8, None) == _lib.TF_ERR_ARG
    assert lib.tf_swiglu_fwd(None, _lib.TF_BF16, None, 0, 8, None) == _lib.TF_OK
    assert lib.tf_gated_concat_fwd(None, 0, None, 9, None, 1, 8, None) == _lib.TF_ERR_ARG
    assert lib.tf_mask_rows_fwd(None, None, None, 0, 16, None) == _lib.TF_OK
    assert lib.tf_reverse_valid_fwd(None, None, None, 2, 3, 16, None) == _lib.TF_ERR_ARG
    assert lib.tf_pool4_fwd(None, 1, None, None, 0, 10, 8, None) == _lib.TF_OK
    assert lib.tf_masked_mean_fwd(None, 5, None, None, 1, 10, 8, None) == _lib.TF_ERR_ARG
    assert lib.tf_end_gather_fwd(None, None, None, 2, 0, 16, None) == _lib.TF_ERR_ARG
    strides = _lib.int64_array([24, 12, 1, 24, 12, 2])  # ddt innermost stride 2: layout error
    assert lib.tf_mamba_controls_fwd(None, None, 1, strides, None, 1e-4, None, None, 1, 2, 3,
                                     None) == _lib.TF_ERR_ARG
    buf = ctypes.c_void_p(1)
    assert lib.tf_mamba_controls_fwd(buf, buf, 1, strides, buf, 1e-4, buf, buf, 1, 2, 3,
                                     None) == _lib.TF_ERR_LAYOUT


def test_satellite_wrappers_reject_cpu_tensors():
    from trifusion_b200.kernels import gated_concat, reverse_valid, swiglu
    from trifusion_b200.kernels import native
    from trifusion_b200.kernels.buffers import Pool4, mamba_controls, mask_buffer

    x = torch.zeros(2, 8, 16, dtype=torch.bfloat16)
    lengths = torch.tensor([8, 3])
    calls = [
        lambda: swiglu(x),
        lambda: reverse_valid(x, lengths),
        lambda: gated_concat(torch.zeros(2, 8, 48, dtype=torch.bfloat16), torch.zeros(2, 8, 3)),
        lambda: native.rms(x, torch.ones(16)),
        lambda: native.mean_norm(x, x, torch.ones(16)),
        lambda: native.masked_mean(x, lengths),
        lambda: Pool4.apply(x, lengths),
        lambda: mask_buffer(x, torch.ones(2, 8, dtype=torch.bool)),
        lambda: mamba_controls(x[..., :4], x[..., 4:8], torch.zeros(4), 1e-4),
    ]
    for call in calls:
        with pytest.raises(RuntimeError, match="CUDA tensors"):
            call()
