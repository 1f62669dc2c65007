"""ctypes binding of the C-ABI library ``libtrifusion_b200.so``.

The library is the product's only compute path: if it is missing or the
current device is not a B200, calls raise; nothing falls back to PyTorch or
the CPU. Signatures mirror ``include/trifusion_b200.h``.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import os

# TRIFUSION_B200_BOUNDS=1 loads the bounds-checked debug build (build.py --debug-bounds).
LIB_PATH = Path(__file__).resolve().parent / "_native" / (
    "libtrifusion_b200_bounds.so" if os.environ.get("TRIFUSION_B200_BOUNDS") == "1" else "libtrifusion_b200.so")

TF_OK, TF_ERR_SHAPE, TF_ERR_ARG, TF_ERR_LAYOUT, TF_ERR_DEVICE, TF_ERR_LAUNCH, TF_ERR_SIZE = range(7)
TF_F32, TF_BF16 = 0, 1
SHAPE_MESSAGE = "L4 recurrence requires state=128, head=64, rotary=32"

_p = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_z = ctypes.c_size_t
_q = ctypes.c_int64

# name -> argtypes; every function returns int unless listed in _RESTYPES.
SIGNATURES = {
    "tf_status_string": [_i],
    "tf_version": [],
    "tf_last_cuda_error": [],
    "tf_device_error": [_i],
    "tf_error_watch_init": [],
    "tf_device_error_pending": [],
    "tf_set_flag_wait_ns": [ctypes.c_longlong],
    "tf_recurrence_workspace_size": [_i, _i, _i],
    "tf_fused_mamba_fwd": [_p, _p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p,
                           _i, _i, _i, _i, _p, _z, _p],
    "tf_mamba_recurrence_fwd": [_p, _p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p,
                                _i, _i, _i, _i, _p, _p, _f, _p, _p, _z, _p],
    "tf_mamba_recurrence_fwd_static": [_p, _p, _p, _p, _p, _p, _i, _p, _p, _p, _p, _p, _p, _p,
                                       _i, _i, _i, _i, _p, _p, _f, _p, _p],
    "tf_recurrence_workspace_size_multi": [_i, _i, _i, _i],
    "tf_mamba_recurrence_multi_fwd": [_p, _i, _i, _i, _i, _i, _f, _p, _p, _z, _p],
    # Satellite operators (argument order of include/trifusion_b200.h).
    "tf_rms_fwd": [_p, _i, _p, _p, _q, _i, _f, _p],
    "tf_evidence_norm_fwd": [_p, _i, _p, _p, _i, _p, _p, _p, _q, _i, _f, _p],
    "tf_mean_norm_fwd": [_p, _p, _i, _p, _p, _q, _i, _f, _p],
    "tf_mamba_controls_fwd": [_p, _p, _i, _p, _p, _f, _p, _p, _i, _i, _i, _p],
    "tf_mask_rows_fwd": [_p, _p, _p, _q, _q, _p],
    "tf_reverse_valid_fwd": [_p, _p, _p, _i, _i, _q, _p],
    "tf_swiglu_fwd": [_p, _i, _p, _q, _i, _p],
    "tf_gated_concat_fwd": [_p, _i, _p, _i, _p, _q, _i, _p],
    "tf_gated_branches_fwd": [_p, _p, _p, _i, _p, _p, _i, _p, _q, _i, _p],
    "tf_gate_branches_fwd": [_p, _q, _p, _q, _p, _p, _p, _p, _q, _i, _p],
    "tf_pooled_attention_fwd": [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "tf_evidence_norm_pitched_fwd": [_p, _i, _p, _p, _i, _q, _p, _p, _p, _i, _q, _i, _f, _p],
    "tf_query_read_state_floats": [_i, _i],
    "tf_query_read_fwd": [_p, _p, _q, _p, _i, _p, _q, _p, _i, _i, _p],
    "tf_rms_pitched_fwd": [_p, _i, _p, _p, _i, _q, _p, _q, _q, _i, _f, _p],
    "tf_mean_norm_copy_fwd": [_p, _p, _i, _p, _p, _p, _q, _q, _i, _f, _p],
    "tf_pool4_fwd": [_p, _i, _p, _p, _i, _i, _i, _p],
    "tf_masked_mean_fwd": [_p, _i, _p, _p, _i, _i, _i, _p],
    "tf_end_gather_fwd": [_p, _p, _p, _i, _i, _q, _p],
    "tf_depthwise_masked_fwd": [_p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "tf_rotary_qkv_fwd": [_p, _p, _p, _p, _i, _i, _i, _i, _p],
    "tf_interpolate_fwd": [_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "tf_front_norm_fwd": [_p, _i, _p, _p, _p, _i, _i, _i, _i, _f, _i, _p],
    "tf_front_stem_fwd": [_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _f, _p],
    "tf_masked_add_fwd": [_p, _p, _i, _p, _p, _q, _i, _p],
    "tf_rms_out_fwd": [_p, _i, _p, _p, _i, _q, _i, _f, _p],
    "tf_evidence_norm_out_fwd": [_p, _i, _p, _p, _i, _p, _p, _p, _i, _q, _i, _f, _p],
    "tf_depthwise_residual_fwd": [_p, _i, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "tf_rms_silu_fwd": [_p, _i, _p, _p, _q, _i, _f, _p],
    "tf_add_rms_fwd": [_p, _p, _i, _p, _p, _p, _i, _q, _i, _f, _p],
    "tf_pool4_out_fwd": [_p, _i, _p, _p, _i, _i, _i, _i, _p],
    "tf_front_residual_fwd": [_p, _p, _i, _p, _p, _i, _i, _i, _i, _p],
    "tf_bands_fwd": [_p, _i, _p, _i, _i, _i, _i, _p],
    "tf_ragged_copy_fwd": [_p, _p, _p, _p, _p, _i, _p, _i, _i, _p],
    "tf_glu_depthwise_fwd": [_p, _p, _p, _p, _p, _i, _i, _i, _i, _p],
    "tf_local_topk_fwd": [_p, _q, _p, _q, _p, _p, _p, _i, _i, _p],
    "tf_decoder_heads_scratch_bytes": [_i],
    "tf_decoder_heads_fwd": [_p] * 18 + [_q, _p, _i, _p],
}
_RESTYPES = {"tf_status_string": ctypes.c_char_p, "tf_last_cuda_error": ctypes.c_char_p,
             "tf_recurrence_workspace_size": ctypes.c_size_t,
             "tf_recurrence_workspace_size_multi": ctypes.c_size_t,
             "tf_query_read_state_floats": ctypes.c_int64,
             "tf_decoder_heads_scratch_bytes": ctypes.c_int64}


class RecurrenceIO(ctypes.Structure):
    """``tf_recurrence_io`` of include/trifusion_b200.h (one direction of a launch)."""

    _fields_ = [
        ("q", _p), ("k", _p), ("v", _p), ("z", _p), ("angles", _p),
        ("qb", _p), ("kb", _p), ("d", _p), ("adt", _p), ("dt", _p),
        ("trap", _p), ("trap_dtype", _i), ("a_raw", _p), ("ddt_raw", _p),
        ("dt_bias", _p), ("a_floor", _f), ("q_norm_w", _p), ("k_norm_w", _p),
        ("out", _p), ("strides", ctypes.c_int64 * 39), ("reverse", _i),
    ]

_lib = None


def lib():
    """Load (once) and return the library, with argument types declared."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"trifusion_b200 native library not built ({LIB_PATH}); run "
                "`python trifusion-fp-kernel_b200/build.py` (needs nvcc, no GPU)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = handle
    return _lib


def check(status):
    """Raise the reference-compatible exception for a non-zero status."""
    if status == TF_OK:
        return
    if status == TF_ERR_SHAPE:
        raise ValueError(SHAPE_MESSAGE)
    text = lib().tf_status_string(status).decode()
    detail = lib().tf_last_cuda_error().decode()
    if status == TF_ERR_ARG:
        raise ValueError(f"trifusion_b200: {text}")
    raise RuntimeError(f"trifusion_b200: {text}" + (f" ({detail})" if detail else ""))


DEVICE_ERROR_MESSAGE = ("trifusion_b200: a recurrence kernel gave up one of its bounded waits "
                        "(outputs of that launch are invalid)")
_watch = {"ready": False}


def error_watch():
    """Set up (once, outside stream capture) the host-mapped word that the kernels
    set when a bounded wait gives up, so later calls can see it without a sync."""
    if _watch["ready"]:
        return
    import torch

    if torch.cuda.is_current_stream_capturing():
        return
    _watch["ready"] = lib().tf_error_watch_init() == TF_OK


def check_device_error():
    """Raise ``RuntimeError`` if an earlier launch recorded a device-side timeout
    (read from the host-mapped word: no synchronisation). The word is cleared, so
    the error is raised once."""
    if _watch["ready"] and lib().tf_device_error_pending():
        lib().tf_device_error(1)
        raise RuntimeError(DEVICE_ERROR_MESSAGE)


def set_flag_wait_ns(ns):
    """Limit of the kernels' waits on other CTAs' chunk flags in later launches, in
    nanoseconds (0: the default 2 s). A diagnostic control for tests."""
    check(lib().tf_set_flag_wait_ns(int(ns)))


def int64_array(values):
    values = list(values)
    return (ctypes.c_int64 * len(values))(*values)


def dtype_code(x, op):
    """TF_F32 / TF_BF16 for a tensor's dtype; other dtypes are rejected."""
    import torch

    if x.dtype == torch.float32:
        return TF_F32
    if x.dtype == torch.bfloat16:
        return TF_BF16
    raise TypeError(f"{op}: expected float32 or bfloat16, got {x.dtype}")


def require_cuda(op, *tensors):
    """All tensors on one CUDA device (there is no CPU path)."""
    dev = tensors[0].device
    if dev.type != "cuda" or any(t.device != dev for t in tensors):
        raise RuntimeError(f"{op}: all tensors must be CUDA tensors on one device")
    return dev


def launch(fn, device, *args):
    """Call a C-ABI entry point on `device`'s current stream and check its status."""
    import torch

    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        check(getattr(lib(), fn)(*args, stream))


_workspaces = {}
# Outgrown workspaces are kept, never freed: a CUDA graph captured while one of them was
# current has its address baked into its recurrence launches.
_retired_workspaces = []


def workspace(device, nbytes):
    """Zero-filled device workspace of at least `nbytes`, cached per device.

    The kernels keep it consistent between launches themselves, so it is
    zeroed only when (re)allocated. Launches sharing it must not overlap in
    time, which holds for calls issued from one stream, or serialised across
    streams, as the reference requires of its callers (docs/api.md:47-48).
    When a call needs more, a new buffer of at least twice the size replaces it
    for later calls, and the old one stays allocated for the graphs that use it.
    """
    import torch

    error_watch()
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _workspaces.get(idx)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 1 << 20, 2 * buf.numel() if buf is not None else 0)
        if buf is not None:
            _retired_workspaces.append(buf)
        buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[idx] = buf
    return buf
