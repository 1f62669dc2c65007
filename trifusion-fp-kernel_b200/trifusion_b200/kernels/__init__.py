"""Inference operators on B200 with the interface of ``trifusion_l4.kernels``
(reference ``kernels/__init__.py``).

``backend="l4"`` (the name the reference's checkpoints and configs use for the
optimized path) runs the CUDA kernels of ``libtrifusion_b200.so``;
``backend="reference"`` evaluates the reference's own PyTorch formulas, which
the reference model uses when it is loaded with ``optimized=False``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .. import _lib


def rms_reference(x, weight, eps):
    """PyTorch RMSNorm formula (reference ``kernels/__init__.py:10-11``)."""
    xf = x.to(torch.float64 if x.dtype == torch.float64 else torch.float32)
    inv = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * inv * weight).to(x.dtype)


class RMSNorm(nn.Module):
    """RMSNorm with the reference's parameter layout (``weight``) and backends."""

    def __init__(self, dim, eps=1e-5, backend="reference"):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps
        self.backend = backend
        self.native_kernels = False

    def forward(self, x):
        if self.backend == "reference":
            return rms_reference(x, self.weight, self.eps)
        from .native import rms

        return rms(x, self.weight, self.eps)


def swiglu(x, backend="l4"):
    """``silu(g) * u`` for ``g, u = x.chunk(2, -1)`` (reference ``kernels/__init__.py:30-40``)."""
    if backend == "reference":
        half = x.shape[-1] // 2
        g, u = x.float().split(half, dim=-1)
        return (F.silu(g) * u).to(x.dtype)
    x = x.contiguous()
    dev = _lib.require_cuda("swiglu", x)
    d = x.shape[-1] // 2
    y = x.new_empty((*x.shape[:-1], d))
    rows = y.numel() // d if d else 0
    _lib.launch("tf_swiglu_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "swiglu"), y.data_ptr(),
                rows, d)
    return y


def reverse_valid(x, lengths, backend="l4"):
    """``y[b, t] = x[b, len-1-t]`` inside the valid prefix, zero after it
    (reference ``kernels/__init__.py:43-54``)."""
    if backend == "reference":
        steps = torch.arange(x.shape[1], device=x.device).unsqueeze(0)
        src = (lengths.unsqueeze(1) - 1 - steps).clamp(min=0)
        rows = torch.take_along_dim(x, src.unsqueeze(-1), dim=1)
        valid = (steps < lengths.unsqueeze(1)).unsqueeze(-1)
        return torch.where(valid, rows, 0.0)
    x = x.contiguous()
    dev = _lib.require_cuda("reverse_valid", x, lengths)
    b, t = x.shape[:2]
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty_like(x)
    row_bytes = (x.numel() // (b * t) if b * t else 0) * x.element_size()
    _lib.launch("tf_reverse_valid_fwd", dev, x.data_ptr(), lengths.data_ptr(), y.data_ptr(), b, t,
                row_bytes)
    return y


def gated_concat(x, gate, backend="l4"):
    """``x[..., j, :] * 2 sigmoid(gate[..., j])`` for the three branches
    (reference ``kernels/__init__.py:57-81``)."""
    if backend == "reference":
        scale = 2 * torch.sigmoid(gate.float()).unsqueeze(-1)
        return (x.float().unflatten(-1, (3, -1)) * scale).flatten(-2).to(x.dtype)
    x, gate = x.contiguous(), gate.contiguous()
    dev = _lib.require_cuda("gated_concat", x, gate)
    d = x.shape[-1] // 3
    rows = gate.numel() // 3
    if gate.shape[-1] != 3 or x.numel() != rows * 3 * d:
        raise ValueError("gated_concat: x must be [..., 3*d] and gate [..., 3]")
    y = torch.empty_like(x)
    _lib.launch("tf_gated_concat_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "gated_concat"),
                gate.data_ptr(), _lib.dtype_code(gate, "gated_concat"), y.data_ptr(), rows, d)
    return y


def gate_branches(s, x1, weight, bias=None, gate_out=None):
    """``gated_concat(cat(s0, x1, s2), linear(s, weight, bias))`` in one pass under BF16
    arithmetic: ``s`` is the BF16 gate-input row ``[..., 3 d]`` (rows evenly spaced;
    its first and last thirds are the gated branches 0 and 2), ``x1`` the FP32 branch 1,
    ``weight`` ``[3, 3 d]`` and ``bias`` ``[3]`` BF16. The gate values are the BF16
    projection with FP32 sums (the GEMM's up to summation order), written to
    ``gate_out`` ([..., 3] BF16) when given. Returns the FP32 ``[..., 3 d]`` row
    (reference ``model.py:185-186``)."""
    from .native import _row_pitch

    dev = _lib.require_cuda("gate_branches", s, x1, weight)
    d = x1.shape[-1]
    x1 = x1.contiguous()
    if s.dtype != torch.bfloat16 or s.shape[:-1] != x1.shape[:-1] or s.shape[-1] != 3 * d:
        raise ValueError("gate_branches: s must be BF16 [..., 3 d] with x1 [..., d]")
    if x1.dtype != torch.float32 or weight.dtype != torch.bfloat16 or tuple(weight.shape) != (3, 3 * d):
        raise ValueError("gate_branches: x1 must be FP32 and weight BF16 [3, 3 d]")
    weight = weight.contiguous()
    if bias is not None:
        if bias.dtype != torch.bfloat16 or bias.numel() != 3:
            raise ValueError("gate_branches: bias must be BF16 [3]")
        bias = bias.contiguous()
    rows = x1.numel() // d if d else 0
    y = torch.empty((*x1.shape[:-1], 3 * d), device=dev, dtype=torch.float32)
    if gate_out is not None and (gate_out.dtype != torch.bfloat16 or gate_out.shape != (*x1.shape[:-1], 3)
                                 or not gate_out.is_contiguous()):
        raise ValueError("gate_branches: gate_out must be a contiguous BF16 [..., 3] tensor")
    _lib.launch("tf_gate_branches_fwd", dev, s.data_ptr(), _row_pitch(s, 3 * d, "gate_branches"), x1.data_ptr(),
                d, weight.data_ptr(), None if bias is None else bias.data_ptr(), y.data_ptr(),
                None if gate_out is None else gate_out.data_ptr(), rows, d)
    return y


def gated_branches(x0, x1, x2, gate):
    """``gated_concat(torch.cat((x0, x1, x2), -1), gate)`` without the concatenation:
    x0 and x2 share a dtype (they may be slices of a wider row buffer), x1 is FP32, the
    result is the FP32 ``[..., 3 d]`` row, bit-equal to the concatenated form
    (reference ``model.py:185-186``)."""
    from .native import _row_pitch

    dev = _lib.require_cuda("gated_branches", x0, x1, x2, gate)
    d = x1.shape[-1]
    x1 = x1.contiguous()
    if x1.dtype != torch.float32 or x0.dtype != x2.dtype or x0.shape != x1.shape or x2.shape != x1.shape:
        raise ValueError("gated_branches: x1 must be FP32, x0/x2 of one dtype, all of one shape")
    if gate.shape != (*x1.shape[:-1], 3):
        raise ValueError("gated_branches: gate must be [..., 3]")
    gate = gate.contiguous()
    rows = gate.numel() // 3
    pitches = _lib.int64_array([_row_pitch(x0, d, "gated_branches"), _row_pitch(x1, d, "gated_branches"),
                                _row_pitch(x2, d, "gated_branches")])
    y = torch.empty((*x1.shape[:-1], 3 * d), device=dev, dtype=torch.float32)
    _lib.launch("tf_gated_branches_fwd", dev, x0.data_ptr(), x1.data_ptr(), x2.data_ptr(),
                _lib.dtype_code(x0, "gated_branches"), pitches, gate.data_ptr(),
                _lib.dtype_code(gate, "gated_branches"), y.data_ptr(), rows, d)
    return y
