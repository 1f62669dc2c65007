"""Length masks and the per-batch time grids of the model (reference
``masking.py``): the main-rate mask, the 4x-pooled attention grid, the
interpolation map back to the main rate, and the attention rotary table.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


def time_mask(lengths, time):
    """``[B, time]`` bool, True at steps inside each length (``masking.py:6-7``)."""
    return torch.arange(time, device=lengths.device).unsqueeze(0) < lengths.unsqueeze(1)


def masked(x, mask):
    """Zero the rows of ``x`` ([B, T, ...]) where ``mask`` is False (``masking.py:10-11``)."""
    return torch.where(mask.unsqueeze(-1), x, 0.0)  # a Python scalar: no device fill per call


def rotary_table(steps, head_dim, device):
    """cos/sin of ``t * 10000^(-2i/head_dim)`` for t < steps, i < head_dim/2."""
    inv_freq = torch.pow(10000.0, -torch.arange(0, head_dim, 2, device=device).float() / head_dim)
    angle = torch.outer(torch.arange(steps, device=device).float(), inv_freq)
    return angle.cos(), angle.sin()


@dataclass
class Grids:
    """Time grids of one batch (reference ``masking.py:14-80``)."""

    lengths: torch.Tensor
    mask: torch.Tensor
    low_lengths: torch.Tensor
    low_mask: torch.Tensor
    left: torch.Tensor
    right: torch.Tensor
    alpha: torch.Tensor
    rope_cos: torch.Tensor
    rope_sin: torch.Tensor
    buffer_fusion: bool = False
    native_kernels: bool = False

    @classmethod
    def make(cls, lengths, time, head_dim=64, buffer_fusion=False, native_kernels=False):
        low_lengths = (lengths + 3) // 4
        low_time = (time + 3) // 4
        # Linear interpolation from the pooled grid back to the main grid with
        # half-pixel centres (align_corners=False), per batch entry's own lengths.
        centre = torch.arange(time, device=lengths.device).float().unsqueeze(0) + 0.5
        src = centre * low_lengths.unsqueeze(1) / lengths.unsqueeze(1) - 0.5
        last = (low_lengths - 1).unsqueeze(1)
        src = torch.minimum(src.clamp(min=0), last)
        left = src.long()
        right = torch.minimum(left + 1, last)
        cos, sin = rotary_table(low_time, head_dim, lengths.device)
        return cls(lengths, time_mask(lengths, time), low_lengths, time_mask(low_lengths, low_time),
                   left, right, src - left, cos, sin, buffer_fusion, native_kernels)

    def pool(self, x, out_dtype=None):
        """Mean over groups of 4 valid frames → ``[B, ceil(T/4), D]`` (in ``out_dtype``:
        the means rounded once, or x's type)."""
        if self.buffer_fusion:
            from .kernels.buffers import Pool4

            return Pool4.apply(x.contiguous(), self.lengths, out_dtype)
        b, t, d = x.shape
        pad = (-t) % 4
        xs = torch.nn.functional.pad(masked(x, self.mask).float(), (0, 0, 0, pad))
        ms = torch.nn.functional.pad(self.mask, (0, pad)).view(b, -1, 4)
        total = xs.view(b, -1, 4, d).sum(2)
        return (total / ms.sum(2).clamp(min=1).unsqueeze(-1)).to(out_dtype or x.dtype)

    def interpolate(self, low):
        """Back to the main grid: ``a + (b - a) * alpha`` of the two nearest pooled
        rows, zero past each length."""
        if self.native_kernels and low.is_cuda and low.dtype == torch.bfloat16 and low.shape[-1] % 4 == 0:
            from .kernels.native import interpolate

            return interpolate(low, self)
        idx_shape = (*self.left.shape, low.shape[-1])
        a = low.gather(1, self.left.unsqueeze(-1).expand(idx_shape)).float()
        b = low.gather(1, self.right.unsqueeze(-1).expand(idx_shape)).float()
        y = (a + (b - a) * self.alpha.unsqueeze(-1)).to(low.dtype)
        return masked(y, self.mask)
