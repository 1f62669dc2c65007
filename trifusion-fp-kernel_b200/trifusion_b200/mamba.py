"""Frozen Mamba-3 SISO layer with the reference's parameter layout (reference
``mamba.py``), running the B200 recurrence.

Optimized path (``fused_recurrence=True``, what ``load_student`` sets): one
cuBLAS GEMM (``in_proj``, both directions of a pair in one, rows padded to 16 bytes),
ONE recurrence launch that also computes the A/dt
controls from the projection, applies the C/B RMSNorm of the raw q/k rows and
the length mask, and one cuBLAS GEMM (``out_proj``); ``bidirectional_pair``
runs a block's two directions in one launch. With ``fused_recurrence=False``
the controls, norms and mask run as separate kernels around ``fused_mamba``
(the reference's unfused arrangement); ``backend="reference"`` evaluates the
norms and controls with the reference's PyTorch formulas.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .kernels import RMSNorm


def projections(mods, u):
    """``[m.in_proj(u) for m in mods]`` as ONE GEMM over the stacked weights, each padded
    with zero rows to a multiple of 8: views of a ``[..., len(mods) * pitch]`` output whose
    rows are 16-byte aligned
    (the in_proj width, 1860 at dim 384, is not a multiple of 8; cuBLAS then falls
    back to kernels without TMA). The operands are what ``in_proj`` would use: under
    autocast the weights in the autocast type, otherwise in their own type."""
    from .kernels.buffers import stacked_linear

    dev = u.device.type
    dtype = torch.get_autocast_dtype(dev) if torch.is_autocast_enabled(dev) else mods[0].in_proj.weight.dtype
    w, _, pitch = stacked_linear([m.in_proj for m in mods], dtype, multiple=8)
    width = mods[0].in_proj.weight.shape[0]
    p = F.linear(u, w)
    return [p[..., i * pitch:i * pitch + width] for i in range(len(mods))]


def paired_mean(fwd, bwd, y):
    """``(fwd.out_proj(y_f) + bwd.out_proj(y_b)) / 2`` for ``y = [y_f | y_b]`` (rows of
    ``2 * d_inner``) as ONE GEMM over K = 2 * d_inner with the two weights side by side
    and halved (exact in binary floating point): the mean is rounded once, in the
    GEMM's output type, instead of each projection being rounded before the average."""
    dev = y.device.type
    dtype = torch.get_autocast_dtype(dev) if torch.is_autocast_enabled(dev) else fwd.out_proj.weight.dtype
    from .kernels.buffers import _STACKED

    wf, wb = fwd.out_proj.weight, bwd.out_proj.weight
    w = _STACKED.get(("paired_mean", id(wf), id(wb), dtype), (wf, wb),
                     lambda: (0.5 * torch.cat((wf.detach().float(), wb.detach().float()), 1)).to(dtype))
    return F.linear(y, w)


def bidirectional_rows(fwd, bwd, u, lengths):
    """Both directions of a block in one recurrence launch (as ``bidirectional_pair``),
    written side by side into one BF16 ``[B, T, 2 * d_inner]`` row buffer, forward
    half first (the launch takes output strides)."""
    from .mamba_fused import fused_recurrence_multi

    b, t, _ = u.shape
    e = fwd.d_inner
    pf, pb = projections([fwd, bwd], u) if u.is_cuda else (fwd.in_proj(u), bwd.in_proj(u))
    y = torch.empty(b, t, 2 * e, dtype=torch.bfloat16, device=u.device)
    df, db = fwd._direction(pf, b, t), bwd._direction(pb, b, t, reverse=True)
    df["out"] = y[..., :e].view(b, t, fwd.nheads, fwd.headdim)
    db["out"] = y[..., e:].view(b, t, bwd.nheads, bwd.headdim)
    fused_recurrence_multi([df, db], lengths=lengths, eps=fwd.C_norm.eps)
    return y


class Mamba3Inference(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.d_inner = config.dim * 2
        self.nheads = self.d_inner // 64
        self.headdim = 64
        self.d_state = config.state_dim
        self.num_bc_heads = 1
        self.num_rope_angles = self.d_state // 4
        self.A_floor = 1e-4
        self.chunk_size = 64
        self.backend = config.backend
        width = 2 * self.d_inner + 2 * self.d_state + 3 * self.nheads + self.num_rope_angles
        self.in_proj = nn.Linear(config.dim, width, bias=False)
        self.out_proj = nn.Linear(self.d_inner, config.dim, bias=False)
        self.dt_bias = nn.Parameter(torch.full((self.nheads,), -4.0))
        self.B_bias = nn.Parameter(torch.ones(self.nheads, 1, self.d_state))
        self.C_bias = nn.Parameter(torch.ones_like(self.B_bias))
        self.D = nn.Parameter(torch.ones(self.nheads))
        self.B_norm = RMSNorm(self.d_state, backend=config.backend)
        self.C_norm = RMSNorm(self.d_state, backend=config.backend)
        self.fused_recurrence = False

    def _split(self, p):
        n, h, e = self.d_state, self.nheads, self.d_inner
        return p.split([e, e, n, n, h, h, h, self.num_rope_angles], -1)

    def _controls(self, a, ddt):
        if self.backend == "reference":
            af = a.float()
            decay = -(af.clamp(min=0) + 1 / (1 - af.clamp(max=0))).clamp(min=self.A_floor)
            dt = F.softplus(ddt.float() + self.dt_bias)
            return (decay * dt).transpose(1, 2).contiguous(), dt.transpose(1, 2).contiguous()
        from .kernels.buffers import mamba_controls

        return mamba_controls(a, ddt, self.dt_bias, self.A_floor)

    def _direction(self, p, b, t, reverse=False):
        """Arguments of one fused launch from the projection ``p``: the C/B norms,
        the controls (from the a/ddt views) and the length mask run inside it."""
        z, v, k, q, ddt, a, trap, angles = self._split(p)
        heads = (b, t, self.nheads, self.headdim)
        return dict(q=q.reshape(b, t, 1, self.d_state), k=k.reshape(b, t, 1, self.d_state),
                    v=v.reshape(heads), z=z.reshape(heads), trap=trap.transpose(1, 2),
                    angles=angles.unsqueeze(2).expand(b, t, self.nheads, self.num_rope_angles),
                    qb=self.C_bias[:, 0], kb=self.B_bias[:, 0], d=self.D, a_raw=a, ddt_raw=ddt,
                    dt_bias=self.dt_bias, a_floor=self.A_floor, q_norm=self.C_norm.weight,
                    k_norm=self.B_norm.weight, reverse=reverse)

    def forward(self, u, lengths=None):
        """``u`` [B, T, dim] → [B, T, dim]. With ``lengths`` ([B] int64), rows at
        or past each length come out zero (the block's length mask)."""
        b, t, _ = u.shape
        if self.fused_recurrence and self.backend != "reference":
            from .mamba_fused import fused_recurrence_multi

            p = projections([self], u)[0] if u.is_cuda else self.in_proj(u)
            y = fused_recurrence_multi([self._direction(p, b, t)], lengths=lengths, eps=self.C_norm.eps)[0]
            return self._out(y, b, t)
        p = self.in_proj(u)
        z, v, k, q, ddt, a, trap, angles = self._split(p)
        adt, dt = self._controls(a, ddt)
        angles = angles.unsqueeze(2).expand(b, t, self.nheads, self.num_rope_angles)
        heads = (b, t, self.nheads, self.headdim)
        q = q.reshape(b, t, 1, self.d_state)
        k = k.reshape(b, t, 1, self.d_state)
        from .mamba_fused import fused_mamba

        y = fused_mamba(self.C_norm(q), self.B_norm(k), v.reshape(heads), adt, dt, trap.transpose(1, 2),
                        self.C_bias[:, 0], self.B_bias[:, 0], angles, self.D, z.reshape(heads))
        if lengths is not None:
            from .masking import masked, time_mask

            y = masked(y.reshape(b, t, -1), time_mask(lengths, t))
        return self._out(y, b, t)

    def _out(self, y, b, t):
        y = y.reshape(b, t, self.d_inner)
        if not torch.is_autocast_enabled(y.device.type):
            y = y.to(self.out_proj.weight.dtype)
        return self.out_proj(y)


def bidirectional_pair(fwd, bwd, u, lengths):
    """Both directions of a block (model.py:175-179) in one recurrence launch.

    The backward direction reads and writes every row's valid prefix in reverse
    time order inside the launch. ``in_proj`` and ``out_proj`` act row by row and
    rows past the length are zero, so this equals
    ``reverse_valid(bwd(reverse_valid(u)))`` without the two copies. Returns the
    two directions' outputs, both in forward time order, zero past the lengths.
    """
    from .mamba_fused import fused_recurrence_multi

    b, t, _ = u.shape
    pf, pb = projections([fwd, bwd], u) if u.is_cuda else (fwd.in_proj(u), bwd.in_proj(u))
    yf, yb = fused_recurrence_multi([fwd._direction(pf, b, t), bwd._direction(pb, b, t, reverse=True)],
                                    lengths=lengths, eps=fwd.C_norm.eps)
    return fwd._out(yf, b, t), bwd._out(yb, b, t)
