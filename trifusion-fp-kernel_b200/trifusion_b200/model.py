"""TriFusion-FP v3 student with the reference's parameter layout (reference
``model.py``), running on the B200 kernels.

Parameter names, shapes and the checkpoint format are the reference's, so its
checkpoints load unchanged (``runtime.load_student``). The optimized backend
(``"l4"``, the name the reference's checkpoints carry) runs these operators on
``libtrifusion_b200.so``: the length mask, the row norms (pre/local/branch/FFN
norms, evidence norm, bidirectional mean norm), Pool4, the fused Mamba-3
recurrence (with its B/C norms, controls and length mask), the valid-prefix
reversal, the branch gate and SwiGLU. GEMMs and convolutions run on
cuBLAS/cuDNN; attention on PyTorch's SDPA in FP32; the depthwise time
convolutions, the rotary q/k (writing the FP32 attention operands) and the
grid interpolation run on the library too.
``backend="reference"`` evaluates the reference's PyTorch formulas instead.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from .attention import masked_attention
from .front import Frontend
from .kernels import RMSNorm, gate_branches, gated_concat, reverse_valid, swiglu
from .masking import Grids, masked


@dataclass
class ModelConfig:
    """The reference's configuration record (``model.py:14-34``); every field is
    kept so that saved ``model_config`` dictionaries load unchanged."""

    dim: int = 1024
    depth: int = 16
    ffn_dim: int = 2816
    heads: int = 16
    state_dim: int = 128
    evidence_rank: int = 64
    dropout: float = 0.1
    backend: str = "l4"
    checkpoint_blocks: bool = False
    checkpoint_frontend: bool = False
    channels_last: bool = False
    buffer_fusion: bool = True
    native_kernels: bool = True
    mamba_packed: bool = True
    paired_mamba: bool = False
    mamba_parallel_bwd: bool = True
    mamba_fast_launch: bool = True
    paired_mamba_grid_limit: int = 64


def mamba_factory(config):
    from .mamba import Mamba3Inference

    return Mamba3Inference(config)


def rope(x, cos, sin):
    """Rotate adjacent (even, odd) pairs of the last dim by the table angles."""
    d = x.shape[-1]
    even, odd = x.float().unflatten(-1, (d // 2, 2)).unbind(-1)
    return torch.stack((even * cos - odd * sin, even * sin + odd * cos), -1).flatten(-2).to(x.dtype)


def _mask_rows(x, mask, optimized):
    if optimized:
        from .kernels.buffers import mask_buffer

        return mask_buffer(x, mask)
    return masked(x, mask)


def _depthwise(x, conv, mask, lengths, optimized):
    """Depthwise Conv1d over time ([B, T, C] layout) with bias, zero past each
    length (the reference's ``depthwise_masked``). The optimized path is one
    channels-last kernel; otherwise cuDNN on the transposed rows."""
    bf16_out = torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
    if optimized and x.is_cuda and bf16_out and x.shape[-1] % 4 == 0:
        from .kernels.buffers import depthwise_masked

        return depthwise_masked(x, conv, lengths)
    dtype = torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype
    y = F.conv1d(x.to(dtype).transpose(1, 2), conv.weight.to(dtype), conv.bias.to(dtype),
                 padding=conv.padding, groups=conv.groups)
    return masked(y.transpose(1, 2), mask)


def _bf16_autocast(x):
    return x.is_cuda and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16


def _plus_depthwise(x, conv, mask, lengths, optimized):
    """``x + depthwise(x)`` as the next projection's input. On the optimized path under
    BF16 autocast this is one kernel returning the sum rounded to BF16 — what autocast
    would pass to the projection; otherwise the FP32 sum."""
    if optimized and _bf16_autocast(x) and x.dtype == torch.float32 and x.shape[-1] % 4 == 0:
        from .kernels.buffers import depthwise_masked

        return depthwise_masked(x, conv, lengths, residual=True)
    return x + _depthwise(x, conv, mask, lengths, optimized)


class LocalCNN(nn.Module):
    """GLU up-projection, depthwise conv (k=7), RMSNorm, SiLU, out-projection."""

    def __init__(self, c):
        super().__init__()
        self.backend = c.backend
        self.buffer_fusion = c.buffer_fusion
        self.native_kernels = c.native_kernels
        self.up = nn.Linear(c.dim, 2 * c.dim, bias=False)
        self.dw = nn.Conv1d(c.dim, c.dim, 7, padding=3, groups=c.dim)
        self.norm = RMSNorm(c.dim, backend=c.backend)
        self.out = nn.Linear(c.dim, c.dim, bias=False)

    def forward(self, x, mask, lengths):
        u = self.up(x)
        if (self.backend != "reference" and _bf16_autocast(u) and u.dtype == torch.bfloat16
                and u.shape[-1] % 8 == 0):
            from .kernels.buffers import glu_depthwise

            h = glu_depthwise(u, self.dw, lengths)  # the GLU formed inside the depthwise pass
        else:
            h = F.glu(u, dim=-1)
            if self.backend == "reference":
                h = masked(h, mask)
            h = _depthwise(h, self.dw, mask, lengths, self.backend != "reference")
        if self.backend != "reference" and h.is_cuda:
            from .kernels import native

            y = self.out(native.rms_silu(h, self.norm.weight, self.norm.eps))  # norm and SiLU, one pass
        else:
            y = self.out(F.silu(self.norm(h)))
        return masked(y, mask) if self.backend == "reference" else y


class GlobalAttention(nn.Module):
    """Attention over the 4x-pooled sequence with rotary q/k, interpolated back."""

    def __init__(self, c):
        super().__init__()
        self.heads, self.head_dim = c.heads, c.dim // c.heads
        self.backend, self.buffer_fusion = c.backend, c.buffer_fusion
        self.native_kernels = c.native_kernels
        self.qkv = nn.Linear(c.dim, 3 * c.dim, bias=False)
        self.out = nn.Linear(c.dim, c.dim, bias=False)

    def forward(self, x, grids):
        # The pooled rows feed only the qkv projection: BF16 under autocast on the optimized path.
        bf16 = self.backend != "reference" and _bf16_autocast(x) and x.dtype == torch.float32
        p = grids.pool(x, torch.bfloat16 if bf16 else None)
        b, t = p.shape[:2]
        qkv = self.qkv(p)
        mask = grids.low_mask[:, None, None, :]
        if (self.backend != "reference" and self.buffer_fusion and qkv.is_cuda and qkv.dtype == torch.bfloat16
                and self.head_dim == 64):
            # One kernel: rotary q/k, FP32 masked attention, rows in the out projection's layout.
            from .kernels.native import pooled_attention

            y = pooled_attention(qkv, grids.rope_cos, grids.rope_sin, grids.low_lengths, self.heads)
            return grids.interpolate(self.out(y))
        if self.backend != "reference" and self.buffer_fusion and qkv.is_cuda and qkv.dtype == torch.bfloat16:
            # One kernel: rotary q/k and the FP32 attention operands.
            from .kernels.buffers import RotaryQKV

            q, k, v = RotaryQKV.apply(qkv, grids.rope_cos, grids.rope_sin, self.heads, torch.float32).unbind(0)
            y = masked_attention(q, k, v, mask, out_dtype=torch.bfloat16)
            y = self.out(y.transpose(1, 2).reshape(b, t, -1))
            return grids.interpolate(y)
        q, k, v = qkv.view(b, t, 3, self.heads, self.head_dim).permute(2, 0, 3, 1, 4).unbind(0)
        q, k = rope(q, grids.rope_cos, grids.rope_sin), rope(k, grids.rope_cos, grids.rope_sin)
        y = masked_attention(q, k, v, mask)
        y = self.out(y.transpose(1, 2).reshape(b, t, -1))
        return grids.interpolate(y)


class TriFusionBlock(nn.Module):
    def __init__(self, c):
        super().__init__()
        d, r = c.dim, c.evidence_rank
        self.backend = c.backend
        self.buffer_fusion = c.buffer_fusion
        self.native_kernels = c.native_kernels
        self.paired_mamba = c.paired_mamba
        self.paired_mamba_grid_limit = c.paired_mamba_grid_limit
        self.pre = RMSNorm(d, backend=c.backend)
        self.local, self.attention = LocalCNN(c), GlobalAttention(c)
        self.cn, self.an, self.mn = [RMSNorm(d, backend=c.backend) for _ in range(3)]
        self.e_down = nn.Linear(2 * d, r)
        self.e_value, self.e_gate = nn.Linear(r, d), nn.Linear(r, d)
        self.u_norm = RMSNorm(d, backend=c.backend)
        self.forward_mamba, self.backward_mamba = mamba_factory(c), mamba_factory(c)
        self.gate = nn.Linear(3 * d, 3)
        self.merge_dw = nn.Conv1d(3 * d, 3 * d, 3, padding=1, groups=3 * d)
        self.merge = nn.Linear(3 * d, d, bias=False)
        self.ff_norm = RMSNorm(d, backend=c.backend)
        self.gate_up = nn.Linear(d, 2 * c.ffn_dim, bias=False)
        self.down = nn.Linear(c.ffn_dim, d, bias=False)
        self.dropout = nn.Dropout(c.dropout)
        # Initialisation of a fresh block (model.py:135-144).
        for layer in (self.e_gate, self.gate):
            nn.init.zeros_(layer.weight)
            nn.init.zeros_(layer.bias)
        nn.init.normal_(self.e_value.weight, std=1e-3)
        nn.init.zeros_(self.e_value.bias)
        with torch.no_grad():
            for layer in (self.merge, self.down):
                layer.weight.mul_(1 / math.sqrt(2 * c.depth))

    def forward(self, x, grids, input_masked=False, need_directions=True):
        """``input_masked``: the rows of ``x`` past each length are already zero (the
        previous block's output on the optimized path), so the input mask is skipped.
        ``need_directions=False``: the two Mamba directions' outputs are not returned
        (None), so the optimized path may form only their mean."""
        mask, lengths = grids.mask, grids.lengths
        opt = self.backend != "reference"

        def keep_zero(value):  # the optimized path's operators already keep padded rows at zero
            return value if opt else masked(value, mask)

        if opt and not input_masked:
            x = _mask_rows(x, mask, True)
        if opt and x.is_cuda and _bf16_autocast(x) and x.dtype == torch.float32 and x.shape[-1] % 4 == 0:
            from .kernels import native

            # The pre-norm writes the FP32 rows (pooled by the attention branch) and their
            # BF16 copy (the local branch's up projection input, autocast's cast) in one pass.
            h, h16 = torch.empty_like(x), torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
            native.rms_into(x, self.pre.weight, self.pre.eps, h, h16)
            local, attended = self.local(h16, mask, lengths), self.attention(h, grids)
        else:
            h = keep_zero(self.pre(x))
            local, attended = self.local(h, mask, lengths), self.attention(h, grids)
        d = local.shape[-1]
        # BF16 branch outputs on the GPU: the cn/an norms write their parts of e_down's
        # input row and of the gate's BF16 input row in place of the two concatenations
        # (and of autocast's cast of the FP32 one); every value is the same.
        split = (opt and x.is_cuda and local.dtype == torch.bfloat16 and attended.dtype == torch.bfloat16
                 and d % 4 == 0)
        if split:
            from .kernels import native

            e_in = local.new_empty(*local.shape[:-1], 2 * d)
            s16 = local.new_empty(*local.shape[:-1], 3 * d)
            cn = native.rms_into(local, self.cn.weight, self.cn.eps, e_in[..., :d], s16[..., :d])
            an = native.rms_into(attended, self.an.weight, self.an.eps, e_in[..., d:], s16[..., 2 * d:])
            z = F.silu(self.e_down(e_in))
        else:
            cn = keep_zero(self.cn(local))
            an = keep_zero(self.an(attended))
            z = F.silu(self.e_down(torch.cat((cn, an), -1)))
        if opt and x.is_cuda:
            from .kernels import native

            # u feeds only the Mamba in_proj GEMMs: under BF16 autocast it is written in BF16
            # (the FP32 result rounded once, as autocast would) instead of being cast twice.
            if _bf16_autocast(x):
                from .kernels.buffers import stacked_linear

                # e_value and e_gate share z: one GEMM over both weights; the norm reads the
                # two halves of its output rows in place.
                w_ev, b_ev, pitch = stacked_linear([self.e_value, self.e_gate], torch.bfloat16)
                ev = F.linear(z, w_ev, b_ev)
                value, gate = ev[..., :d], ev[..., pitch:pitch + d]
            else:
                value, gate = self.e_value(z), self.e_gate(z)
            u = native.evidence_norm(x, value, gate, self.u_norm.weight, mask, self.u_norm.eps,
                                     out_dtype=torch.bfloat16 if _bf16_autocast(x) else torch.float32)
            # Both directions in one launch; the recurrence zeroes rows past each length
            # itself (out_proj has no bias) and runs the backward direction reversed.
            fwd, bwd = self.forward_mamba, self.backward_mamba
            if fwd.fused_recurrence and bwd.fused_recurrence and split and not need_directions:
                from .mamba import bidirectional_rows, paired_mean

                # Both directions' rows side by side, then ONE GEMM over both out_proj weights
                # (halved) gives their mean, rounded once; the norm writes mn and its BF16 copy.
                avg = paired_mean(fwd, bwd, bidirectional_rows(fwd, bwd, u, lengths))
                mn = torch.empty(avg.shape, dtype=torch.float32, device=avg.device)
                native.rms_into(avg, self.mn.weight, self.mn.eps, mn, s16[..., d:2 * d])
                mf = mb = None
            else:
                if fwd.fused_recurrence and bwd.fused_recurrence:
                    from .mamba import bidirectional_pair

                    mf, mb = bidirectional_pair(fwd, bwd, u, lengths)
                else:
                    mf = fwd(u, lengths)
                    mb = reverse_valid(bwd(reverse_valid(u, lengths), lengths), lengths)
                mn = native.mean_norm(mf, mb, self.mn.weight, self.mn.eps,
                                      copy_to=s16[..., d:2 * d] if split else None)
        else:
            evidence = self.e_value(z).float() * (2 * torch.sigmoid(self.e_gate(z).float()))
            u = _mask_rows(self.u_norm(x + evidence), mask, opt)
            mf = _mask_rows(self.forward_mamba(u), mask, opt)
            mb = reverse_valid(self.backward_mamba(reverse_valid(u, lengths, self.backend)),
                               lengths, self.backend)
            mn = keep_zero(self.mn((mf.float() + mb.float()) * 0.5))
        if split:
            from .kernels.buffers import _param_bf16

            # The three-output gate projection and the branch gate in one pass (one warp
            # per row) instead of a GEMM with N = 3 and a second pass.
            v = gate_branches(s16, mn, _param_bf16(self.gate.weight, tuple(self.gate.weight.shape)),
                              None if self.gate.bias is None else _param_bf16(self.gate.bias, (3,)))
        else:
            s = torch.cat((cn, mn, an), -1)
            v = keep_zero(gated_concat(s, self.gate(s), self.backend))
        merged = self.dropout(self.merge(_plus_depthwise(v, self.merge_dw, mask, lengths, opt)))
        if opt and _bf16_autocast(x) and x.dtype == torch.float32 and x.shape[-1] % 4 == 0:
            from .kernels import native

            # The residual sum and ff_norm in one pass; ff_norm feeds only gate_up, so it is
            # written in BF16 (the FP32 norm rounded once, as autocast would).
            r, normed = native.add_rms(x, merged, self.ff_norm.weight, self.ff_norm.eps)
        else:
            r = keep_zero(x + merged)
            normed = self.ff_norm(r)
        f = swiglu(self.gate_up(normed), self.backend)
        y = self.dropout(self.down(f))
        if opt and r.is_cuda and r.dtype == torch.float32 and r.shape[-1] % 4 == 0:
            from .kernels.buffers import masked_add

            out = masked_add(r, y, mask)  # one pass: the residual add and the length mask
        else:
            out = _mask_rows(r + y, mask, opt)
        return out, mf, mb


class TriFusion(nn.Module):
    def __init__(self, config=None):
        super().__init__()
        self.config = config or ModelConfig()
        c = self.config
        if c.dim % c.heads or c.dim % 32:
            raise ValueError("dim must divide attention heads and Mamba headdim")
        self.front = Frontend(c.backend, c.channels_last, c.checkpoint_frontend)
        self.front_projection = nn.Identity() if c.dim == 1024 else nn.Linear(1024, c.dim, bias=False)
        self.blocks = nn.ModuleList([TriFusionBlock(c) for _ in range(c.depth)])
        from .decoder import Decoder

        self.decoder = Decoder(c.dim)
        self.memory_head = nn.Linear(c.dim, 2)
        self.set_buffer_fusion(c.buffer_fusion)
        self.set_native_kernels(c.native_kernels)

    def _set(self, name, value):
        for module in self.modules():
            if hasattr(module, name):
                setattr(module, name, value)

    def set_backend(self, backend):
        """Switch between ``"l4"`` (B200 kernels) and ``"reference"`` formulas."""
        if backend not in ("reference", "l4"):
            raise ValueError(backend)
        self._set("backend", backend)
        self.config.backend = backend

    def set_buffer_fusion(self, enabled):
        self._set("buffer_fusion", bool(enabled))
        self.config.buffer_fusion = bool(enabled)

    def set_native_kernels(self, enabled):
        self._set("native_kernels", bool(enabled))
        self.config.native_kernels = bool(enabled)

    def encode(self, audio, lengths, channels):
        x, fine, main_lengths, fine_lengths = self.front(audio, lengths, channels)
        x = self.front_projection(x).float()
        optimized = self.config.backend == "l4"
        grids = Grids.make(main_lengths, x.shape[1], self.config.dim // self.config.heads,
                           self.config.buffer_fusion and optimized,
                           self.config.native_kernels and optimized)
        mf = mb = None
        for i, block in enumerate(self.blocks):
            # Each optimized block's output is zero past the lengths: the next one needn't mask it.
            # Only the last block's per-direction outputs reach the decoder.
            x, mf, mb = block(x, grids, input_masked=optimized and i > 0,
                              need_directions=i == len(self.blocks) - 1)
        return x, fine, grids, fine_lengths, mf, mb

    def forward(self, audio, lengths, channels):
        return self.decoder(*self.encode(audio, lengths, channels))
