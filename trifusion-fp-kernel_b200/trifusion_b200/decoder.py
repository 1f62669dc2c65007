"""Classification decoder with the reference's parameter layout (reference
``decoder.py``). On the GPU the masked time mean, the last-valid-row read of the
forward Mamba output and the two query reads run on kernels of
``libtrifusion_b200.so``; under BF16 autocast so does the tail (top-k local
evidence, the voice/music/file heads and the logits row). The projections
before the tail are cuBLAS GEMMs.
"""

from __future__ import annotations

import torch
from torch import nn

from .attention import masked_attention
from .masking import time_mask


def sin_position(time, dim, device):
    """Interleaved (sin, cos) position code of width ``dim`` (``decoder.py:9-15``)."""
    inv = torch.pow(10000.0, -torch.arange(0, dim, 2, device=device).float() / dim)
    angle = torch.outer(torch.arange(time, device=device).float(), inv)
    return torch.stack((angle.sin(), angle.cos()), -1).flatten(-2)


_POSITIONS = {}


def _position_table(time, dim, device, dtype):
    """``sin_position(time, dim)`` in ``dtype``, computed once per (time, device, dtype):
    a constant table, so steady-state forwards launch nothing for it."""
    key = (time, dim, str(device), dtype)
    table = _POSITIONS.get(key)
    if table is None:
        table = _POSITIONS[key] = sin_position(time, dim, device).to(dtype)
    return table


class QueryRead(nn.Module):
    """10 learned queries × 8 heads of width 32 attend over a sequence; the
    outputs are averaged in groups of 4/4/2 (``decoder.py:18-33``)."""

    def __init__(self, input_dim):
        super().__init__()
        self.kv = nn.Linear(input_dim, 512, bias=False)
        self.q = nn.Linear(256, 256, bias=False)
        self.out = nn.Linear(256, 256, bias=False)

    def _native_rows(self, qp, kv, lengths, keys_per_length):
        if kv.is_cuda and kv.dtype == torch.bfloat16 and qp.dtype == torch.bfloat16:
            from .kernels.native import query_read

            return self.out(query_read(qp, kv, lengths, keys_per_length))
        return None

    def rows(self, query, x, lengths, keys_per_length=1):
        """The out projection's ``[B, 10, 256]`` rows (before the 4/4/2 group means) when
        the split-key kernel applies (GPU, BF16 projections), else None."""
        return self._native_rows(self.q(query), self.kv(x), lengths, keys_per_length)

    def forward(self, query, x, mask, lengths=None, keys_per_length=1):
        """``mask`` [B, T] bool, or None with ``lengths`` given (key j valid when
        ``j < lengths * keys_per_length``). With ``lengths`` on the GPU under BF16
        arithmetic the attention runs as one split-key kernel over the projection
        rows (``native.query_read``)."""
        b, t, _ = x.shape
        kv, qp = self.kv(x), self.q(query)
        h = self._native_rows(qp, kv, lengths, keys_per_length) if lengths is not None else None
        if h is not None:
            return h[:, :4].mean(1), h[:, 4:8].mean(1), h[:, 8:].mean(1)
        if mask is None:
            mask = time_mask(lengths * keys_per_length, t)
        k, v = kv.view(b, t, 2, 8, 32).permute(2, 0, 3, 1, 4).unbind(0)
        q = qp.view(10, 8, 32).transpose(0, 1).unsqueeze(0).expand(b, -1, -1, -1)
        h = masked_attention(q, k, v, mask[:, None, None, :])
        h = self.out(h.transpose(1, 2).reshape(b, 10, 256))
        return h[:, :4].mean(1), h[:, 4:8].mean(1), h[:, 8:].mean(1)


class Decoder(nn.Module):
    def __init__(self, dim):
        super().__init__()
        self.query = nn.Parameter(torch.randn(10, 256) * 0.02)
        self.band = nn.Parameter(torch.randn(8, 64) * 0.02)
        self.deep_read, self.fine_read = QueryRead(dim), QueryRead(64)
        self.global_proj, self.memory_proj = nn.Linear(dim, 256), nn.Linear(2 * dim, 256)
        self.local_logits = nn.Linear(512, 2)
        self.local_features = nn.Linear(512, 256)
        self.voice_lat = nn.Sequential(nn.Linear(1280, 256), nn.SiLU())
        self.music_lat = nn.Sequential(nn.Linear(1280, 256), nn.SiLU())
        self.voice_head, self.music_head = nn.Linear(256, 2), nn.Linear(256, 2)
        self.file_head = nn.Sequential(nn.Linear(1536, 256), nn.SiLU(), nn.Linear(256, 1))
        self.native_kernels = False
        # With native kernels under BF16 autocast: the tail after the query reads as this
        # library's kernels (False keeps the PyTorch tail, e.g. to compare the two).
        self.fused_tail = True

    def _pooled(self, x, mf, lengths, mask):
        if self.native_kernels and x.is_cuda:
            from .kernels.native import end_gather, masked_mean

            return masked_mean(x, lengths), end_gather(mf, lengths)
        mean = (x.float() * mask.unsqueeze(-1)).sum(1) / lengths.unsqueeze(1)
        return mean, mf[torch.arange(x.shape[0], device=x.device), lengths - 1]

    def forward(self, x, fine, grids, fine_lengths, mf, mb):
        b, tf_, _, _ = fine.shape
        fine_mask = time_mask(fine_lengths, tf_)
        native = self.native_kernels and x.is_cuda
        bf16_autocast = (x.is_cuda and torch.is_autocast_enabled("cuda")
                         and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        if native:
            from .kernels.buffers import _param_bf16

            band = _param_bf16(self.band, (8, 64)) if fine.dtype == torch.bfloat16 else self.band.to(fine.dtype)
            fp = fine + _position_table(tf_, 64, fine.device, fine.dtype)[None, :, None, :] + band[None, None]
        else:
            fp = (fine + sin_position(tf_, 64, fine.device)[None, :, None, :].to(fine.dtype)
                  + self.band.to(fine.dtype)[None, None, :, :])
        # The query reads' out-projection rows, from the split-key kernel (GPU, BF16).
        deep_h = fine_h = None
        if native and bf16_autocast:
            deep_h = self.deep_read.rows(self.query, x, grids.lengths)
            fine_h = self.fine_read.rows(self.query, fp.flatten(1, 2), fine_lengths, keys_per_length=8)
        mean, end = self._pooled(x, mf, grids.lengths, grids.mask)
        global_feature = self.global_proj(mean)
        memory = self.memory_proj(torch.cat((end, mb[:, 0]), -1))
        flat = fine.flatten(2)
        if native and bf16_autocast and flat.dtype == torch.bfloat16:
            import torch.nn.functional as F

            from .kernels.buffers import concat_linear

            # local_logits and local_features as one GEMM over the shared input.
            w, bias, offs = concat_linear([self.local_logits, self.local_features], torch.bfloat16)
            both = F.linear(flat, w, bias)
            local, features = both[..., offs[0]:offs[0] + 2], both[..., offs[1]:offs[1] + 256]
        else:
            local, features = self.local_logits(flat), self.local_features(flat)
        if (self.fused_tail and deep_h is not None and fine_h is not None and local.dtype == torch.bfloat16
                and global_feature.dtype == torch.bfloat16 and memory.dtype == torch.bfloat16):
            from .kernels.native import decoder_heads, local_topk

            # The rest is four launches instead of ~40: the top-k evidence over the GEMM's
            # rows, and the heads with the logits row (group means and concatenations read
            # in place).
            local_f32, top = local_topk(local, features, fine_lengths)
            return {
                "logits": decoder_heads(deep_h, fine_h, global_feature, memory, top, self),
                "local_logits": local_f32,
                "local_mask": fine_mask,
                "features": x,
                "feature_mask": grids.mask,
                "embedding": global_feature.float(),
            }
        if deep_h is not None:
            deep_q = (deep_h[:, :4].mean(1), deep_h[:, 4:8].mean(1), deep_h[:, 8:].mean(1))
        else:
            deep_q = self.deep_read(self.query, x, grids.mask)
        if fine_h is not None:
            fine_q = (fine_h[:, :4].mean(1), fine_h[:, 4:8].mean(1), fine_h[:, 8:].mean(1))
        else:
            fine_q = self.fine_read(self.query, fp.flatten(1, 2),
                                    fine_mask[:, :, None].expand(b, tf_, 8).reshape(b, -1))
        k = min(25, tf_)
        scores = local.float().masked_fill(~fine_mask.unsqueeze(-1), -torch.inf)
        idx = scores.transpose(1, 2).topk(k, -1).indices
        picked = features.unsqueeze(1).expand(-1, 2, -1, -1).gather(
            2, idx.unsqueeze(-1).expand(-1, -1, -1, 256))
        valid_k = torch.arange(k, device=x.device)[None, :] < fine_lengths.clamp(max=k)[:, None]
        top = (picked.float() * valid_k[:, None, :, None]).sum(2) / valid_k.sum(1)[:, None, None]
        voice = self.voice_lat(torch.cat((deep_q[0], fine_q[0], global_feature, top[:, 0], memory), -1))
        music = self.music_lat(torch.cat((deep_q[1], fine_q[1], global_feature, top[:, 1], memory), -1))
        v, m = self.voice_head(voice), self.music_head(music)
        f = self.file_head(torch.cat((deep_q[2], fine_q[2], global_feature, memory, voice, music), -1))
        logits = torch.cat((f, v[:, :1], m[:, :1], v[:, 1:], m[:, 1:]), -1).float()
        return {
            "logits": logits,
            "local_logits": local.float(),
            "local_mask": fine_mask,
            "features": x,
            "feature_mask": grids.mask,
            "embedding": global_feature.float(),
        }
