"""Spectrogram front end (reference ``front.py``): STFT power on cuFFT, three
residual Conv2d stages on cuDNN, and frequency band pooling.

Parameter names match the reference's checkpoints. The convolutions and the
STFT are library calls; on the optimized backend the activations stay
channels-last and the masked channel norms (+SiLU), the residual tails and the
band pooling run as single-pass kernels of ``libtrifusion_b200.so``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .kernels import RMSNorm
from .masking import time_mask


def _channel_norm(x, norm, valid):
    """RMSNorm over the channels of ``x`` [B, C, T, F] at every (t, f), with
    invalid time steps zeroed first; returns [B, C, T, F] (channels-last strides)."""
    rows = x.masked_fill(~valid, 0).permute(0, 2, 3, 1)
    return norm(rows.contiguous()).permute(0, 3, 1, 2)


class CNNStage(nn.Module):
    """Residual stage: conv3x3 (time stride, freq stride 2) → norm → SiLU →
    conv3x3 → norm, plus a 1x1 strided skip (reference ``front.py:8-43``)."""

    def __init__(self, cin, cout, stride, backend):
        super().__init__()
        self.stride = stride
        self.backend = backend
        self.buffer_fusion = False
        self.conv1 = nn.Conv2d(cin, cout, 3, stride=(stride, 2), padding=1, bias=False)
        self.conv2 = nn.Conv2d(cout, cout, 3, padding=1, bias=False)
        self.skip = nn.Conv2d(cin, cout, 1, stride=(stride, 2), bias=False)
        self.norm1, self.norm2 = RMSNorm(cout, backend=backend), RMSNorm(cout, backend=backend)

    def _stem_fusable(self, x):
        """The 1 -> 32 channel, time-stride-1 first stage under BF16 autocast."""
        return (self.stride == 1 and x.shape[1] == 1 and self.conv1.weight.shape[0] == 32
                and x.dtype == torch.float32 and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") == torch.bfloat16)

    def _skip_rows(self, x):
        """The strided 1x1 skip convolution of channels-last ``x`` as one GEMM over the
        subsampled positions: ``skip(x)[b, :, t, f] = W x[b, :, s t, 2 f]``, returned
        channels-last. (For these shapes cuDNN's heuristics pick kernels several
        times slower than the GEMM plus the gather of the subsampled rows.)"""
        rows = x.permute(0, 2, 3, 1)[:, ::self.stride, ::2, :]  # [B, T', F', C], a strided view
        b, tp, fp, c = rows.shape
        w = self.skip.weight.reshape(self.skip.weight.shape[0], c)
        return F.linear(rows.reshape(-1, c), w).view(b, tp, fp, -1).permute(0, 3, 1, 2)

    def forward(self, x, lengths):
        lengths = (lengths + self.stride - 1) // self.stride
        if self.backend != "reference" and x.is_cuda:
            # Channels-last activations: each channel norm reads contiguous rows,
            # and mask + norm + SiLU (and the residual tail) are one pass each.
            from .kernels.buffers import front_norm, front_residual, front_stem

            if self._stem_fusable(x):
                # First stage: both convolutions of the single input channel, the
                # first norm and SiLU in one pass over the spectrogram.
                h, skip = front_stem(x, lengths, self.conv1, self.skip, self.norm1)
                h = front_norm(self.conv2(h), lengths, self.norm2)
                return front_residual(h, skip, lengths)
            x = x.contiguous(memory_format=torch.channels_last)
            h = front_norm(self.conv1(x), lengths, self.norm1, silu=True)
            h = front_norm(self.conv2(h), lengths, self.norm2)
            # BF16 activations (the autocast path): the skip as a gather + GEMM. FP32 ones keep
            # cuDNN's convolution, whose TF32 setting the GEMM would not share.
            skip = self._skip_rows(x) if x.dtype == torch.bfloat16 else self.skip(x)
            return front_residual(h, skip, lengths)
        h = self.conv1(x)
        valid = time_mask(lengths, h.shape[2])[:, None, :, None]
        # A zero row stays zero through the bias-free norm and SiLU, so masking
        # before each norm is enough; the stage output is masked once more.
        h = F.silu(_channel_norm(h, self.norm1, valid))
        h = _channel_norm(self.conv2(h), self.norm2, valid)
        skip = self.skip(x).masked_fill(~valid, 0)
        return F.silu(h + skip).masked_fill(~valid, 0)


def band_pool(x, native=False):
    """Average the frequency axis of [B, C, T, F] into 8 bands → [B, T, 8, C]
    (band i covers [floor(iF/8), ceil((i+1)F/8)); reference ``front.py:80-87``)."""
    if native and x.is_cuda:
        from .kernels.native import bands

        return bands(x)
    return F.adaptive_avg_pool2d(x, (x.shape[2], 8)).permute(0, 2, 3, 1).contiguous()


class Frontend(nn.Module):
    """Log-power STFT (n_fft 512, hop 160, Hann 400) and three CNN stages
    (reference ``front.py:46-114``)."""

    def __init__(self, backend="l4", channels_last=True, checkpoint_stages=False):
        super().__init__()
        self.backend, self.native_kernels = backend, False
        self.register_buffer("window", torch.hann_window(400, periodic=True), persistent=False)
        self.stages = nn.ModuleList([
            CNNStage(1, 32, 1, backend),
            CNNStage(32, 64, 2, backend),
            CNNStage(64, 128, 2, backend),
        ])
        self.channels_last, self.checkpoint_stages = channels_last, checkpoint_stages
        if channels_last:
            self.to(memory_format=torch.channels_last)

    def main_lengths(self, sample_lengths):
        """Valid frames at the main (stage-3) rate for `sample_lengths` samples."""
        lengths = sample_lengths // 160 + 1
        for stage in self.stages:
            lengths = (lengths + stage.stride - 1) // stage.stride
        return lengths

    def spectrogram(self, audio, sample_lengths, channels):
        b, c, n = audio.shape
        with torch.autocast(device_type=audio.device.type, enabled=False):
            keep = time_mask(sample_lengths, n)[:, None, :]
            keep = keep & (torch.arange(c, device=audio.device)[None, :, None] < channels[:, None, None])
            wave = torch.where(keep, audio.float(), 0.0)
            spec = torch.stft(wave.reshape(b * c, n), n_fft=512, hop_length=160, win_length=400,
                              window=self.window.float(), center=True, pad_mode="constant",
                              return_complex=True)
            power = (spec.real.square() + spec.imag.square()).reshape(b, c, 257, -1).sum(1)
            power = power / channels[:, None, None]
            log = torch.log(power + 1e-6).transpose(1, 2).unsqueeze(1)
            lengths = sample_lengths // 160 + 1
            log = log.masked_fill(~time_mask(lengths, log.shape[2])[:, None, :, None], 0)
        return log, lengths

    def forward(self, audio, sample_lengths, channels):
        x, lengths = self.spectrogram(audio, sample_lengths, channels)
        if self.channels_last:
            x = x.contiguous(memory_format=torch.channels_last)
        fine = fine_lengths = None
        for i, stage in enumerate(self.stages):
            x = stage(x, lengths)
            lengths = (lengths + stage.stride - 1) // stage.stride
            if i == 1:
                fine, fine_lengths = band_pool(x, self.native_kernels), lengths
        return band_pool(x, self.native_kernels).flatten(2), fine, lengths, fine_lengths
