"""Audio files to model input: WAV decoding, exact 16-kHz preprocessing and length
buckets (reference ``audio.py:12-95``).

``inspect_audio`` reads a file's header into an ``AudioFile`` record;
``decode_audio`` reads the samples as float32, resamples to 16 kHz with
``scipy.signal.resample_poly`` (up/down factors reduced by their gcd) and
quantises to the PCM16 grid, ``clip(rint(x * 32768), -32768, 32767) / 32768``
(the reference's canonical preprocessing, ``audio.py:35-49``);
``plan_batches`` groups clips by (channels, bucket length) and
``decoded_batches`` decodes a plan with a thread pool, at most two batches ahead.

The reference reads files through ``soundfile`` (libsndfile). That library is not
part of this package's environment, so files are read by the RIFF/WAVE reader
below: PCM (unsigned 8-bit, 16/24/32-bit integer) and IEEE float (32/64-bit),
plain or WAVE_FORMAT_EXTENSIBLE, scaled to float32 the way libsndfile does
(integer samples divided by 2^(bits-1)). Other containers (FLAC, Ogg, MP3) raise
``ValueError``.
"""

from __future__ import annotations

import math
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from pathlib import Path

import numpy as np

SAMPLE_RATE = 16000
MAX_SAMPLES = 72 * SAMPLE_RATE
BUCKET_SECONDS = (4, 8, 12, 16, 24, 32, 40, 48, 60, 72)

_PCM, _FLOAT, _EXTENSIBLE = 1, 3, 0xFFFE


@dataclass(frozen=True)
class AudioFile:
    index: int
    path: Path
    samples: int
    channels: int


@dataclass(frozen=True)
class WavInfo:
    frames: int
    samplerate: int
    channels: int
    format_tag: int
    bits: int
    data_offset: int
    data_bytes: int


def wav_info(path) -> WavInfo:
    """Header of a RIFF/WAVE file (format, rate, channels, sample layout)."""
    with open(path, "rb") as f:
        head = f.read(12)
        if len(head) < 12 or head[:4] != b"RIFF" or head[8:12] != b"WAVE":
            raise ValueError(f"Unsupported audio container (only WAV is readable here): {path}")
        fmt = None
        while True:
            hdr = f.read(8)
            if len(hdr) < 8:
                raise ValueError(f"WAV file without a data chunk: {path}")
            cid, size = hdr[:4], struct.unpack("<I", hdr[4:])[0]
            if cid == b"fmt ":
                body = f.read(size)
                tag, channels, rate, _, _, bits = struct.unpack("<HHIIHH", body[:16])
                if tag == _EXTENSIBLE and len(body) >= 26:
                    tag = struct.unpack("<H", body[24:26])[0]  # first field of the sub-format GUID
                fmt = (tag, channels, rate, bits)
            elif cid == b"data":
                if fmt is None:
                    raise ValueError(f"WAV data before its format chunk: {path}")
                tag, channels, rate, bits = fmt
                if tag not in (_PCM, _FLOAT) or channels < 1 or bits % 8 or not bits:
                    raise ValueError(f"Unsupported WAV sample format (tag {tag}, {bits} bits): {path}")
                if tag == _FLOAT and bits not in (32, 64):
                    raise ValueError(f"Unsupported WAV float width ({bits} bits): {path}")
                frames = size // (channels * bits // 8)
                return WavInfo(frames, rate, channels, tag, bits, f.tell(), frames * channels * bits // 8)
            else:
                f.seek(size + (size & 1), 1)
            if cid == b"fmt " and size & 1:
                f.seek(1, 1)


def read_wav(path):
    """Samples of a WAV file as float32 ``[frames, channels]`` and its sample rate."""
    info = wav_info(path)
    with open(path, "rb") as f:
        f.seek(info.data_offset)
        raw = f.read(info.data_bytes)
    width = info.bits // 8
    if info.format_tag == _FLOAT:
        x = np.frombuffer(raw, dtype="<f4" if width == 4 else "<f8").astype(np.float32)
    elif width == 1:
        x = (np.frombuffer(raw, dtype=np.uint8).astype(np.float32) - 128.0) / 128.0
    elif width == 2:
        x = np.frombuffer(raw, dtype="<i2").astype(np.float32) / 32768.0
    elif width == 3:
        b = np.frombuffer(raw, dtype=np.uint8).reshape(-1, 3).astype(np.int32)
        v = b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)
        v = np.where(v >= 1 << 23, v - (1 << 24), v)
        x = v.astype(np.float32) / float(1 << 23)
    elif width == 4:
        x = (np.frombuffer(raw, dtype="<i4").astype(np.float64) / float(1 << 31)).astype(np.float32)
    else:
        raise ValueError(f"Unsupported WAV sample width ({info.bits} bits): {path}")
    return x.reshape(-1, info.channels), info.samplerate


def inspect_audio(index, path):
    """The record of one file: 16-kHz sample count and channels (reference ``audio.py:24-30``)."""
    path = Path(path)
    info = wav_info(path)
    samples = math.ceil(info.frames * SAMPLE_RATE / info.samplerate)
    if info.channels not in (1, 2) or not 0 < samples <= MAX_SAMPLES:
        raise ValueError(f"Unsupported audio dimensions: {path}")
    return AudioFile(index, path, samples, info.channels)


def decode_audio(record):
    """``[channels, samples]`` float32 tensor on the PCM16 grid (reference ``audio.py:33-49``)."""
    import torch
    from scipy.signal import resample_poly

    audio, sr = read_wav(record.path)
    if sr != SAMPLE_RATE:
        divisor = math.gcd(sr, SAMPLE_RATE)
        audio = resample_poly(audio, SAMPLE_RATE // divisor, sr // divisor, axis=0).astype(np.float32)
    if len(audio) != record.samples or audio.shape[1] != record.channels or not np.isfinite(audio).all():
        raise ValueError(f"Audio metadata or finite-value check failed: {record.path}")
    pcm = np.clip(np.rint(audio * 32768), -32768, 32767).astype(np.int16)
    return torch.from_numpy(np.ascontiguousarray((pcm.astype(np.float32) / 32768).T))


def bucket_samples(samples):
    """Padded length (samples) of the smallest bucket that holds `samples`."""
    for seconds in BUCKET_SECONDS:
        if samples <= seconds * SAMPLE_RATE:
            return seconds * SAMPLE_RATE
    raise ValueError(f"clip of {samples} samples exceeds the {MAX_SAMPLES}-sample limit")


def plan_batches(records, padded_seconds=120, max_batch=16, round_buckets=True):
    """``[(padded_samples, [records...]), ...]`` in (channels, length) order.

    Batch size per group = max(1, min(max_batch, padded_seconds * 16000 // length)).
    """
    groups = {}
    for r in records:
        limit = bucket_samples(r.samples) if round_buckets else r.samples
        groups.setdefault((r.channels, limit), []).append(r)
    plan = []
    for (_, limit), rows in sorted(groups.items()):
        size = max(1, min(max_batch, int(padded_seconds * SAMPLE_RATE) // limit))
        plan.extend((limit, rows[i:i + size]) for i in range(0, len(rows), size))
    return plan


def decoded_batches(plan, workers=4):
    """Decode a plan batch by batch (reference ``audio.py:69-95``): files are decoded
    on a thread pool, at most two batches are pending, and each batch is a zero-padded
    ``[n, channels, limit]`` float32 tensor (pinned when a GPU is present) with its
    lengths, channels and clip indices."""
    import torch

    with ThreadPoolExecutor(max_workers=workers) as pool:
        iterator = iter(plan)

        def submit():
            try:
                limit, rows = next(iterator)
            except StopIteration:
                return None
            return limit, rows, [pool.submit(decode_audio, r) for r in rows]

        pending = submit()
        while pending is not None:
            limit, rows, futures = pending
            pending = submit()
            audio = torch.zeros(len(rows), rows[0].channels, limit, pin_memory=torch.cuda.is_available())
            for i, (record, future) in enumerate(zip(rows, futures)):
                audio[i, :, :record.samples] = future.result()
            yield dict(audio=audio, lengths=torch.tensor([r.samples for r in rows]),
                       channels=torch.tensor([r.channels for r in rows]), indices=[r.index for r in rows])
