"""WAV decoding, 16-kHz resampling and PCM16 quantisation (reference audio.py:12-95).

The canonical case is the reference's own (tests/test_submission.py:63-82): a
stereo 44.1 kHz float32 file of N(0, 0.1) noise from ``default_rng(77)``, decoded
and compared bit for bit with ``clip(rint(resample_poly(x, 160, 441) * 32768))
/ 32768``. The reference writes its files with soundfile; here they are written
by the small RIFF writer below (soundfile is not installed), in the same formats.
"""

import struct

import numpy as np
import pytest
import torch
from scipy.signal import resample_poly

from trifusion_b200.audio import (AudioFile, decode_audio, decoded_batches, inspect_audio, plan_batches,
                                  read_wav)


def write_wav(path, data, rate, kind="float32"):
    """RIFF/WAVE file of ``data`` [frames, channels]: kind float32, float64, pcm16, pcm24, pcm8."""
    data = np.asarray(data)
    if data.ndim == 1:
        data = data[:, None]
    frames, channels = data.shape
    if kind in ("float32", "float64"):
        tag, bits = 3, 32 if kind == "float32" else 64
        payload = data.astype("<f4" if bits == 32 else "<f8").tobytes()
    elif kind == "pcm16":
        tag, bits = 1, 16
        payload = data.astype("<i2").tobytes()
    elif kind == "pcm24":
        tag, bits = 1, 24
        v = data.astype(np.int32).reshape(-1) & 0xFFFFFF
        payload = np.stack([v & 0xFF, (v >> 8) & 0xFF, (v >> 16) & 0xFF], 1).astype(np.uint8).tobytes()
    elif kind == "pcm8":
        tag, bits = 1, 8
        payload = data.astype(np.uint8).tobytes()
    else:
        raise ValueError(kind)
    block = channels * bits // 8
    fmt = struct.pack("<HHIIHH", tag, channels, rate, rate * block, block, bits)
    body = b"WAVE" + b"fmt " + struct.pack("<I", len(fmt)) + fmt + b"data" + struct.pack("<I", len(payload)) + payload
    path.write_bytes(b"RIFF" + struct.pack("<I", len(body)) + body)
    return path


def expected_pcm16(x, rate):
    if rate != 16000:
        g = np.gcd(rate, 16000)
        x = resample_poly(x, 16000 // g, rate // g, axis=0).astype(np.float32)
    return (np.clip(np.rint(x * 32768), -32768, 32767).astype(np.int16).astype(np.float32) / 32768).T


def test_canonical_resampling_and_quantization(tmp_path):
    rng = np.random.default_rng(77)
    source = rng.normal(0, 0.1, (44100, 2)).astype(np.float32)
    path = write_wav(tmp_path / "stereo.wav", source, 44100)
    record = inspect_audio(0, path)
    assert (record.samples, record.channels) == (16000, 2)
    actual = decode_audio(record).numpy()
    np.testing.assert_array_equal(actual, expected_pcm16(source, 44100))


@pytest.mark.parametrize("kind,rate,channels", [("pcm16", 16000, 1), ("pcm24", 48000, 2), ("pcm8", 8000, 1),
                                                ("float64", 22050, 2)])
def test_integer_and_double_formats(tmp_path, kind, rate, channels):
    rng = np.random.default_rng(5)
    n = rate // 2 + 7
    if kind == "pcm16":
        ints = rng.integers(-32768, 32768, (n, channels))
        scaled = ints / 32768.0
    elif kind == "pcm24":
        ints = rng.integers(-(1 << 23), 1 << 23, (n, channels))
        scaled = ints / float(1 << 23)
    elif kind == "pcm8":
        ints = rng.integers(0, 256, (n, channels))
        scaled = (ints - 128) / 128.0
    else:
        ints = rng.normal(0, 0.2, (n, channels))
        scaled = ints
    path = write_wav(tmp_path / f"{kind}.wav", ints, rate, kind)
    x, sr = read_wav(path)
    assert sr == rate and x.dtype == np.float32
    np.testing.assert_array_equal(x, scaled.astype(np.float32))
    record = inspect_audio(3, path)
    assert record.samples == -(-n * 16000 // rate) and record.channels == channels
    np.testing.assert_array_equal(decode_audio(record).numpy(), expected_pcm16(scaled.astype(np.float32), rate))


def test_rejections(tmp_path):
    with pytest.raises(ValueError, match="Unsupported audio dimensions"):
        inspect_audio(0, write_wav(tmp_path / "three.wav", np.zeros((100, 3), np.float32), 16000))
    with pytest.raises(ValueError, match="Unsupported audio dimensions"):
        inspect_audio(0, write_wav(tmp_path / "long.wav", np.zeros(72 * 16000 + 1, np.float32), 16000))
    bad = np.zeros(1600, np.float32)
    bad[5] = np.nan
    record = inspect_audio(0, write_wav(tmp_path / "nan.wav", bad, 16000))
    with pytest.raises(ValueError, match="finite-value"):
        decode_audio(record)
    (tmp_path / "x.flac").write_bytes(b"fLaC" + bytes(40))
    with pytest.raises(ValueError, match="only WAV"):
        inspect_audio(0, tmp_path / "x.flac")


def test_decoded_batches_pad_and_order(tmp_path):
    rng = np.random.default_rng(9)
    records = []
    for i, (sec, ch) in enumerate([(1.5, 1), (3.0, 1), (0.5, 2), (5.0, 1)]):
        x = rng.normal(0, 0.1, (int(sec * 16000), ch)).astype(np.float32)
        records.append(inspect_audio(i, write_wav(tmp_path / f"{i}.wav", x, 16000)))
    plan = plan_batches(records, padded_seconds=8, max_batch=2)
    seen = []
    for batch, (limit, rows) in zip(decoded_batches(plan, workers=2), plan):
        a = batch["audio"]
        assert a.shape == (len(rows), rows[0].channels, limit)
        for j, r in enumerate(rows):
            assert int(batch["lengths"][j]) == r.samples and int(batch["channels"][j]) == r.channels
            assert torch.equal(a[j, :, :r.samples], decode_audio(r))
            assert not a[j, :, r.samples:].any()
        seen += batch["indices"]
    assert sorted(seen) == [0, 1, 2, 3]
    assert isinstance(records[0], AudioFile)
