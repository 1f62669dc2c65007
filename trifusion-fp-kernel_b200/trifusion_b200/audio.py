"""Length buckets for batched inference (reference ``audio.py:12-66``).

Clips are grouped by (channels, bucket length) — the bucket is the smallest of
``BUCKET_SECONDS`` that holds the clip — and each group is cut into batches of
at most ``max_batch`` clips whose padded length totals about
``padded_seconds``. File decoding (``soundfile``/``resample_poly``) is not part
of this package; callers hand over clips as records with their sample counts.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

SAMPLE_RATE = 16000
MAX_SAMPLES = 72 * SAMPLE_RATE
BUCKET_SECONDS = (4, 8, 12, 16, 24, 32, 40, 48, 60, 72)


@dataclass(frozen=True)
class AudioFile:
    index: int
    path: Path
    samples: int
    channels: int


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
