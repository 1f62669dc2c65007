"""Helpers to load the committed golden vectors (tests/golden/*.npz)."""

import ast
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def recurrence_cases():
    return sorted(p.stem for p in GOLDEN.glob("rec_*.npz"))


def load_case(name):
    data = dict(np.load(GOLDEN / f"{name}.npz"))
    shape = tuple(int(x) for x in data["shape"])
    kw = dict(ast.literal_eval(str(data["kw"])))
    return shape, kw, data


def input_checksum(arrays):
    """Same checksum as make_golden.checksum, on numpy arrays."""
    total = 0.0
    for i, a in enumerate(arrays):
        x = np.ascontiguousarray(np.asarray(a, dtype=np.float64)).reshape(-1)
        w = np.cos(np.arange(x.size) * 0.37 + i)
        total += float((x * w).sum())
    return total


def compare_packed(actual, data):
    """Max abs error and the reference scale, for a full or sampled golden."""
    y = np.asarray(actual, dtype=np.float64)
    if "out" in data:
        ref = data["out"].astype(np.float64)
        return float(np.abs(y - ref).max()), float(np.abs(ref).max()), \
            float(np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30))
    ref = data["sample"]
    got = y.reshape(-1)[data["sample_idx"]]
    rows = data["row_sums"]
    err = max(float(np.abs(got - ref).max()), float(np.abs(y.sum(-1) - rows).max()) / 64)
    rel = float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))
    return err, float(np.abs(ref).max()), rel
