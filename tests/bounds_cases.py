"""Odd-shape recurrence launches for the bounds-checked debug build (GPU only).

Run by ``tests/test_bounds_gpu.py`` in a fresh process with ``TRIFUSION_B200_BOUNDS=1``,
which makes ``trifusion_b200`` load ``libtrifusion_b200_bounds.so``: every global access
of the recurrence kernel is checked against the tensors' extents there, and an
out-of-range one records device error 2 (and is skipped). Each case is also held to
the oracle. Exits non-zero on any failure.
"""

import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for _p in (ROOT, ROOT / "trifusion-fp-kernel_b200", ROOT / "tests"):
    sys.path.insert(0, str(_p))

import torch  # noqa: E402

from oracle import mamba_oracle as O  # noqa: E402
from parity import assert_recurrence_close, oracle_out  # noqa: E402
from trifusion_b200 import _lib, fused_mamba, fused_recurrence  # noqa: E402
from trifusion_b200.mamba_fused import fused_recurrence_multi  # noqa: E402
from trifusion_b200.synthetic import recurrence_inputs  # noqa: E402

DEV = "cuda"


def reverse_rows(x, lengths):
    b, t = x.shape[:2]
    pos = torch.arange(t, device=x.device)[None, :]
    idx = torch.where(pos < lengths[:, None], lengths[:, None] - 1 - pos, pos)
    return torch.take_along_dim(x, idx.view(b, t, *([1] * (x.dim() - 2))), dim=1)


def check_reversed(args, lengths, what):
    names = ("q", "k", "v", "adt", "dt", "trap", "qb", "kb", "angles", "d", "z")
    d = dict(zip(names, args))
    rev = fused_recurrence_multi([dict(d, reverse=True)], lengths=lengths)[0]
    flipped = dict(d)
    for name in ("q", "k", "v", "z", "angles"):
        flipped[name] = reverse_rows(d[name], lengths).contiguous()
    for name in ("adt", "dt", "trap"):
        flipped[name] = reverse_rows(d[name].transpose(1, 2), lengths).transpose(1, 2).contiguous()
    ref = O.mask_rows(oracle_out([flipped[n] for n in names]), lengths.cpu().numpy())
    assert_recurrence_close(reverse_rows(rev, lengths), ref, what)


def run():
    assert _lib.LIB_PATH.name == "libtrifusion_b200_bounds.so", _lib.LIB_PATH
    lib = _lib.lib()
    lib.tf_device_error(1)
    for t in (1, 63, 65):
        args = recurrence_inputs(2, t, 3, kind="reftest", device=DEV)
        assert_recurrence_close(fused_mamba(*args), oracle_out(args), f"T={t}")
    args = recurrence_inputs(2, 100, 4, groups=2, kind="baseline", device=DEV)
    assert_recurrence_close(fused_mamba(*args), oracle_out(args), "Hq=2")
    # 2-byte-aligned v and z views.
    b, t, h = 2, 70, 4
    base = recurrence_inputs(b, t, h, kind="reftest", device=DEV)
    q, k, v, adt, dt, trap, qb, kb, angles, d, z = base
    buf = torch.zeros(b, t, h * 64 * 2 + 3, dtype=torch.bfloat16, device=DEV)
    buf[:, :, 1:1 + h * 64] = v.reshape(b, t, -1)
    buf[:, :, 2 + h * 64: 2 + 2 * h * 64] = z.reshape(b, t, -1)
    v2 = buf[:, :, 1:1 + h * 64].reshape(b, t, h, 64)
    z2 = buf[:, :, 2 + h * 64: 2 + 2 * h * 64].reshape(b, t, h, 64)
    assert_recurrence_close(fused_mamba(q, k, v2, adt, dt, trap, qb, kb, angles, d, z2), oracle_out(base),
                            "2-byte views")
    # Lengths (incl. 0 and 1), short and long (TMA-staged, look-back) rows, reversed rows.
    for b, t, lens in ((5, 150, [150, 97, 1, 0, 64]), (2, 700, [700, 451])):
        args = recurrence_inputs(b, t, 4, kind="baseline", seed=t, device=DEV)
        lengths = torch.tensor(lens, device=DEV)
        out = fused_recurrence(*args, lengths=lengths)
        assert_recurrence_close(out, O.mask_rows(oracle_out(args), lengths.cpu().numpy()), f"lengths T={t}")
        check_reversed(args, lengths, f"reversed T={t}")
    torch.cuda.synchronize()
    err = lib.tf_device_error(0)
    assert err == 0, f"device error {err} (2: an out-of-range access in the bounds build)"
    print("bounds cases ok")


if __name__ == "__main__":
    if os.environ.get("TRIFUSION_B200_BOUNDS") != "1":
        sys.exit("run with TRIFUSION_B200_BOUNDS=1")
    run()
