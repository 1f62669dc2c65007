"""Generate golden vectors by running the reference's own code on the CPU.

Run in a container that holds the reference source tree (read-only) and
Triton:

    python tests/golden/make_golden.py --reference-src <path>/src

It imports the reference package ``trifusion_l4`` with ``TRITON_INTERPRET=1``
so its Triton kernels execute on CPU tensors through Triton's interpreter.
The interpreter cannot run inline PTX, so before the kernel modules are
imported the reference's ``cos_approx``/``sin_approx``/``tanh_approx``
(``vendor/utils.py:13-69``) are replaced with exact ``tl.cos``/``tl.sin``/tanh.
BF16 ``tl.dot`` is unreliable in the interpreter, so the recurrence runs on the
FP32 path: the same BF16-valued inputs widened to FP32 (the path the CUDA
kernel is held to).

The interpreter truncates (rather than rounds to nearest) when it stores
into a BF16 tensor, so its BF16-output satellites are good to one BF16 ulp;
the reference's PyTorch formulas are stored beside them as the bit-level
goldens.

Each case writes ``<name>.npz`` next to this script with the generator
parameters, an input checksum and the reference outputs. Large outputs are
stored as a deterministic sample of elements plus per-row sums. The tests
regenerate inputs with ``trifusion_b200.synthetic`` and compare.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
FULL_LIMIT = 1 << 16
SAMPLE = 16384


def _setup(reference_src):
    # The JIT resolves `tl` through the module globals of the patched functions.
    global triton, tl
    os.environ["TRITON_INTERPRET"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(reference_src))
    sys.path.insert(0, str(REPO / "trifusion-fp-kernel_b200"))
    import triton
    import triton.language as tl
    import trifusion_l4.vendor.utils as utils

    @triton.jit
    def cos_exact(x):
        return tl.cos(x)

    @triton.jit
    def sin_exact(x):
        return tl.sin(x)

    @triton.jit
    def tanh_exact(x):
        e = tl.exp(-2.0 * tl.abs(x))
        t = (1.0 - e) / (1.0 + e)
        return tl.where(x >= 0, t, -t)

    utils.cos_approx, utils.sin_approx, utils.tanh_approx = cos_exact, sin_exact, tanh_exact

    # libdevice externs do not run in the interpreter; `_controls`
    # (primitives.py:396) calls log1p. Goldberg's accurate form:
    # log1p(x) = log(u) * x / (u - 1) with u = 1 + x (x itself when u == 1).
    @triton.jit
    def log1p_interp(x):
        u = 1.0 + x
        return tl.where(u == 1.0, x, tl.log(u) * (x / (u - 1.0)))

    import triton.language.extra.cuda.libdevice as libdevice
    libdevice.log1p = log1p_interp


def checksum(arrays):
    """Order-sensitive float64 checksum of a list of tensors."""
    total = 0.0
    for i, a in enumerate(arrays):
        x = a.detach().double().contiguous().reshape(-1).numpy()
        w = np.cos(np.arange(x.size) * 0.37 + i)
        total += float((x * w).sum())
    return total


def pack_output(out):
    """Full output when small; else a seeded element sample plus row sums."""
    y = out.detach().double().numpy()
    if y.size <= FULL_LIMIT:
        return {"out": y.astype(np.float32)}
    rng = np.random.default_rng(1234)
    idx = np.sort(rng.choice(y.size, SAMPLE, replace=False))
    return {"sample_idx": idx.astype(np.int64), "sample": y.reshape(-1)[idx],
            "row_sums": y.sum(-1)}


RECURRENCE_CASES = [
    # name, (B, T, H), kwargs for synthetic.recurrence_inputs
    ("rec_reftest_1x1x4", (1, 1, 4), dict(kind="reftest")),
    ("rec_reftest_2x26x4", (2, 26, 4), dict(kind="reftest")),
    ("rec_reftest_1x63x8", (1, 63, 8), dict(kind="reftest")),
    ("rec_reftest_1x64x8", (1, 64, 8), dict(kind="reftest")),
    ("rec_reftest_2x65x4", (2, 65, 4), dict(kind="reftest")),
    ("rec_reftest_1x255x8", (1, 255, 8), dict(kind="reftest")),
    ("rec_reftest_1x1501x2", (1, 1501, 2), dict(kind="reftest")),
    ("rec_groups2_2x100x4", (2, 100, 4), dict(kind="reftest", groups=2)),
    ("rec_distinct_1x90x3", (1, 90, 3), dict(kind="reftest", distinct_angles=True)),
    ("rec_baseline_cfg0", (2, 200, 12), dict(kind="baseline")),
]


def make_recurrence(name, shape, kw):
    import torch
    from trifusion_l4.mamba_fused import fused_mamba
    from trifusion_l4.angle import angle_dt_fwd
    from trifusion_l4.mamba_portable import mamba3_siso_fwd
    from trifusion_b200.synthetic import recurrence_inputs

    args = recurrence_inputs(*shape, **kw)
    f32 = [a.float() if a.is_floating_point() else a for a in args]
    q, k, v, adt, dt, trap, qb, kb, angles, d, z = f32
    fused = fused_mamba(*f32)
    phase = angle_dt_fwd(angles.float(), dt, chunk_size=64)
    portable = mamba3_siso_fwd(q, k, v, adt, dt, trap, qb, kb, phase, d, z, chunk_size=64)[0]
    rel = float((fused - portable).norm() / portable.norm().clamp_min(1e-20))
    assert rel < 1e-5, (name, rel)
    meta = dict(kind="recurrence", shape=np.array(shape), kw=repr(sorted(kw.items())),
                input_checksum=checksum(f32), fused_vs_portable_rel=rel)
    data = {**{k_: np.asarray(v_) for k_, v_ in meta.items()}, **pack_output(fused)}
    if phase.numel() <= FULL_LIMIT:
        data["phase"] = phase.numpy().astype(np.float32)
    np.savez_compressed(HERE / f"{name}.npz", **data)
    print(name, shape, "fused-vs-portable rel", rel)


def make_satellites():
    """Reference Triton satellite kernels (interpreter) and PyTorch formulas."""
    import torch
    from trifusion_l4.kernels import native, rms_reference, reverse_valid, swiglu, gated_concat
    from trifusion_l4.kernels.buffers import mask_buffer, mamba_controls, Pool4
    from trifusion_l4.masking import Grids, time_mask

    g = torch.Generator().manual_seed(99)
    bf = torch.bfloat16
    b, t, dim, h = 3, 37, 48, 4
    lengths = torch.tensor([37, 20, 1], dtype=torch.int64)
    out = {}
    # B/C RMSNorm over the 128-wide q/k: Triton MODE 0 and the PyTorch formula.
    x = torch.randn(b, t, 1, 128, generator=g).to(bf) * 3
    w = 1 + 0.02 * torch.randn(128, generator=g)
    out["rms_x"], out["rms_w"] = x.float().numpy(), w.numpy()
    out["rms_triton"] = native.rms(x, w, 1e-5).float().numpy()
    out["rms_torch"] = rms_reference(x, w, 1e-5).float().numpy()
    # mean_norm of the bidirectional pair (FP32 output).
    mf = torch.randn(b, t, dim, generator=g).to(bf)
    mb = torch.randn(b, t, dim, generator=g).to(bf)
    wm = 1 + 0.02 * torch.randn(dim, generator=g)
    out["mn_a"], out["mn_b"], out["mn_w"] = mf.float().numpy(), mb.float().numpy(), wm.numpy()
    out["mean_norm_triton"] = native.mean_norm(mf, mb, wm, 1e-5).numpy()
    # Evidence norm (MODE 1): FP32 residual + BF16 value/gate, masked rows.
    xe = torch.randn(b, t, dim, generator=g)
    ve = torch.randn(b, t, dim, generator=g).to(bf)
    ge = torch.randn(b, t, dim, generator=g).to(bf)
    me = time_mask(lengths, t)
    out["ev_x"], out["ev_v"], out["ev_g"], out["ev_mask"] = (
        xe.numpy(), ve.float().numpy(), ge.float().numpy(), me.numpy())
    out["evidence_norm_triton"] = native.evidence_norm(xe, ve, ge, wm, me, 1e-5).numpy()
    # A/dt controls from strided BF16 projection views.
    p = torch.randn(b, t, 3 * h + 5, generator=g).to(bf) * 4
    a, ddt = p[..., :h], p[..., h:2 * h]
    bias = torch.full((h,), -4.0) + torch.randn(h, generator=g)
    oa, od = mamba_controls(a, ddt, bias, 1e-4)
    out["ctl_a"], out["ctl_ddt"], out["ctl_bias"] = a.float().numpy(), ddt.float().numpy(), bias.numpy()
    out["ctl_adt"], out["ctl_dt"] = oa.numpy(), od.numpy()
    # Length mask, valid-prefix reversal, SwiGLU, gate, Pool4.
    xm = torch.randn(b, t, dim, generator=g).to(bf)
    mask = time_mask(lengths, t)
    out["lengths"], out["x"] = lengths.numpy(), xm.float().numpy()
    out["mask_triton"] = mask_buffer(xm, mask).float().numpy()
    out["reverse_triton"] = reverse_valid(xm, lengths, "l4").float().numpy()
    out["reverse_torch"] = reverse_valid(xm, lengths, "reference").float().numpy()
    xs = torch.randn(b, t, 2 * dim, generator=g).to(bf) * 2
    out["sw_x"] = xs.float().numpy()
    out["swiglu_triton"] = swiglu(xs, "l4").float().numpy()
    out["swiglu_torch"] = swiglu(xs, "reference").float().numpy()
    xg = torch.randn(b, t, 3 * dim, generator=g).to(bf)
    gate = torch.randn(b, t, 3, generator=g).to(bf) * 2
    out["gate_x"], out["gate_g"] = xg.float().numpy(), gate.float().numpy()
    out["gate_triton"] = gated_concat(xg, gate, "l4").float().numpy()
    out["gate_torch"] = gated_concat(xg, gate, "reference").float().numpy()
    grids = Grids.make(lengths, t, 16, buffer_fusion=False)
    out["pool_torch"] = grids.pool(xm).float().numpy()
    out["pool_triton"] = Pool4.apply(xm.contiguous(), lengths).float().numpy()
    # Decoder masked mean and end-state gather (decoder.py:60-63).
    xf = xm.float()
    out["masked_mean_torch"] = ((xf * grids.mask[..., None]).sum(1) / lengths[:, None]).numpy()
    out["end_torch"] = xf[torch.arange(b), lengths - 1].numpy()
    np.savez_compressed(HERE / "satellites.npz", **out)
    print("satellites", sorted(out))


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference-src", required=True, type=Path)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    _setup(args.reference_src)
    for name, shape, kw in RECURRENCE_CASES:
        if args.only and args.only not in name:
            continue
        make_recurrence(name, shape, kw)
    if not args.only or "sat" in args.only:
        make_satellites()


if __name__ == "__main__":
    main()
