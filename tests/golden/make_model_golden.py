"""Whole-model golden vectors from the reference's own model, run on the CPU.

    python tests/golden/make_model_golden.py --reference-src <path>/src

For each case it builds the reference ``TriFusion`` with the case's
configuration, checks that its parameter layout (names and shapes) equals this
package's, writes a checkpoint whose weights come from
``trifusion_b200.synthetic.student_state`` (a function of name, shape and seed
only), loads it with the reference's ``load_student(optimized=False,
device="cpu")`` (its FP32 reference path; the recurrence runs through the
reference's portable Triton kernels under ``TRITON_INTERPRET=1``, set up as in
``make_golden.py``) and runs one forward pass on ``synthetic_audio``.

A second pass runs the same model under CPU BF16 autocast with BF16
recurrence inputs/outputs — the reference's deployed (L4) arithmetic — giving
``logits_bf16``.

Stored per case (``model_<name>.npz``): the configuration, seeds, audio shape
and lengths, an audio checksum, and the reference's ``logits``/``embedding``
(FP32 path) and ``logits_bf16``.
``student_keys.json`` records the parameter layout for the CPU key test.
"""

from __future__ import annotations

import argparse
import json
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

CASES = {
    "small": dict(config=dict(dim=128, depth=2, heads=2, ffn_dim=256, state_dim=128),
                  batch=3, samples=16000, lengths=[16000, 11000, 4000], channels=[1, 2, 1]),
    "cfg3": dict(config=dict(dim=384, depth=8, heads=6, ffn_dim=1536, state_dim=128),
                 batch=2, samples=64000, lengths=[64000, 41000], channels=[1, 1]),
}
WEIGHT_SEED, AUDIO_SEED = 0, 3


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference-src", required=True, type=Path)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    import make_golden

    make_golden._setup(args.reference_src)
    import torch
    from trifusion_l4.model import ModelConfig as RefConfig, TriFusion as RefModel
    from trifusion_l4.runtime import load_student as ref_load
    from trifusion_b200.model import ModelConfig, TriFusion
    from trifusion_b200.synthetic import student_checkpoint, synthetic_audio

    layouts = {}
    for name, case in CASES.items():
        if args.only and args.only != name:
            continue
        cfg = case["config"]
        ref_shapes = {k: list(v.shape) for k, v in RefModel(RefConfig(**cfg)).state_dict().items()}
        with torch.device("meta"):
            ours = {k: list(v.shape) for k, v in TriFusion(ModelConfig(**cfg)).state_dict().items()}
        assert ref_shapes == ours, set(ref_shapes) ^ set(ours)
        layouts[name] = {"config": cfg, "shapes": ref_shapes}
        with tempfile.TemporaryDirectory() as tmp:
            path = student_checkpoint(Path(tmp) / "student.pt", cfg, seed=WEIGHT_SEED)
            model = ref_load(path, optimized=False, device="cpu")
        audio, lengths, channels = synthetic_audio(case["batch"], case["samples"],
                                                   channels=case["channels"],
                                                   lengths=case["lengths"], seed=AUDIO_SEED)
        start = time.perf_counter()
        with torch.inference_mode():
            out = model(audio, lengths, channels)
        print(name, "reference forward", round(time.perf_counter() - start, 1), "s",
              out["logits"].tolist())
        # The reference's deployed arithmetic: BF16 GEMM/convolution operands
        # under autocast (runtime.py:77-78, 52-56) and a recurrence with BF16
        # inputs and output (mamba_fused.py:161). The interpreter cannot run
        # BF16 dots, so its portable kernel gets the BF16 values widened to FP32.
        import trifusion_l4.mamba as ref_mamba

        portable = ref_mamba.mamba3_siso_fwd

        def bf16_io(**kw):
            out_dtype = kw["V"].dtype
            kw = {k: (v.float() if torch.is_tensor(v) and v.is_floating_point() else v)
                  for k, v in kw.items()}
            res = portable(**kw)
            return (res[0].to(out_dtype),) + tuple(res[1:])

        ref_mamba.mamba3_siso_fwd = bf16_io
        try:
            with torch.inference_mode(), torch.autocast("cpu", dtype=torch.bfloat16):
                out_bf16 = model(audio, lengths, channels)
        finally:
            ref_mamba.mamba3_siso_fwd = portable
        print(name, "reference forward under BF16 autocast", out_bf16["logits"].float().tolist())
        np.savez_compressed(
            HERE / f"model_{name}.npz",
            config=json.dumps(cfg), weight_seed=WEIGHT_SEED, audio_seed=AUDIO_SEED,
            audio_shape=np.array(audio.shape), lengths=lengths.numpy(), channels=channels.numpy(),
            audio_sum=np.float64(audio.double().sum()), audio_abs=np.float64(audio.double().abs().sum()),
            logits=out["logits"].float().numpy(), embedding=out["embedding"].float().numpy(),
            logits_bf16=out_bf16["logits"].float().numpy())
    if not args.only:
        (HERE / "student_keys.json").write_text(json.dumps(layouts, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
