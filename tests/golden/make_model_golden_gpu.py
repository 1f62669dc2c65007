"""Whole-model logits of the reference's own deployed path on a GPU.

    python tests/golden/make_model_golden_gpu.py      (needs a CUDA GPU and the
                                                       reference under baseline/_ref)

The reference installs offline into ``baseline/_ref`` (``pip install --no-index
--no-build-isolation --no-deps --target baseline/_ref`` from a copy of its
sources). For each case of ``make_model_golden.py`` (same synthetic checkpoint,
audio and lengths) this loads the checkpoint with the reference's
``load_student(optimized=True)`` and runs its ``InferenceEngine(graphs=False)``:
its fused Triton kernels under BF16 autocast (``runtime.py:11-85``), the path it
deploys. It also runs ``load_student(optimized=False)`` on the GPU (its FP32
portable path) as a cross-check of the CPU goldens.

Stored per case (``model_<name>_ref_gpu.npz``): ``logits_deployed``,
``logits_portable`` and the GPU name. The tests hold this library's model to the
gap between the reference's deployed logits and its FP32 logits.
"""

from __future__ import annotations

import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]


def main():
    sys.path[:0] = [str(ROOT), str(ROOT / "trifusion-fp-kernel_b200"), str(ROOT / "baseline" / "_ref")]
    import torch
    from trifusion_l4.runtime import InferenceEngine as RefEngine, load_student as ref_load
    from trifusion_b200.synthetic import student_checkpoint, synthetic_audio

    for name in ("small", "cfg3"):
        g = dict(np.load(HERE / f"model_{name}.npz"))
        cfg = json.loads(str(g["config"]))
        b, _, n = (int(v) for v in g["audio_shape"])
        audio, lengths, channels = synthetic_audio(b, n, channels=g["channels"], lengths=g["lengths"],
                                                   seed=int(g["audio_seed"]))
        inputs = (audio.cuda(), lengths.cuda(), channels.cuda())
        with tempfile.TemporaryDirectory() as tmp:
            path = student_checkpoint(Path(tmp) / "student.pt", cfg, seed=int(g["weight_seed"]))
            deployed = RefEngine(ref_load(path, optimized=True, device="cuda"), graphs=False)(*inputs)
            with torch.inference_mode():
                portable = ref_load(path, optimized=False, device="cuda")(*inputs)["logits"]
        deployed = deployed.float().cpu().numpy()
        portable = portable.float().cpu().numpy()
        gap = np.abs(1 / (1 + np.exp(-deployed)) - 1 / (1 + np.exp(-g["logits"]))).max()
        print(name, "reference deployed vs its FP32 logits, max probability difference", gap)
        np.savez_compressed(HERE / f"model_{name}_ref_gpu.npz", logits_deployed=deployed,
                            logits_portable=portable, gpu=torch.cuda.get_device_name())


if __name__ == "__main__":
    main()
