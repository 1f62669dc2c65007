"""Host-side model checks that need no GPU.

* The student's parameter layout equals the reference's (names and shapes,
  recorded from the reference by ``tests/golden/make_model_golden.py``), so
  reference checkpoints load with a strict key check.
* ``load_student`` keeps the reference's behaviour: unknown configuration
  fields raise, deployed weights are BF16, the training-only head is dropped.
* The whole host model (front end, blocks, decoder, grids, masks) reproduces
  the reference model's logits when its recurrence is evaluated by the CPU
  oracle — the model code is checked here, the CUDA recurrence on the GPU.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import mamba_oracle as O
from trifusion_b200.model import ModelConfig, TriFusion
from trifusion_b200.runtime import configure_runtime, load_student
from trifusion_b200.synthetic import student_checkpoint, synthetic_audio

GOLDEN = Path(__file__).resolve().parent / "golden"


def layouts():
    return json.loads((GOLDEN / "student_keys.json").read_text())


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_parameter_layout_matches_reference(case):
    ref = layouts()[case]
    with torch.device("meta"):
        model = TriFusion(ModelConfig(**ref["config"]))
    ours = {k: list(v.shape) for k, v in model.state_dict().items()}
    assert ours == ref["shapes"]


def test_load_student_rules(tmp_path):
    cfg = layouts()["small"]["config"]
    path = student_checkpoint(tmp_path / "s.pt", cfg)
    model = load_student(path, optimized=True, device="cpu")
    assert not hasattr(model, "memory_head")
    assert model.blocks[0].forward_mamba.fused_recurrence and model.blocks[0].backward_mamba.fused_recurrence
    assert model.blocks[0].forward_mamba.in_proj.weight.dtype == torch.bfloat16
    assert model.blocks[0].pre.weight.dtype == torch.float32
    assert model.config.backend == "l4" and model.front.window.shape == (400,)
    assert not any(p.requires_grad for p in model.parameters())
    ref = load_student(path, optimized=False, device="cpu")
    assert ref.config.backend == "reference"
    assert ref.blocks[0].forward_mamba.in_proj.weight.dtype == torch.float32
    # Unknown configuration fields are rejected, missing weights too.
    saved = torch.load(path, weights_only=True)
    torch.save({"model_config": {**saved["model_config"], "extra": 1}, "model": saved["model"]},
               tmp_path / "bad.pt")
    with pytest.raises(ValueError, match="Unsupported model configuration fields"):
        load_student(tmp_path / "bad.pt", device="cpu")
    state = dict(saved["model"])
    state.pop("decoder.query")
    torch.save({"model_config": saved["model_config"], "model": state}, tmp_path / "missing.pt")
    with pytest.raises(RuntimeError, match="decoder.query"):
        load_student(tmp_path / "missing.pt", device="cpu")


def test_configure_runtime_requires_a_gpu():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    with pytest.raises(RuntimeError, match="CUDA GPU is required"):
        configure_runtime()


def _oracle_fused_mamba(q, k, v, adt, dt, trap, qb, kb, angles, d, z, warps=8):
    arrays = [t.detach().float().numpy() for t in (q, k, v, adt, dt, trap, qb, kb, angles, d, z)]
    return torch.from_numpy(np.asarray(O.fused_mamba(*arrays), dtype=np.float32))


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_host_model_matches_reference_with_oracle_recurrence(case, tmp_path, monkeypatch):
    g = dict(np.load(GOLDEN / f"model_{case}.npz"))
    cfg = json.loads(str(g["config"]))
    b, c, n = (int(v) for v in g["audio_shape"])
    audio, lengths, channels = synthetic_audio(b, n, channels=g["channels"], lengths=g["lengths"],
                                               seed=int(g["audio_seed"]))
    assert float(audio.double().sum()) == pytest.approx(float(g["audio_sum"]), rel=0, abs=1e-9)
    path = student_checkpoint(tmp_path / "s.pt", cfg, seed=int(g["weight_seed"]))
    model = load_student(path, optimized=False, device="cpu")
    import trifusion_b200.mamba_fused as mf

    monkeypatch.setattr(mf, "fused_mamba", _oracle_fused_mamba)
    with torch.inference_mode():
        out = model(audio, lengths, channels)
    np.testing.assert_allclose(out["logits"].numpy(), g["logits"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(out["embedding"].numpy(), g["embedding"], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_reference_gpu_goldens_are_consistent(case):
    """The reference's FP32 path run on the GPU (``make_model_golden_gpu.py``) reproduces
    its CPU FP32 goldens, and its deployed BF16 path stays within 1e-2 of them: the
    GPU fixture is the same model on the same audio."""
    sig = lambda x: 1 / (1 + np.exp(-np.asarray(x, np.float64)))  # noqa: E731
    g = np.load(GOLDEN / f"model_{case}.npz")
    r = np.load(GOLDEN / f"model_{case}_ref_gpu.npz")
    assert r["logits_portable"].shape == g["logits"].shape == r["logits_deployed"].shape
    assert np.abs(sig(r["logits_portable"]) - sig(g["logits"])).max() <= 1e-3
    assert np.abs(sig(r["logits_deployed"]) - sig(g["logits"])).max() <= 1e-2
