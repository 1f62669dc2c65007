"""Whole-model parity on the GPU: ``load_student`` + ``InferenceEngine`` on the
B200 kernels against the reference model's own FP32 logits (golden vectors
from ``tests/golden/make_model_golden.py``, same synthetic weights and audio).

Tolerances, on sigmoid probabilities:

* 2e-3 for the recurrence's share: the model with the CUDA recurrence against
  the same model whose recurrence is the FP64 CPU oracle (RMSNorm → recurrence
  → length mask, on the same BF16 operands, BF16 output like the kernel's),
  with FP32 GEMMs/convolutions so that nothing else rounds. (Under BF16
  autocast the logits themselves are BF16: one ulp of a logit near 2 is
  ~1.6e-3 in probability, and 16 recurrence calls feeding BF16 GEMMs flip a
  few ulps for any change in the recurrence's last bit.)
* 1e-2 against the reference's FP32 path (``logits``) and against its BF16
  autocast arithmetic (``logits_bf16``). BF16 GEMM/convolution operands alone
  move this randomly initialised network by 6-7e-3 (the reference's own
  arithmetic under BF16 autocast, measured by the golden generator), so two
  BF16 realisations differ by several 1e-3 regardless of the recurrence.

CUDA-graph replay must equal eager execution exactly.
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from oracle import mamba_oracle as O  # noqa: E402
from trifusion_b200 import InferenceEngine, load_student  # noqa: E402
from trifusion_b200.synthetic import student_checkpoint, synthetic_audio  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"
PROB_TOL = 2e-3    # the recurrence's share (CUDA vs oracle recurrence in the same model)
PROB_TOL_BF16 = 1e-2  # whole model vs the reference's FP32 / BF16-autocast logits


def case_inputs(case, tmp_path):
    g = dict(np.load(GOLDEN / f"model_{case}.npz"))
    cfg = json.loads(str(g["config"]))
    b, c, n = (int(v) for v in g["audio_shape"])
    audio, lengths, channels = synthetic_audio(b, n, channels=g["channels"], lengths=g["lengths"],
                                               seed=int(g["audio_seed"]))
    path = student_checkpoint(tmp_path / f"{case}.pt", cfg, seed=int(g["weight_seed"]))
    return g, path, (audio.cuda(), lengths.cuda(), channels.cuda())


def probabilities(logits):
    return torch.as_tensor(logits).float().sigmoid().cpu().numpy()


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_optimized_model_matches_reference_probabilities(case, tmp_path):
    g, path, inputs = case_inputs(case, tmp_path)
    model = load_student(path, optimized=True)
    eager = InferenceEngine(model, graphs=False)(*inputs)
    assert torch.isfinite(eager).all()
    for key in ("logits", "logits_bf16"):
        diff = np.abs(probabilities(eager) - probabilities(g[key])).max()
        print(case, key, "max probability difference", diff)
        assert diff <= PROB_TOL_BF16, diff
    graph_engine = InferenceEngine(model, graphs=True, max_graphs=1)
    first = graph_engine(*inputs)
    second = graph_engine(*inputs)
    assert graph_engine.graph_hits == 2 and not graph_engine.disabled_shapes
    assert torch.equal(first, eager) and torch.equal(second, eager)


def _oracle_recurrence(q, k, v, adt, dt, trap, qb, kb, angles, d, z, *, q_norm=None,
                      k_norm=None, lengths=None, eps=1e-5, out=None):
    """rms (BF16 out) → FP64 recurrence → length mask, on the CPU; BF16 result
    on the input's device (the kernel's output type)."""
    host = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    # The kernel's operands are BF16: round the BF16-typed inputs the same way.
    q, k, v, angles, z = (t.to(torch.bfloat16) for t in (q, k, v, angles, z))
    qn = O.rms(host(q), host(q_norm), eps) if q_norm is not None else host(q)
    kn = O.rms(host(k), host(k_norm), eps) if k_norm is not None else host(k)
    y = O.fused_mamba(qn, kn, *(host(t) for t in (v, adt, dt, trap, qb, kb, angles, d, z)))
    if lengths is not None:
        y = O.mask_rows(y, host(lengths).astype(np.int64))
    return torch.from_numpy(np.asarray(y, np.float32)).to(device=v.device, dtype=torch.bfloat16)


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_recurrence_share_of_model_probabilities(case, tmp_path, monkeypatch):
    g, path, inputs = case_inputs(case, tmp_path)
    model = load_student(path, optimized=True).float()  # FP32 GEMMs, no autocast below
    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    monkeypatch.setattr(torch.backends.cuda.matmul, "allow_tf32", False)
    with torch.inference_mode():
        cuda = model(*inputs)["logits"]
        import trifusion_b200.mamba_fused as mf

        monkeypatch.setattr(mf, "fused_recurrence", _oracle_recurrence)
        oracle = model(*inputs)["logits"]
    diff = np.abs(probabilities(cuda) - probabilities(oracle)).max()
    print(case, "CUDA vs oracle recurrence, max probability difference", diff)
    assert diff <= PROB_TOL, diff


def test_reference_backend_and_unfused_launches_agree(tmp_path):
    g, path, inputs = case_inputs("small", tmp_path)
    ref_model = load_student(path, optimized=False)
    ref = InferenceEngine(ref_model, graphs=False)(*inputs)
    assert np.abs(probabilities(ref) - probabilities(g["logits"])).max() <= PROB_TOL_BF16
    model = load_student(path, optimized=True)
    fused = InferenceEngine(model, graphs=False)(*inputs)
    for block in model.blocks:
        block.forward_mamba.fused_recurrence = block.backward_mamba.fused_recurrence = False
    unfused = InferenceEngine(model, graphs=False)(*inputs)
    diff = np.abs(probabilities(unfused) - probabilities(fused)).max()
    print("fused vs unfused launches, max probability difference", diff)
    assert diff <= PROB_TOL_BF16, diff


def test_padding_does_not_change_a_clip(tmp_path):
    # The same clip alone and zero-padded inside a longer batch.
    g, path, (audio, lengths, channels) = case_inputs("small", tmp_path)
    model = load_student(path, optimized=True)
    engine = InferenceEngine(model, graphs=False)
    batch = engine(audio, lengths, channels)
    n = int(lengths[2])
    alone = engine(audio[2:3, :1, :n].contiguous(), lengths[2:3], channels[2:3])
    assert np.abs(probabilities(alone) - probabilities(batch[2:3])).max() <= 4e-3
