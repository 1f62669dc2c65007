"""Whole-model parity on the GPU: ``load_student`` + ``InferenceEngine`` on the
B200 kernels against the reference model's own logits (golden vectors from
``tests/golden/make_model_golden.py``, same synthetic weights and audio).

Bounds, on sigmoid probabilities (measured values in brackets: small, cfg3):

* the recurrence's share, 2.5e-3 [4.1e-4, 2.0e-3]: the model with the CUDA
  recurrence against the same model whose recurrence is the FP64 CPU oracle
  under the kernel's BF16 I/O contract, with FP32 GEMMs so that nothing else
  rounds differently. Before its BF16 output rounding the kernel is 6e-5 (relative
  L2) from the oracle, 30x below that rounding itself; the gap is one-ulp BF16
  flips of the 16 recurrence outputs propagated through the network.
* 8e-3 for the optimized model under BF16 autocast against the reference's FP32
  logits [6.8e-3, 5.4e-3] and its BF16-autocast logits [2.9e-3, 5.2e-3]. BF16
  GEMM/convolution operands alone move this randomly initialised network by
  6-7e-3 (the reference's FP32 against its own BF16 autocast).
* the reference's own deployed path (its fused Triton kernels under BF16 autocast,
  ``load_student(optimized=True)`` + ``InferenceEngine``, run on a B200 by
  ``tests/golden/make_model_golden_gpu.py``) is itself [4.9e-3, 8.0e-3] from its FP32
  logits on these synthetic models, so the north star's 2e-3 is out of reach for the
  reference as well. This library's model is held to that gap: against the FP32 logits
  within the reference's worst deployed gap over the cases (8.05e-3) [6.8e-3, 5.4e-3],
  and against the reference's deployed logits within 1.2e-2 [1.9e-3, 9.7e-3].
* with FP32 GEMMs and no autocast, against the reference's FP32 logits: 1.2e-2 with
  the oracle recurrence on FP32 operands [3.5e-3, 9.4e-3] and 1.5e-2 with the CUDA
  recurrence [4.0e-3, 1.1e-2]. This library's norm, front-end and attention kernels
  keep BF16 intermediates (what their consumers read under autocast), so this model
  is not an FP32 model end to end.

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
PROB_TOL = 2.5e-3      # the recurrence's share (CUDA vs oracle recurrence in the same model)
PROB_TOL_BF16 = 8e-3   # whole model (BF16 autocast) vs the reference's FP32 / BF16-autocast logits
PROB_TOL_FP32_REST = 1.2e-2  # FP32 GEMMs, oracle recurrence on FP32 operands, vs reference FP32 logits
PROB_TOL_FP32 = 1.5e-2       # FP32 GEMMs, CUDA recurrence, vs reference FP32 logits
PROB_TOL_DEPLOYED = 1.2e-2   # optimized model vs the reference's deployed (GPU, BF16) logits


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


def reference_deployed_gap():
    """The largest probability difference, over the golden cases, between the
    reference's deployed logits (GPU, fused Triton, BF16 autocast) and its FP32 logits."""
    return max(np.abs(probabilities(np.load(GOLDEN / f"model_{c}_ref_gpu.npz")["logits_deployed"])
                      - probabilities(np.load(GOLDEN / f"model_{c}.npz")["logits"])).max()
               for c in ("small", "cfg3"))


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_model_within_the_reference_deployed_gap(case, tmp_path):
    g, path, inputs = case_inputs(case, tmp_path)
    deployed = np.load(GOLDEN / f"model_{case}_ref_gpu.npz")["logits_deployed"]
    model = load_student(path, optimized=True)
    ours = probabilities(InferenceEngine(model, graphs=False)(*inputs))
    gap = np.abs(ours - probabilities(g["logits"])).max()
    bound = reference_deployed_gap()
    direct = np.abs(ours - probabilities(deployed)).max()
    print(case, "vs reference FP32", gap, "(reference deployed gap", bound, ") vs reference deployed", direct)
    assert gap <= bound, (gap, bound)
    assert direct <= PROB_TOL_DEPLOYED, direct


def _oracle_multi(bf16_io):
    """Stand-in for ``fused_recurrence_multi`` running the FP64 CPU oracle: in-launch
    controls from the projection views, reversed rows, C/B RMSNorm, length mask,
    outputs written into the given views. ``bf16_io``: the kernel's contract (BF16
    operands, RMSNorm output and result); otherwise FP32 throughout, like the
    reference's FP32 path."""
    def run(directions, *, lengths=None, eps=1e-5):
        host = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
        io = (lambda t: t.detach().to(torch.bfloat16)) if bf16_io else (lambda t: t.detach().float())
        outs = []
        for d_ in directions:
            v = io(d_["v"])
            b, t, h, _ = v.shape
            lens = host(lengths).astype(np.int64) if lengths is not None else np.full(b, t, np.int64)
            q, k, z, ang = (host(io(d_[n])) for n in ("q", "k", "z", "angles"))
            v = host(v)
            trap = host(d_["trap"]).transpose(0, 2, 1)  # [B,T,H]
            if d_.get("a_raw") is not None:
                adt, dt = O.mamba_controls(host(io(d_["a_raw"])), host(io(d_["ddt_raw"])), host(d_["dt_bias"]),
                                           d_.get("a_floor", 1e-4))
                adt, dt = adt.transpose(0, 2, 1), dt.transpose(0, 2, 1)
            else:
                adt, dt = host(d_["adt"]).transpose(0, 2, 1), host(d_["dt"]).transpose(0, 2, 1)
            if d_.get("reverse"):
                q, k, v, z, ang, trap, adt, dt = (O.reverse_valid(x, lens) for x in (q, k, v, z, ang, trap, adt, dt))
            if d_.get("q_norm") is not None:
                q = O.rms(q, host(d_["q_norm"]), eps, out_bf16=bf16_io)
                k = O.rms(k, host(d_["k_norm"]), eps, out_bf16=bf16_io)
            y = O.fused_mamba(q, k, v, adt.transpose(0, 2, 1), dt.transpose(0, 2, 1), trap.transpose(0, 2, 1),
                              host(d_["qb"]), host(d_["kb"]), ang, host(d_["d"]), z)
            y = O.mask_rows(y, lens)
            if d_.get("reverse"):
                y = O.reverse_valid(y, lens)
            y = torch.from_numpy(np.asarray(y, np.float32)).to(d_["v"].device)
            if d_.get("out") is not None:
                d_["out"].copy_(y)
                y = d_["out"]
            else:
                y = y.to(torch.bfloat16 if bf16_io else torch.float32)
            outs.append(y)
        return outs
    return run


def _fp32_model(case, tmp_path, monkeypatch):
    g, path, inputs = case_inputs(case, tmp_path)
    model = load_student(path, optimized=True).float()  # FP32 GEMMs, no autocast below
    monkeypatch.setattr(torch.backends.cudnn, "allow_tf32", False)
    monkeypatch.setattr(torch.backends.cuda.matmul, "allow_tf32", False)
    return g, model, inputs


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_recurrence_share_of_model_probabilities(case, tmp_path, monkeypatch):
    """The model with the CUDA recurrence against the same model whose recurrence is
    the FP64 oracle under the kernel's BF16 I/O contract: within 2e-3."""
    import trifusion_b200.mamba_fused as mf

    g, model, inputs = _fp32_model(case, tmp_path, monkeypatch)
    with torch.inference_mode():
        cuda = model(*inputs)["logits"]
        monkeypatch.setattr(mf, "fused_recurrence_multi", _oracle_multi(True))
        oracle = model(*inputs)["logits"]
    diff = np.abs(probabilities(cuda) - probabilities(oracle)).max()
    print(case, "CUDA vs oracle recurrence, max probability difference", diff)
    assert 0 < diff <= PROB_TOL, diff  # (exactly 0: the stand-in was not reached)


@pytest.mark.parametrize("case", ["small", "cfg3"])
def test_fp32_model_matches_reference_fp32_logits(case, tmp_path, monkeypatch):
    """Against the reference model's FP32 logits, with FP32 GEMMs and convolutions:
    the model with the FP64 oracle recurrence on FP32 operands (the rest of the path)
    and with the CUDA recurrence (BF16 I/O by contract)."""
    import trifusion_b200.mamba_fused as mf

    g, model, inputs = _fp32_model(case, tmp_path, monkeypatch)
    ref = probabilities(g["logits"])
    with torch.inference_mode():
        cuda = model(*inputs)["logits"]
        monkeypatch.setattr(mf, "fused_recurrence_multi", _oracle_multi(False))
        fp32_io = model(*inputs)["logits"]
    d_cuda = np.abs(probabilities(cuda) - ref).max()
    d_fp32 = np.abs(probabilities(fp32_io) - ref).max()
    print(case, "FP32 model vs reference FP32 logits: CUDA", d_cuda, "oracle recurrence with FP32 I/O", d_fp32)
    assert d_fp32 <= PROB_TOL_FP32_REST, d_fp32
    assert d_cuda <= PROB_TOL_FP32, d_cuda


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
