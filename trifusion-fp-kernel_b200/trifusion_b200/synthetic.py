"""Seeded synthetic inputs for the fused Mamba-3 recurrence and its satellites.

Two recipes exist:

* ``"reftest"`` follows the reference's parity test generator
  (``tests/test_recurrence.py:15-31``): q/k ``randn*0.2`` BF16 ``[B,T,1,128]``;
  v, z and angles are strided views of one ``[B,T,H*128+32]`` BF16 buffer;
  dt ~ U(0.01, 0.11); adt = -dt*U(0.2, 2.2); trap ~ N(0,1); qb, kb ~ N(1, 0.1);
  d = 1.
* ``"baseline"`` follows the benchmark configurations: q/k ~ N(0,1)/sqrt(128);
  v, z ~ N(0,1); raw angles ~ U(-pi, pi) shared by all heads (head stride 0);
  dt = exp(U(ln 1e-3, ln 1e-1)); A = -exp(U(ln 1, ln 16)) per head; adt = A*dt;
  trap ~ N(0,1); D ~ N(0,1); qb, kb = 1 + N(0, 0.1).

Everything is drawn on the CPU from one ``torch.Generator`` so the values are
identical on every machine, then moved to ``device``.
"""

from __future__ import annotations

import math

import torch

STATE, HEAD, ROTARY = 128, 64, 32


def recurrence_inputs(batch, time, heads, *, groups=1, kind="baseline", seed=None,
                      distinct_angles=False, trap_dtype=torch.float32, strided=None,
                      device="cpu"):
    """Return the 11 ``fused_mamba`` arguments as a tuple, in reference order:
    ``(q, k, v, adt, dt, trap, qb, kb, angles, d, z)``."""
    if seed is None:
        seed = 121 + time if kind == "reftest" else 0
    if strided is None:
        strided = kind == "reftest"
    g = torch.Generator().manual_seed(seed)
    b, t, h = batch, time, heads
    bf = torch.bfloat16

    def randn(*shape):
        return torch.randn(*shape, generator=g)

    def rand(*shape):
        return torch.rand(*shape, generator=g)

    if kind == "reftest":
        q = (randn(b, t, groups, STATE).to(bf) * 0.2)
        k = (randn(b, t, groups, STATE).to(bf) * 0.2)
        raw_v = randn(b, t, h * HEAD).to(bf) * 0.2
        raw_z = randn(b, t, h * HEAD).to(bf) * 0.2
        raw_a = randn(b, t, (h if distinct_angles else 1) * ROTARY).to(bf) * 0.2
        dt = rand(b, h, t) * 0.1 + 0.01
        adt = -dt * (rand(b, h, t) * 2 + 0.2)
        trap = randn(b, h, t)
        qb = randn(h, STATE) * 0.1 + 1
        kb = randn(h, STATE) * 0.1 + 1
        d = torch.ones(h)
    elif kind == "baseline":
        q = (randn(b, t, groups, STATE) / math.sqrt(STATE)).to(bf)
        k = (randn(b, t, groups, STATE) / math.sqrt(STATE)).to(bf)
        raw_v = randn(b, t, h * HEAD).to(bf)
        raw_z = randn(b, t, h * HEAD).to(bf)
        raw_a = ((rand(b, t, (h if distinct_angles else 1) * ROTARY) * 2 - 1) * math.pi).to(bf)
        dt = torch.exp(math.log(1e-3) + rand(b, h, t) * (math.log(1e-1) - math.log(1e-3)))
        a_head = -torch.exp(rand(h) * math.log(16.0))
        adt = a_head[None, :, None] * dt
        trap = randn(b, h, t)
        qb = 1 + 0.1 * randn(h, STATE)
        kb = 1 + 0.1 * randn(h, STATE)
        d = randn(h)
    else:
        raise ValueError(kind)
    if trap_dtype != torch.float32:
        trap = trap.to(trap_dtype)
    ha = h if distinct_angles else 1
    if strided:
        # One packed projection row per token, like the reference test's buffer.
        width = 2 * h * HEAD + ha * ROTARY
        buf = torch.cat([raw_v, raw_z, raw_a], -1).reshape(b, t, width)
        v = buf[:, :, : h * HEAD].reshape(b, t, h, HEAD)
        z = buf[:, :, h * HEAD: 2 * h * HEAD].reshape(b, t, h, HEAD)
        ang = buf[:, :, 2 * h * HEAD:].reshape(b, t, ha, ROTARY)
    else:
        v = raw_v.reshape(b, t, h, HEAD).contiguous()
        z = raw_z.reshape(b, t, h, HEAD).contiguous()
        ang = raw_a.reshape(b, t, ha, ROTARY).contiguous()
    angles = ang if distinct_angles else ang.expand(b, t, h, ROTARY)
    args = (q, k, v, adt, dt, trap, qb, kb, angles, d, z)
    if device != "cpu":
        args = tuple(_to_device(a, device) for a in args)
    return args


def _to_device(x, device):
    """Move a (possibly strided / expanded) view to `device`, keeping its strides."""
    if x.is_contiguous():
        return x.to(device)
    base = x
    while base._base is not None:
        base = base._base
    # Re-create the same view on a device copy of the underlying storage.
    storage = torch.empty(0, dtype=x.dtype)
    storage.set_(x.untyped_storage())
    dev = storage.to(device)
    return dev.as_strided(x.shape, x.stride(), x.storage_offset())


def lengths_uniform(batch, low, high, seed=0):
    """Lengths ~ U{low..high} (int64), seeded."""
    g = torch.Generator().manual_seed(seed + 7)
    return torch.randint(low, high + 1, (batch,), generator=g, dtype=torch.int64)


def norm_weight(width, seed=0):
    """RMSNorm weights ~ 1 + N(0, 0.02) (benchmark configuration 1)."""
    g = torch.Generator().manual_seed(seed + 11)
    return 1 + 0.02 * torch.randn(width, generator=g)


# ---------------------------------------------------------------------------
# Synthetic student checkpoints and audio (the model-level configurations).
# Weights are a function of (parameter name, shape, seed) alone, so any model
# with the reference's parameter layout — this package's or the reference's —
# receives identical values.
# ---------------------------------------------------------------------------

def _name_seed(name, seed):
    import zlib

    return (zlib.crc32(name.encode()) + 7919 * seed) % (2 ** 31)


def parameter_value(name, shape, seed=0, depth=1):
    """Deterministic FP32 value of one student parameter.

    Matrices and convolution kernels ~ N(0, 1/fan_in) (the three logit heads
    0.1x that, so that the logits stay in sigmoid's unsaturated range; the
    residual ``merge``/``down`` projections 1/sqrt(2 depth) that, as the
    reference initialises them); norm
    weights 1 + N(0, 0.02);
    biases N(0, 0.02); Mamba ``dt_bias`` -4 + N(0, 0.3), ``B_bias``/``C_bias``
    1 + N(0, 0.1), ``D`` ~ N(0, 1); decoder queries/bands N(0, 0.02).
    """
    g = torch.Generator().manual_seed(_name_seed(name, seed))
    x = torch.randn(*shape, generator=g)
    leaf = name.rsplit(".", 1)[-1]
    if leaf == "dt_bias":
        return -4.0 + 0.3 * x
    if leaf in ("B_bias", "C_bias"):
        return 1.0 + 0.1 * x
    if leaf == "D":
        return x
    if leaf in ("query", "band"):
        return 0.02 * x
    if leaf == "bias":
        return 0.02 * x
    if len(shape) == 1:  # RMSNorm weights
        return 1.0 + 0.02 * x
    fan_in = math.prod(shape[1:])
    if name.startswith(_HEADS):  # keep the logits in sigmoid's unsaturated range
        return 0.1 * x / math.sqrt(fan_in)
    if name.endswith((".merge.weight", ".down.weight")):  # residual branches (model.py:142-144)
        return x / math.sqrt(fan_in * 2 * depth)
    return x / math.sqrt(fan_in)


_HEADS = ("decoder.file_head.2.", "decoder.voice_head.", "decoder.music_head.")


def student_state(shapes, seed=0):
    """State dict for ``{name: shape}`` (a model's parameter/buffer layout)."""
    blocks = {int(k.split(".")[1]) for k in shapes if k.startswith("blocks.")}
    depth = max(blocks) + 1 if blocks else 1
    return {name: parameter_value(name, tuple(shape), seed, depth)
            for name, shape in sorted(shapes.items())}


def student_checkpoint(path, config, seed=0):
    """Write a reference-format checkpoint (``{"model_config", "model"}``) with
    synthetic weights for ``config`` (a dict of ``ModelConfig`` fields)."""
    from .model import ModelConfig, TriFusion

    with torch.device("meta"):
        model = TriFusion(ModelConfig(**config))
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    torch.save({"model_config": dict(config), "model": student_state(shapes, seed)}, path)
    return path


def synthetic_audio(batch, samples, *, channels=None, lengths=None, seed=0):
    """PCM16-quantised Gaussian noise (sigma 0.1) ``[B, C, samples]`` FP32,
    zero past each length and in absent channels; returns (audio, lengths,
    channels) as CPU tensors."""
    g = torch.Generator().manual_seed(seed)
    if channels is None:
        channels = torch.ones(batch, dtype=torch.int64)
    channels = torch.as_tensor(channels, dtype=torch.int64)
    if lengths is None:
        lengths = torch.full((batch,), samples, dtype=torch.int64)
    lengths = torch.as_tensor(lengths, dtype=torch.int64)
    c = int(channels.max())
    wave = torch.randn(batch, c, samples, generator=g) * 0.1
    wave = torch.clamp(torch.round(wave * 32768), -32768, 32767) / 32768
    keep = torch.arange(samples)[None, None, :] < lengths[:, None, None]
    keep = keep & (torch.arange(c)[None, :, None] < channels[:, None, None])
    return wave * keep, lengths, channels


def clip_set(count=1024, *, seed=0, min_seconds=1.0, max_seconds=72.0, stereo_fraction=0.3):
    """Synthetic clip records for the box-level sweep: durations log-uniform in
    [min_seconds, max_seconds], ``stereo_fraction`` of them two-channel."""
    from .audio import SAMPLE_RATE, AudioFile

    g = torch.Generator().manual_seed(seed)
    u = torch.rand(count, generator=g, dtype=torch.float64)
    seconds = torch.exp(math.log(min_seconds) + u * (math.log(max_seconds) - math.log(min_seconds)))
    stereo = torch.rand(count, generator=g, dtype=torch.float64) < stereo_fraction
    return [AudioFile(i, None, max(1, min(int(round(float(s) * SAMPLE_RATE)), 72 * SAMPLE_RATE)),
                      2 if bool(st) else 1)
            for i, (s, st) in enumerate(zip(seconds, stereo))]


def batch_audio(limit, rows, *, seed=0):
    """Padded ``[len(rows), channels, limit]`` audio for one planned batch, each
    clip PCM16-quantised noise from its own seed; returns (audio, lengths, channels)."""
    c = max(r.channels for r in rows)
    audio = torch.zeros(len(rows), c, limit)
    for i, r in enumerate(rows):
        clip, _, _ = synthetic_audio(1, r.samples, channels=[r.channels], seed=seed * 1_000_003 + r.index)
        audio[i, :r.channels, :r.samples] = clip[0, :r.channels]
    lengths = torch.tensor([r.samples for r in rows], dtype=torch.int64)
    channels = torch.tensor([r.channels for r in rows], dtype=torch.int64)
    return audio, lengths, channels
