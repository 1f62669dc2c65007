"""CPU oracle for the fused Mamba-3 recurrence hot path.

TEST INFRASTRUCTURE ONLY. This module is the checker for the CUDA kernels in
``trifusion-fp-kernel_b200/csrc``. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and its ``--impl reference`` arm)
import it. The product path never calls it, and there is no CPU fallback.

Everything here is a numpy restatement of the reference's arithmetic
(tlstngud/TriFusion-FP-Kernel 0.1.0, package ``trifusion_l4``). Each function
cites the reference lines it follows. Parity is pinned by
``tests/test_oracle_golden.py`` against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own Triton
kernels (under the Triton interpreter, FP32 inputs) and the reference's own
PyTorch formulas.

Two flavours of the recurrence exist:

* ``bf16=False`` (default) is the reference's FP32 path: the reference kernels
  fed FP32 tensors, where every ``.to(Q.dtype)`` rounding point is a no-op.
  This is what the CUDA output is held to (atol/rtol 1e-2).
* ``bf16=True`` rounds to BF16 at exactly the points the reference's fused
  kernel does with BF16 inputs (``mamba_fused.py:127-132,143,146,151-152``).

Trigonometric and hyperbolic functions are evaluated exactly (numpy), where
the reference uses ``cos.approx``/``sin.approx``/``tanh.approx``
(``vendor/utils.py:13-69``); the difference is far below the tolerance.
"""

from __future__ import annotations

import numpy as np

# Literal constants of the reference kernel (mamba_fused.py:105,107,140).
LOG2E = 1.44269504089
PI = 3.141592653589793
TWO_PI = 6.283185307179586
CHUNK = 64
STATE = 128  # N, width of q/k (mamba_fused.py:159)
HEAD = 64  # P, head dim of v/z/out
ROTARY = 32  # R, rotated pairs (the remaining N/2-R pairs have phase 0)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest BF16 value (ties to even).

    Returns float32 arrays holding BF16-representable values, which is how
    ``tensor.to(torch.bfloat16)`` rounds finite numbers.
    """
    f = np.ascontiguousarray(x, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(f.shape)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen raw BF16 bit patterns (uint16) to float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Raw BF16 bit patterns (uint16) of float32 values, rounded to nearest even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def fused_mamba(q, k, v, adt, dt, trap, qb, kb, angles, d, z, *, bf16=False,
                dtype=np.float64, chunk=CHUNK):
    """Chunked Mamba-3 SISO forward: the arithmetic of ``mamba_fused.py:72-152``.

    Shapes follow the reference contract (``docs/api.md:61-69``):
    q, k ``[B,T,Hq,128]``; v, z ``[B,T,H,64]``; adt, dt, trap ``[B,H,T]``;
    qb, kb ``[H,128]``; angles ``[B,T,H,32]`` (raw, pre-tanh); d ``[H]``.
    Returns ``[B,T,H,64]`` in ``dtype`` (BF16-rounded when ``bf16``).

    Vectorised over (batch, head); the chunk loop is serial as in the
    reference (``mamba_fused.py:93``).
    """
    q, k, v, z, angles = (np.asarray(a, dtype=dtype) for a in (q, k, v, z, angles))
    adt, dt, trap = (np.asarray(a, dtype=dtype) for a in (adt, dt, trap))
    qb, kb, d = (np.asarray(a, dtype=dtype) for a in (qb, kb, d))
    b, t, h, p = v.shape
    n = q.shape[-1]
    r = angles.shape[-1]
    hq = q.shape[2]
    if n != STATE or p != HEAD or r != ROTARY:
        raise ValueError("L4 recurrence requires state=128, head=64, rotary=32")
    if h % hq:
        raise ValueError("heads must be divisible by q/k groups")
    rnd = bf16_round if bf16 else (lambda x: x)
    qh = np.arange(h) // (h // hq)  # mamba_fused.py:74
    out = np.zeros((b, t, h, p), dtype=dtype)
    state = np.zeros((b, h, p, n), dtype=dtype)  # :91
    angle_state = np.zeros((b, h, n // 2), dtype=dtype)  # :92
    ti = np.arange(chunk)
    lower = ti[:, None] > ti[None, :]  # :145 strictly lower triangle
    for c0 in range(0, t, chunk):
        pos = c0 + ti
        valid = pos < t
        nvalid = int(valid.sum())
        sl = slice(c0, c0 + nvalid)

        def ctrl(x, shift, fill):
            # Load a [B,H,T] control at pos+shift; masked lanes read `fill`.
            y = np.full((b, h, chunk), fill, dtype=dtype)
            src = pos + shift
            ok = src < t
            y[:, :, ok] = x[:, :, src[ok]]
            return y

        dtc = ctrl(dt, 0, 0.0)  # :96
        dn = ctrl(dt, 1, 0.0)  # :97
        tr = _sigmoid(ctrl(trap, 0, 0.0))  # :98 (masked lanes give sigmoid(0))
        tn = _sigmoid(ctrl(trap, 1, 0.0))  # :99
        gamma = dtc * tr  # :100
        scale = dn * (1 - tn) + gamma  # :101
        raw = np.zeros((b, h, chunk, n // 2), dtype=dtype)  # :102-104, ri < R
        raw[:, :, :nvalid, :r] = angles[:, sl].transpose(0, 2, 1, 3)
        vals = (np.tanh(raw) * PI) * dtc[..., None]  # :105
        phase = np.cumsum(vals, axis=2) + angle_state[:, :, None, :]  # :106
        phase = phase - TWO_PI * np.floor(phase / TWO_PI)  # :107
        angle_state = angle_state + vals.sum(axis=2)  # :108
        angle_state = angle_state - TWO_PI * np.floor(angle_state / TWO_PI)  # :109
        co, si = np.cos(phase), np.sin(phase)  # :110-111
        qc = np.zeros((b, h, chunk, n), dtype=dtype)
        kc = np.zeros((b, h, chunk, n), dtype=dtype)
        qc[:, :, :nvalid] = q[:, sl][:, :, qh].transpose(0, 2, 1, 3)
        kc[:, :, :nvalid] = k[:, sl][:, :, qh].transpose(0, 2, 1, 3)
        qc = qc + qb[None, :, None, :]  # :112-117
        kc = kc + kb[None, :, None, :]  # :118-123
        qk = (qc * kc).sum(-1) * gamma  # :124 (pre-rotation)
        q0, q1 = qc[..., 0::2], qc[..., 1::2]  # :125 interleaved pairs
        k0, k1 = kc[..., 0::2], kc[..., 1::2]  # :126
        qr = np.empty_like(qc)
        kr = np.empty_like(kc)
        qr[..., 0::2] = q0 * co - q1 * si  # :127
        qr[..., 1::2] = q0 * si + q1 * co
        kr[..., 0::2] = k0 * co - k1 * si  # :130-131
        kr[..., 1::2] = k0 * si + k1 * co
        qr = rnd(qr)
        kr = rnd(kr * scale[..., None])
        qr[:, :, nvalid:] = 0  # :134-135
        kr[:, :, nvalid:] = 0
        vc = np.zeros((b, h, chunk, p), dtype=dtype)  # :136
        zc = np.zeros((b, h, chunk, p), dtype=dtype)  # :137
        vc[:, :, :nvalid] = v[:, sl].transpose(0, 2, 1, 3)
        zc[:, :, :nvalid] = z[:, sl].transpose(0, 2, 1, 3)
        da = ctrl(adt, 0, 0.0) * LOG2E  # :140
        cs = np.cumsum(da, axis=2)  # :141
        total = da.sum(axis=2)  # :142
        acc = (qr @ np.swapaxes(rnd(state), -1, -2)) * np.exp2(cs)[..., None]  # :143
        score = (qr @ np.swapaxes(kr, -1, -2)) * np.exp2(
            np.minimum(cs[..., :, None] - cs[..., None, :], 0.0))  # :144
        score = np.where(lower, score, 0.0)  # :145
        acc = acc + rnd(score) @ vc  # :146
        acc = acc + (d[None, :, None] + qk)[..., None] * vc  # :147
        acc = acc * (zc * _sigmoid(zc))  # :148
        out[:, sl] = acc[:, :, :nvalid].transpose(0, 2, 1, 3)  # :149
        scaled = rnd(vc * np.exp2(total[..., None] - cs)[..., None])  # :151
        state = state * np.exp2(total)[..., None, None] + np.swapaxes(scaled, -1, -2) @ kr  # :152
    return bf16_round(out).astype(dtype) if bf16 else out


def fused_mamba_stepwise_f64(q, k, v, adt, dt, trap, qb, kb, angles, d, z):
    """Independent unchunked FP64 recurrence of ``tests/test_recurrence.py:54-85``.

    Generalised from the test's fixed (1,17,4) to any [B,T,H] and any Hq
    dividing H. No chunking, no mod-2pi, no BF16 rounding.
    """
    q, k, v, z = (np.asarray(a, dtype=np.float64) for a in (q, k, v, z))
    adt, dt, trap = (np.asarray(a, dtype=np.float64) for a in (adt, dt, trap))
    qb, kb, d = (np.asarray(a, dtype=np.float64) for a in (qb, kb, d))
    angles = np.asarray(angles, dtype=np.float64)
    b, t, h, p = v.shape
    hq = q.shape[2]
    r = angles.shape[-1]
    qh = np.arange(h) // (h // hq)
    # :54-55 phase = cumsum(tanh(raw)*pi*dt) over time, padded to N/2 pairs
    phase = np.cumsum(np.tanh(angles) * np.pi * dt.transpose(0, 2, 1)[..., None], axis=1)
    phase = np.concatenate([phase, np.zeros(phase.shape[:-1] + (STATE // 2 - r,))], -1)

    def rotate(x, bias):  # :57-62
        x = x[:, :, qh] + bias[None, None]
        a, c = x[..., 0::2], x[..., 1::2]
        y = np.empty_like(x)
        y[..., 0::2] = a * np.cos(phase) - c * np.sin(phase)
        y[..., 1::2] = a * np.sin(phase) + c * np.cos(phase)
        return y

    qr, kr = rotate(q, qb), rotate(k, kb)
    sig = _sigmoid(trap)
    gamma = dt * sig  # :65
    shifted = np.concatenate([(dt * (1 - sig))[:, :, 1:], np.zeros((b, h, 1))], -1)  # :66-68
    scale = gamma + shifted  # :69
    state = np.zeros((b, h, p, STATE))
    out = np.zeros((b, t, h, p))
    qq = q[:, :, qh] + qb[None, None]
    kk = k[:, :, qh] + kb[None, None]
    for i in range(t):  # :72-83
        decay = np.exp(adt[:, :, i])
        vi = v[:, i]
        previous = np.einsum("bhn,bhpn->bhp", qr[:, i], state) * decay[..., None]
        direct = (qq[:, i] * kk[:, i]).sum(-1) * gamma[:, :, i]
        silu = z[:, i] * _sigmoid(z[:, i])
        out[:, i] = (previous + (d + direct)[..., None] * vi) * silu
        state = state * decay[..., None, None] + (
            vi[..., None] * kr[:, i, :, None, :] * scale[:, :, i, None, None])
    return out


def angle_phase(angles, dt, chunk=CHUNK):
    """Phase scan of ``angle.py:103-144``: (cumsum tanh(a)*pi*dt + carry) mod 2pi.

    angles ``[B,T,H,R]`` raw, dt ``[B,H,T]``; returns ``[B,T,H,R]``.
    """
    angles = np.asarray(angles, dtype=np.float64)
    dt = np.asarray(dt, dtype=np.float64)
    b, t, h, r = angles.shape
    out = np.zeros((b, t, h, r))
    state = np.zeros((b, h, r))
    for c0 in range(0, t, chunk):
        sl = slice(c0, min(c0 + chunk, t))
        vals = np.tanh(angles[:, sl]) * PI * dt[:, :, sl].transpose(0, 2, 1)[..., None]
        ph = np.cumsum(vals, axis=1) + state[:, None]
        out[:, sl] = ph - TWO_PI * np.floor(ph / TWO_PI)
        state = state + vals.sum(1)
        state = state - TWO_PI * np.floor(state / TWO_PI)
    return out


# ---------------------------------------------------------------------------
# Satellite operations around the recurrence. Inputs may be BF16-valued float32
# arrays; `out_bf16` rounds the result the way a BF16 output tensor would.
# ---------------------------------------------------------------------------


def rms(x, weight, eps=1e-5, out_bf16=True):
    """RMSNorm with FP32 statistics: ``kernels/__init__.py:10-12``,
    ``kernels/native.py:8-39`` (MODE 0). Output dtype = input dtype."""
    xf = np.asarray(x, dtype=np.float32)
    ms = (xf.astype(np.float64) ** 2).mean(-1, keepdims=True)
    y = xf * (1.0 / np.sqrt(ms + eps)) * np.asarray(weight, dtype=np.float64)
    return bf16_round(y.astype(np.float32)) if out_bf16 else y.astype(np.float32)


def mean_norm(a, b, weight, eps=1e-5):
    """RMSNorm((a+b)/2) with FP32 output: ``native.py:35-37,77-78``;
    reference formula ``model.py:183``."""
    x = (np.asarray(a, np.float64) + np.asarray(b, np.float64)) * 0.5
    ms = (x ** 2).mean(-1, keepdims=True)
    return (x / np.sqrt(ms + eps) * np.asarray(weight, np.float64)).astype(np.float32)


def mamba_controls(a, ddt, dt_bias, floor=1e-4):
    """A/dt controls: ``primitives.py:190-216`` / ``mamba.py:59-63``.

    a, ddt ``[B,T,H]`` -> (adt, dt) ``[B,H,T]`` FP32:
    A = min(-(relu(a) + 1/(1-min(a,0))), -floor); dt = softplus(ddt+bias)
    with the ``v > 20 -> v`` threshold; adt = A*dt.
    """
    a = np.asarray(a, np.float64)
    x = np.asarray(ddt, np.float64) + np.asarray(dt_bias, np.float64)
    control = np.minimum(-(np.maximum(a, 0) + 1 / (1 - np.minimum(a, 0))), -floor)
    step = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))
    adt = (control * step).transpose(0, 2, 1)
    return adt.astype(np.float32), step.transpose(0, 2, 1).astype(np.float32)


def time_mask(lengths, t):
    """``masking.py:6-7``."""
    return np.arange(t)[None, :] < np.asarray(lengths)[:, None]


def mask_rows(x, lengths):
    """Length mask ``masking.py:10-11`` / ``primitives.py:65-70``: rows t >= len are 0."""
    x = np.asarray(x)
    m = time_mask(lengths, x.shape[1])
    return np.where(m.reshape(m.shape + (1,) * (x.ndim - 2)), x, 0).astype(x.dtype)


def reverse_valid(x, lengths):
    """``kernels/__init__.py:44-51``: y[b,t] = x[b,len-1-t] for t < len, else 0."""
    x = np.asarray(x)
    b, t = x.shape[:2]
    lengths = np.asarray(lengths)
    pos = np.arange(t)[None, :]
    idx = np.clip(lengths[:, None] - 1 - pos, 0, None)
    y = np.take_along_axis(x, idx.reshape(idx.shape + (1,) * (x.ndim - 2)), axis=1)
    keep = pos < lengths[:, None]
    return np.where(keep.reshape(keep.shape + (1,) * (x.ndim - 2)), y, 0).astype(x.dtype)


def swiglu(x, out_bf16=True):
    """``kernels/__init__.py:31-34``: silu(gate) * up over halves of the last dim."""
    xf = np.asarray(x, np.float64)
    g, u = np.split(xf, 2, axis=-1)
    y = (g * _sigmoid(g) * u).astype(np.float32)
    return bf16_round(y) if out_bf16 else y


def gated_concat(x, gate, out_bf16=True):
    """``kernels/__init__.py:58-64``: branch i of x scaled by 2*sigmoid(gate_i)."""
    xf = np.asarray(x, np.float64)
    g = np.asarray(gate, np.float64)
    y = (xf.reshape(*xf.shape[:-1], g.shape[-1], -1) * (2 * _sigmoid(g))[..., None])
    y = y.reshape(xf.shape).astype(np.float32)
    return bf16_round(y) if out_bf16 else y


def pool4(x, lengths, out_bf16=True):
    """Masked mean over groups of 4 frames: ``masking.py:59-69`` /
    ``primitives.py:90-113``. Divisor = number of valid frames, at least 1."""
    xf = np.asarray(x, np.float64)
    b, t, dd = xf.shape
    m = time_mask(lengths, t)
    pad = (-t) % 4
    xp = np.concatenate([np.where(m[..., None], xf, 0), np.zeros((b, pad, dd))], 1)
    mp = np.concatenate([m, np.zeros((b, pad), bool)], 1).reshape(b, -1, 4)
    y = xp.reshape(b, -1, 4, dd).sum(2) / np.maximum(mp.sum(2), 1)[..., None]
    y = y.astype(np.float32)
    return bf16_round(y) if out_bf16 else y


def pool4_f32(x, lengths, out_bf16=True):
    """Pool4 in the reference kernel's own arithmetic (``primitives.py:104-111``):
    FP32 accumulator starting at 0, valid frames added in order k = 0..3, one
    IEEE FP32 divide by the count. Bit-exact statement of the kernel."""
    xf = np.asarray(x, np.float32)
    b, t, dd = xf.shape
    lt = (t + 3) // 4
    lengths = np.minimum(np.maximum(np.asarray(lengths, np.int64), 0), t)
    acc = np.zeros((b, lt, dd), np.float32)
    for k in range(4):
        src = 4 * np.arange(lt) + k
        ok = src[None, :] < lengths[:, None]
        rows = np.take(xf, np.minimum(src, t - 1), axis=1)
        acc = np.where(ok[..., None], acc + rows, acc).astype(np.float32)
    y = (acc / pool4_counts(lengths, t).astype(np.float32)[..., None]).astype(np.float32)
    return bf16_round(y) if out_bf16 else y


def evidence_norm(x, value, gate, weight, mask, eps=1e-5):
    """``native.py:28-34,73-74`` (MODE 1): rows with mask set take
    x + value * 2 sigmoid(gate), other rows are zero; then RMSNorm; FP32 out."""
    xf = np.asarray(x, np.float64) + np.asarray(value, np.float64) * (
        2 * _sigmoid(np.asarray(gate, np.float64)))
    xf = np.where(np.asarray(mask, bool)[..., None], xf, 0.0)
    ms = (xf ** 2).mean(-1, keepdims=True)
    return (xf / np.sqrt(ms + eps) * np.asarray(weight, np.float64)).astype(np.float32)


def pool4_counts(lengths, t):
    """Integer divisors of `pool4`: clamp(min(len - 4g, 4), 1) (``primitives.py:294``)."""
    g = np.arange((t + 3) // 4)[None, :]
    return np.maximum(np.minimum(np.asarray(lengths)[:, None] - 4 * g, 4), 1).astype(np.int64)


def masked_mean(x, lengths):
    """Decoder global feature ``decoder.py:60-62``: sum over valid rows / length (FP32)."""
    xf = np.asarray(x, np.float64)
    m = time_mask(lengths, xf.shape[1])
    return ((xf * m[..., None]).sum(1) / np.asarray(lengths)[:, None]).astype(np.float32)


def end_gather(x, lengths):
    """Decoder end-state read ``decoder.py:63``: x[b, len[b]-1]."""
    x = np.asarray(x)
    return x[np.arange(x.shape[0]), np.asarray(lengths) - 1]


def algorithmic_bytes(b, t, h, hq=1, n=STATE, p=HEAD, r=ROTARY, trap_bytes=4,
                      angle_heads=1):
    """HBM bytes one fused_mamba call must move, each tensor touched once:
    q,k reads; v,z reads and out write; adt/dt/trap reads; angle reads
    (once per distinct head); qb,kb,d reads."""
    return (2 * b * t * hq * n * 2 + 3 * b * t * h * p * 2 + b * t * h * (4 + 4 + trap_bytes)
            + b * t * angle_heads * r * 2 + h * (2 * n + 1) * 4)
