"""Row-norm and decoder-read operators on B200 — drop-in for
``trifusion_l4.kernels.native`` (reference ``kernels/native.py``).

Every function launches a kernel of ``libtrifusion_b200.so`` on the current
stream (FP32 statistics, one rounding to the output type). Inputs are made
contiguous first, as the reference wrappers do.
"""

from __future__ import annotations

import torch

from .. import _lib


def _rows(x):
    d = x.shape[-1]
    return (x.numel() // d if d else 0), d


def _weight(weight, d, op):
    w = weight.detach().float().contiguous()
    if w.numel() != d:
        raise ValueError(f"{op}: weight has {w.numel()} elements, rows have {d}")
    return w


def rms(x, weight, eps=1e-5, out_dtype=None):
    """``x * rsqrt(mean(x^2) + eps) * weight``; output dtype = ``x.dtype``
    (reference ``native.py:69-70``), or ``out_dtype`` (FP32/BF16: the FP32 result
    rounded once, what autocast would pass to the next projection)."""
    x = x.contiguous()
    dev = _lib.require_cuda("rms", x, weight)
    code = _lib.dtype_code(x, "rms")
    rows, d = _rows(x)
    w = _weight(weight, d, "rms")
    if out_dtype is None or out_dtype == x.dtype:
        y = torch.empty_like(x)
        _lib.launch("tf_rms_fwd", dev, x.data_ptr(), code, w.data_ptr(), y.data_ptr(), rows, d,
                    float(eps))
        return y
    y = torch.empty(x.shape, device=dev, dtype=out_dtype)
    _lib.launch("tf_rms_out_fwd", dev, x.data_ptr(), code, w.data_ptr(), y.data_ptr(),
                _lib.dtype_code(y, "rms"), rows, d, float(eps))
    return y


def _row_pitch(t, width, op):
    """Elements between consecutive rows of ``t`` (all leading dims flattened into rows):
    ``t`` may be the slice of a wider row buffer, but its last dim must be contiguous
    and its rows evenly spaced."""
    if t.dim() < 1 or t.shape[-1] != width or (width > 1 and t.stride(-1) != 1):
        raise ValueError(f"{op}: output must be [..., {width}] with a contiguous last dim")
    lead = [(t.shape[i], t.stride(i)) for i in range(t.dim() - 1) if t.shape[i] > 1]
    if not lead:
        return width
    pitch = expected = lead[-1][1]
    for size, stride in reversed(lead):
        if stride != expected:
            raise ValueError(f"{op}: output rows must be evenly spaced")
        expected *= size
    if pitch < width:
        raise ValueError(f"{op}: output rows overlap")
    return pitch


def rms_into(x, weight, eps, out, out2=None):
    """RMSNorm of ``x``'s rows written into ``out`` (FP32 or BF16; may be the slice of a
    wider concatenated row) and, when ``out2`` is given, the same values rounded once
    into the BF16 view ``out2``: the norm writes its part of a ``torch.cat`` input
    in place (model.py:159-161, 185). Returns ``out``."""
    x = x.contiguous()
    dev = _lib.require_cuda("rms_into", x, weight, out)
    rows, d = _rows(x)
    w = _weight(weight, d, "rms_into")
    if out.shape != x.shape:
        raise ValueError("rms_into: out must have x's shape")
    pitch = _row_pitch(out, d, "rms_into")
    ptr2, pitch2 = None, 0
    if out2 is not None:
        if out2.shape != x.shape or out2.dtype != torch.bfloat16 or out2.device != out.device:
            raise ValueError("rms_into: out2 must be a BF16 tensor of x's shape on out's device")
        ptr2, pitch2 = out2.data_ptr(), _row_pitch(out2, d, "rms_into")
    _lib.launch("tf_rms_pitched_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "rms_into"), w.data_ptr(),
                out.data_ptr(), _lib.dtype_code(out, "rms_into"), pitch, ptr2, pitch2, rows, d, float(eps))
    return out


def add_rms(x, a, weight, eps=1e-5, out_dtype=torch.bfloat16):
    """``(x + a, rms(x + a))``: the FP32 residual sum (x FP32, a FP32 or BF16) and its
    RMSNorm in ``out_dtype`` (rounded once), in one pass (model.py:197-198)."""
    x, a = x.contiguous(), a.contiguous()
    dev = _lib.require_cuda("add_rms", x, a, weight)
    if x.dtype != torch.float32 or a.shape != x.shape:
        raise ValueError("add_rms: x must be FP32 and a of the same shape")
    rows, d = _rows(x)
    w = _weight(weight, d, "add_rms")
    total = torch.empty_like(x)
    y = torch.empty(x.shape, device=dev, dtype=out_dtype)
    _lib.launch("tf_add_rms_fwd", dev, x.data_ptr(), a.data_ptr(), _lib.dtype_code(a, "add_rms"), w.data_ptr(),
                total.data_ptr(), y.data_ptr(), _lib.dtype_code(y, "add_rms"), rows, d, float(eps))
    return total, y


def rms_silu(x, weight, eps=1e-5):
    """``silu(rms(x))`` with the norm rounded to x's type first, as PyTorch's silu
    sees the norm's output tensor (model.py:120)."""
    x = x.contiguous()
    dev = _lib.require_cuda("rms_silu", x, weight)
    rows, d = _rows(x)
    w = _weight(weight, d, "rms_silu")
    y = torch.empty_like(x)
    _lib.launch("tf_rms_silu_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "rms_silu"), w.data_ptr(), y.data_ptr(),
                rows, d, float(eps))
    return y


def evidence_norm(x, value, gate, weight, mask, eps=1e-5, out_dtype=torch.float32):
    """RMSNorm of ``x + value * 2 sigmoid(gate)`` on rows where ``mask`` is set
    (zero rows elsewhere); FP32 output (reference ``native.py:73-74``), or BF16 (the
    FP32 result rounded once) with ``out_dtype``. ``value`` and ``gate`` may be views
    whose rows share one pitch (the halves of a stacked projection row): they are
    read in place."""
    x = x.contiguous()
    if value.dtype != gate.dtype:
        value, gate = value, gate.to(value.dtype)
    dev = _lib.require_cuda("evidence_norm", x, value, gate, weight, mask)
    rows, d = _rows(x)
    if value.shape != x.shape or gate.shape != x.shape or mask.numel() != rows:
        raise ValueError("evidence_norm: value/gate must match x and mask must have one entry per row")
    try:
        pitch = _row_pitch(value, d, "evidence_norm")
        if _row_pitch(gate, d, "evidence_norm") != pitch:
            raise ValueError("evidence_norm: value and gate rows differ in pitch")
    except ValueError:
        value, gate, pitch = value.contiguous(), gate.contiguous(), d
    w = _weight(weight, d, "evidence_norm")
    m = mask.contiguous()
    m = m.view(torch.uint8) if m.dtype == torch.bool else m.to(torch.uint8)
    y = torch.empty(x.shape, device=dev, dtype=out_dtype)
    _lib.launch("tf_evidence_norm_pitched_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "evidence_norm"),
                value.data_ptr(), gate.data_ptr(), _lib.dtype_code(value, "evidence_norm"), pitch,
                w.data_ptr(), m.data_ptr(), y.data_ptr(), _lib.dtype_code(y, "evidence_norm"), rows, d,
                float(eps))
    return y


def mean_norm(a, b, weight, eps=1e-5, copy_to=None):
    """RMSNorm of ``(a + b) / 2``; FP32 output (reference ``native.py:77-78``). With
    ``copy_to`` (a BF16 view of the output's shape, rows evenly spaced) the result is
    also written there rounded once."""
    a, b = a.contiguous(), b.contiguous()
    if b.dtype != a.dtype:
        b = b.to(a.dtype)
    dev = _lib.require_cuda("mean_norm", a, b, weight)
    if a.shape != b.shape:
        raise ValueError("mean_norm: a and b must have the same shape")
    rows, d = _rows(a)
    w = _weight(weight, d, "mean_norm")
    y = torch.empty(a.shape, device=dev, dtype=torch.float32)
    if copy_to is not None:
        if copy_to.shape != a.shape or copy_to.dtype != torch.bfloat16 or copy_to.device != y.device:
            raise ValueError("mean_norm: copy_to must be a BF16 tensor of the output's shape")
        _lib.launch("tf_mean_norm_copy_fwd", dev, a.data_ptr(), b.data_ptr(), _lib.dtype_code(a, "mean_norm"),
                    w.data_ptr(), y.data_ptr(), copy_to.data_ptr(), _row_pitch(copy_to, d, "mean_norm"), rows, d,
                    float(eps))
        return y
    _lib.launch("tf_mean_norm_fwd", dev, a.data_ptr(), b.data_ptr(), _lib.dtype_code(a, "mean_norm"),
                w.data_ptr(), y.data_ptr(), rows, d, float(eps))
    return y


def masked_mean(x, lengths):
    """``(x.float() * mask).sum(1) / lengths`` over ``[B, T, D]`` → FP32 ``[B, D]``
    (the decoder's global feature, reference ``decoder.py:60-62``)."""
    x = x.contiguous()
    dev = _lib.require_cuda("masked_mean", x, lengths)
    b, t, d = x.shape
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty((b, d), device=dev, dtype=torch.float32)
    _lib.launch("tf_masked_mean_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "masked_mean"),
                lengths.data_ptr(), y.data_ptr(), b, t, d)
    return y


def pooled_attention(qkv, cos, sin, lengths, heads):
    """A block's attention over its pooled rows (reference ``model.py:127-133`` after
    the qkv projection): ``qkv`` BF16 ``[B, LT, 3 * heads * 64]``, q/k rotated by the
    ``[>= LT, 32]`` cos/sin table and rounded to BF16, FP32 masked softmax attention
    with key j valid when ``j < lengths[b]``. Returns the BF16 ``[B, LT, heads * 64]``
    rows the out projection reads."""
    dev = _lib.require_cuda("pooled_attention", qkv, cos, sin, lengths)
    b, t, width = qkv.shape
    if qkv.dtype != torch.bfloat16 or width != 3 * heads * 64:
        raise ValueError("pooled_attention: qkv must be BF16 [B, LT, 3 * heads * 64]")
    if cos.shape[0] < t or cos.shape[-1] != 32 or sin.shape != cos.shape:
        raise ValueError("pooled_attention: the rotary table must be [>= LT, 32]")
    qkv = qkv.contiguous()
    cos, sin = cos.float().contiguous(), sin.float().contiguous()
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty((b, t, heads * 64), device=dev, dtype=torch.bfloat16)
    _lib.launch("tf_pooled_attention_fwd", dev, qkv.data_ptr(), cos.data_ptr(), sin.data_ptr(), lengths.data_ptr(),
                y.data_ptr(), b, t, heads, 64)
    return y


def query_read(q, kv, lengths, keys_per_length=1):
    """The decoder's query-read attention (reference ``decoder.py:26-30``): ``q`` the
    BF16 ``[10, 256]`` query projection, ``kv`` the BF16 ``[B, T, 512]`` key/value
    projection (rows may be the slices of wider rows), key j of batch entry b valid
    when ``j < lengths[b] * keys_per_length``. Returns the BF16 ``[B, 10, 256]`` rows
    the out projection reads (the 8 heads side by side), FP32 softmax inside."""
    dev = _lib.require_cuda("query_read", q, kv, lengths)
    if q.dtype != torch.bfloat16 or kv.dtype != torch.bfloat16 or tuple(q.shape) != (10, 256):
        raise ValueError("query_read: q must be BF16 [10, 256] and kv BF16 [B, T, 512]")
    if kv.dim() != 3 or kv.shape[-1] != 512:
        raise ValueError("query_read: kv must be [B, T, 512]")
    q = q.contiguous()
    b, t, _ = kv.shape
    pitch = _row_pitch(kv, 512, "query_read")
    if kv.data_ptr() % 16 or pitch % 8:
        kv = kv.contiguous()
        pitch = 512
    lengths = lengths.to(torch.int64).contiguous()
    n = int(_lib.lib().tf_query_read_state_floats(b, t))
    state = torch.empty(max(n, 1), device=dev, dtype=torch.float32)
    y = torch.empty((b, 10, 256), device=dev, dtype=torch.bfloat16)
    _lib.launch("tf_query_read_fwd", dev, q.data_ptr(), kv.data_ptr(), pitch, lengths.data_ptr(),
                int(keys_per_length), state.data_ptr(), n, y.data_ptr(), b, t)
    return y


def local_topk(local, features, fine_lengths):
    """The decoder's local evidence (reference ``decoder.py:65-76``): ``local`` the BF16
    ``[B, T, 2]`` local logits and ``features`` the BF16 ``[B, T, 256]`` local features
    (either may be a column slice of wider rows, such as one GEMM's output over both
    layers). Returns ``(local.float(), top)``: the FP32 logits and the FP32 ``[B, 2, 256]``
    masked mean of the features at the ``min(25, T)`` highest-scoring valid frames of each
    class (frames ``t >= fine_lengths[b]`` score -inf; ties at the k-th score resolve to the
    earliest frames)."""
    dev = _lib.require_cuda("local_topk", local, features, fine_lengths)
    if local.dtype != torch.bfloat16 or features.dtype != torch.bfloat16:
        raise ValueError("local_topk: local and features must be BF16")
    if local.dim() != 3 or local.shape[-1] != 2 or features.dim() != 3 or features.shape[-1] != 256:
        raise ValueError("local_topk: local must be [B, T, 2] and features [B, T, 256]")
    if local.shape[:2] != features.shape[:2]:
        raise ValueError("local_topk: local and features must share [B, T]")
    b, t = local.shape[:2]

    def pitch_of(x, width):  # rows evenly spaced (a column slice of wider rows), else a copy
        try:
            return x, _row_pitch(x, width, "local_topk")
        except ValueError:
            return x.contiguous(), width

    local, lp = pitch_of(local, 2)
    features, fp = pitch_of(features, 256)
    fine_lengths = fine_lengths.to(torch.int64).contiguous()
    local_f32 = torch.empty((b, t, 2), device=dev, dtype=torch.float32)
    top = torch.empty((b, 2, 256), device=dev, dtype=torch.float32)
    _lib.launch("tf_local_topk_fwd", dev, local.data_ptr(), lp, features.data_ptr(), fp, fine_lengths.data_ptr(),
                local_f32.data_ptr(), top.data_ptr(), b, t)
    return local_f32, top


def decoder_heads(deep_rows, fine_rows, global_feature, memory, top, decoder):
    """The decoder's heads and logits row (reference ``decoder.py:77-89``) in three
    launches: ``deep_rows``/``fine_rows`` the query reads' BF16 ``[B, 10, 256]``
    out-projection rows (their 4/4/2 group means are taken inside), ``global_feature``
    and ``memory`` BF16 ``[B, 256]``, ``top`` FP32 ``[B, 2, 256]``, ``decoder`` the module
    holding ``voice_lat``, ``music_lat``, ``voice_head``, ``music_head`` and
    ``file_head``. Returns the FP32 ``[B, 5]`` logits ``[f, v0, m0, v1, m1]``; every
    projection rounds to BF16 as under BF16 autocast."""
    from .buffers import _param_bf16

    dev = _lib.require_cuda("decoder_heads", deep_rows, fine_rows, global_feature, memory, top)
    b = deep_rows.shape[0]
    shapes = ((deep_rows, (b, 10, 256), torch.bfloat16), (fine_rows, (b, 10, 256), torch.bfloat16),
              (global_feature, (b, 256), torch.bfloat16), (memory, (b, 256), torch.bfloat16),
              (top, (b, 2, 256), torch.float32))
    for x, shape, dtype in shapes:
        if tuple(x.shape) != shape or x.dtype != dtype:
            raise ValueError(f"decoder_heads: expected {dtype} {list(shape)}, got {x.dtype} {list(x.shape)}")

    def aligned(x):  # contiguous and 16-byte aligned (the kernels read 16-byte vectors)
        x = x.contiguous()
        return x if x.data_ptr() % 16 == 0 else x.clone()

    deep_rows, fine_rows, global_feature, memory, top = (aligned(x) for x in
                                                         (deep_rows, fine_rows, global_feature, memory, top))
    layers = (decoder.voice_lat[0], decoder.music_lat[0], decoder.voice_head, decoder.music_head,
              decoder.file_head[0], decoder.file_head[2])
    params = []
    for layer in layers:
        params += [_param_bf16(layer.weight, tuple(layer.weight.shape)), _param_bf16(layer.bias, tuple(layer.bias.shape))]
    scratch = torch.empty(max(int(_lib.lib().tf_decoder_heads_scratch_bytes(b)), 16), device=dev, dtype=torch.uint8)
    logits = torch.empty((b, 5), device=dev, dtype=torch.float32)
    _lib.launch("tf_decoder_heads_fwd", dev, deep_rows.data_ptr(), fine_rows.data_ptr(), global_feature.data_ptr(),
                memory.data_ptr(), top.data_ptr(), *[t.data_ptr() for t in params], scratch.data_ptr(),
                scratch.numel(), logits.data_ptr(), b)
    return logits


def end_gather(x, lengths):
    """``x[arange(B), lengths - 1]`` — the last valid row of each batch entry
    (reference ``decoder.py:63``); bit-exact."""
    x = x.contiguous()
    dev = _lib.require_cuda("end_gather", x, lengths)
    b, t = x.shape[:2]
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty((b, *x.shape[2:]), device=dev, dtype=x.dtype)
    row_bytes = x[0, 0].numel() * x.element_size() if t else 0
    if b and t == 0:
        raise IndexError("end_gather: time dimension is empty")
    _lib.launch("tf_end_gather_fwd", dev, x.data_ptr(), lengths.data_ptr(), y.data_ptr(), b, t,
                row_bytes)
    return y


def bands(x):
    """Average the frequency axis of [B, C, T, F] into 8 bands -> [B, T, 8, C]
    (reference ``native.py:157-163``)."""
    x = x.contiguous(memory_format=torch.channels_last)
    dev = _lib.require_cuda("bands", x)
    b, c, t, f = x.shape
    y = torch.empty((b, t, 8, c), device=dev, dtype=x.dtype)
    _lib.launch("tf_bands_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "bands"), y.data_ptr(), b, t, f, c)
    return y


def interpolate(low, grids):
    """Pooled rows back to the main grid: ``a + (z - a) * alpha`` of the left and
    right pooled rows, zero past each length (reference ``native.py:119-138``)."""
    low = low.contiguous()
    dev = _lib.require_cuda("interpolate", low, grids.left)
    b, t = grids.left.shape
    d = low.shape[-1]
    if low.dtype != torch.bfloat16 or d % 4:
        raise ValueError("interpolate: expects BF16 rows whose width is a multiple of 4")
    y = low.new_empty((b, t, d))
    left, right = grids.left.contiguous(), grids.right.contiguous()
    alpha = grids.alpha.float().contiguous()
    lengths = grids.lengths.to(torch.int64).contiguous()
    _lib.launch("tf_interpolate_fwd", dev, low.data_ptr(), left.data_ptr(), right.data_ptr(), alpha.data_ptr(),
                lengths.data_ptr(), y.data_ptr(), b, t, low.shape[1], d)
    return y
