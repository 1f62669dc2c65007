"""Buffer operators on B200 — drop-in for ``trifusion_l4.kernels.buffers``
(reference ``kernels/buffers.py``): length mask, Pool4 and the Mamba controls.
"""

from __future__ import annotations

import weakref

import torch

from .. import _lib


def _stamp(params):
    """Identity and state of ``params`` for a cache entry: weak references (a freed
    parameter whose id and address are reused never matches) plus each version
    counter and storage."""
    return tuple((weakref.ref(p), p._version, p.data_ptr(), p.device) for p in params)


def _stamp_matches(stamp, params):
    return len(stamp) == len(params) and all(
        ref() is p and (v, ptr, dev) == (p._version, p.data_ptr(), p.device)
        for (ref, v, ptr, dev), p in zip(stamp, params))


class ParamCache:
    """Tensors derived from parameters (casts, stacks), kept while the parameters
    stay the same live objects with the same version counters and storage.

    When a parameter changes, the entry is rebuilt and the superseded value stays
    allocated beside the new one for as long as the parameters live: a CUDA graph
    captured before the change still reads it (and must be recaptured to see the
    new values). When any of the parameters is garbage-collected, its entries and
    their superseded values are dropped, so loading and freeing models in one
    process does not accumulate device memory.
    """

    def __init__(self):
        self._entries = {}  # key -> (stamp, value, superseded values, token)

    def get(self, key, params, build):
        params = tuple(params)
        hit = self._entries.get(key)
        if hit is not None and _stamp_matches(hit[0], params):
            return hit[1]
        superseded = []
        if hit is not None and all(ref() is p for (ref, *_), p in zip(hit[0], params)):
            superseded = hit[2] + [hit[1]]  # same live parameters, new contents
        token = object()
        self._entries[key] = (_stamp(params), build(), superseded, token)
        for prm in params:
            weakref.finalize(prm, self._drop, key, token)
        return self._entries[key][1]

    def _drop(self, key, token):
        hit = self._entries.get(key)
        if hit is not None and hit[3] is token:
            del self._entries[key]

    def __len__(self):
        return len(self._entries)


_BF16_PARAMS = ParamCache()


def _param_bf16(param, shape):
    """A contiguous BF16 copy of ``param`` reshaped to ``shape``, cached until the
    parameter changes (its version counter or storage), so steady-state calls launch
    no conversion kernel."""
    return _BF16_PARAMS.get((id(param), shape), (param,),
                            lambda: param.detach().to(torch.bfloat16).reshape(shape).contiguous())


_STACKED = ParamCache()


def stacked_linear(layers, dtype, multiple=1):
    """The weights (and biases) of Linear ``layers`` that share an input, stacked into one
    ``[n * pitch, in]`` matrix (and ``[n * pitch]`` bias, or None) of ``dtype``: layer i's
    rows start at ``i * pitch``, its width rounded up to ``multiple`` with zero rows, so
    one GEMM computes all the layers and its output rows have aligned slices. Cached
    until a parameter changes (version counter or storage). Returns (weight, bias, pitch)."""
    params = [p for layer in layers for p in (layer.weight, layer.bias) if p is not None]
    key = (tuple(id(p) for p in params), dtype, multiple)

    def build():
        width, dim = layers[0].weight.shape
        if any(tuple(layer.weight.shape) != (width, dim) for layer in layers):
            raise ValueError("stacked_linear: the layers must have one shape")
        pitch = (width + multiple - 1) // multiple * multiple
        dev = layers[0].weight.device
        w = torch.zeros(len(layers) * pitch, dim, dtype=dtype, device=dev)
        has_bias = layers[0].bias is not None
        b = torch.zeros(len(layers) * pitch, dtype=dtype, device=dev) if has_bias else None
        for i, layer in enumerate(layers):
            w[i * pitch:i * pitch + width] = layer.weight.detach().to(dtype)
            if has_bias:
                b[i * pitch:i * pitch + width] = layer.bias.detach().to(dtype)
        return w, b, pitch

    return _STACKED.get(key, params, build)


def concat_linear(layers, dtype, multiple=8):
    """The weights and biases of Linear ``layers`` of any widths that share an input,
    stacked into one ``[sum of padded widths, in]`` matrix (and bias) of ``dtype``: layer
    i's rows start at ``offsets[i]``, each width rounded up to ``multiple`` with zero rows,
    so one GEMM computes every layer and each layer's output columns start on an aligned
    boundary. Every layer must have a bias. Cached like ``stacked_linear``. Returns
    (weight, bias, offsets)."""
    params = [p for layer in layers for p in (layer.weight, layer.bias)]
    key = ("concat",) + (tuple(id(p) for p in params), dtype, multiple)

    def build():
        dim = layers[0].weight.shape[1]
        if any(layer.weight.shape[1] != dim or layer.bias is None for layer in layers):
            raise ValueError("concat_linear: the layers must share the input width and have biases")
        offsets, rows = [], 0
        for layer in layers:
            offsets.append(rows)
            rows += (layer.weight.shape[0] + multiple - 1) // multiple * multiple
        dev = layers[0].weight.device
        w = torch.zeros(rows, dim, dtype=dtype, device=dev)
        b = torch.zeros(rows, dtype=dtype, device=dev)
        for off, layer in zip(offsets, layers):
            w[off:off + layer.weight.shape[0]] = layer.weight.detach().to(dtype)
            b[off:off + layer.weight.shape[0]] = layer.bias.detach().to(dtype)
        return w, b, tuple(offsets)

    return _STACKED.get(key, params, build)


def _mask_bytes(mask):
    """The mask as one byte per row, without a conversion pass for bool masks."""
    m = mask.contiguous()
    return m.view(torch.uint8) if m.dtype == torch.bool else m.to(torch.uint8)


def masked_add(a, b, mask):
    """``mask(a + b)``: FP32 ``a`` plus ``b`` (FP32 or BF16, added exactly in FP32) on
    rows where ``mask`` ([B, T] bool) is set, zero rows elsewhere; FP32 result
    (reference ``model.py:199``, the residual add and the ``_mask`` of ``buffers.py:6-10``)."""
    a, b = a.contiguous(), b.contiguous()
    dev = _lib.require_cuda("masked_add", a, b, mask)
    if a.dtype != torch.float32 or a.shape != b.shape or a.shape[-1] % 4:
        raise ValueError("masked_add: a must be FP32, b the same shape, width a multiple of 4")
    rows = mask.numel()
    if rows == 0 or a.numel() % rows:
        raise ValueError("masked_add: mask must have one entry per row")
    y = torch.empty_like(a)
    _lib.launch("tf_masked_add_fwd", dev, a.data_ptr(), b.data_ptr(), _lib.dtype_code(b, "masked_add"),
                _mask_bytes(mask).data_ptr(), y.data_ptr(), rows, a.numel() // rows)
    return y


def mask_buffer(x, mask):
    """Rows of ``x`` where ``mask`` ([B, T] bool) is False become zero; the
    others are copied bit for bit (reference ``buffers.py:6-10``)."""
    x = x.contiguous()
    dev = _lib.require_cuda("mask_buffer", x, mask)
    rows = mask.numel()
    if rows == 0 or x.numel() % rows:
        if x.numel() == 0:
            return torch.empty_like(x)
        raise ValueError("mask_buffer: mask must have one entry per row of x")
    m = _mask_bytes(mask)
    y = torch.empty_like(x)
    row_bytes = x.numel() // rows * x.element_size()
    _lib.launch("tf_mask_rows_fwd", dev, x.data_ptr(), m.data_ptr(), y.data_ptr(), rows, row_bytes)
    return y


class Pool4:
    """Mean over groups of 4 valid frames (reference ``buffers.py:35-43``)."""

    @staticmethod
    def apply(x, lengths, out_dtype=None):
        """``out_dtype`` BF16 for FP32 ``x``: the FP32 means rounded once (what autocast
        passes to the next projection)."""
        x = x.contiguous()
        dev = _lib.require_cuda("Pool4", x, lengths)
        b, t, d = x.shape
        lengths = lengths.to(torch.int64).contiguous()
        if out_dtype is None or out_dtype == x.dtype:
            y = x.new_empty((b, (t + 3) // 4, d))
            _lib.launch("tf_pool4_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "Pool4"),
                        lengths.data_ptr(), y.data_ptr(), b, t, d)
            return y
        y = torch.empty((b, (t + 3) // 4, d), device=dev, dtype=out_dtype)
        _lib.launch("tf_pool4_out_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "Pool4"), lengths.data_ptr(),
                    y.data_ptr(), _lib.dtype_code(y, "Pool4"), b, t, d)
        return y


def mamba_controls(a, dt, bias, floor):
    """``adt, dt`` as ``[B, H, T]`` FP32 from the ``[B, T, H]`` projection views
    (reference ``buffers.py:82-101``)."""
    dev = _lib.require_cuda("mamba_controls", a, dt, bias)
    if dt.dtype != a.dtype:
        dt = dt.to(a.dtype)
    if a.stride(-1) != 1:
        a = a.contiguous()
    if dt.stride(-1) != 1:
        dt = dt.contiguous()
    b, t, h = a.shape
    if tuple(dt.shape) != (b, t, h):
        raise ValueError("mamba_controls: a and dt must have the same [B, T, H] shape")
    bias = bias.detach().float().contiguous()
    oa = torch.empty((b, h, t), device=dev, dtype=torch.float32)
    od = torch.empty_like(oa)
    strides = _lib.int64_array([*a.stride(), *dt.stride()])
    _lib.launch("tf_mamba_controls_fwd", dev, a.data_ptr(), dt.data_ptr(),
                _lib.dtype_code(a, "mamba_controls"), strides, bias.data_ptr(), float(floor),
                oa.data_ptr(), od.data_ptr(), b, t, h)
    return oa, od


def _nhwc(x):
    """A [B, C, T, F] tensor in channels-last memory (rows of C contiguous)."""
    return x.contiguous(memory_format=torch.channels_last)


def front_norm(x, lengths, norm, silu=False):
    """Channel RMSNorm of a [B, C, T, F] activation at every (t, f), zero where
    t >= lengths, then SiLU if asked (reference ``buffers.py:58-79``). Returns a
    [B, C, T, F] view of channels-last memory, like the reference."""
    x = _nhwc(x)
    dev = _lib.require_cuda("front_norm", x, lengths, norm.weight)
    b, c, t, f = x.shape
    w = norm.weight.detach().float().contiguous()
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty_like(x)  # channels-last too
    _lib.launch("tf_front_norm_fwd", dev, x.data_ptr(), _lib.dtype_code(x, "front_norm"), w.data_ptr(),
                lengths.data_ptr(), y.data_ptr(), b, t, f, c, float(norm.eps), int(bool(silu)))
    return y


def front_stem(x, lengths, conv1, skip, norm):
    """First CNN stage's conv3x3 (1 -> 32, stride (1, 2)) + masked channel norm + SiLU
    and its 1x1 skip, from the [B, 1, T, F] spectrogram in one pass (reference
    ``front.py:21,33,43``; BF16 autocast semantics). Returns (h, skip) as
    [B, 32, T, F2] views of channels-last BF16 memory."""
    dev = _lib.require_cuda("front_stem", x, lengths, conv1.weight)
    b, c, t, f = x.shape
    if c != 1 or tuple(conv1.weight.shape) != (32, 1, 3, 3) or tuple(skip.weight.shape) != (32, 1, 1, 1):
        raise ValueError("front_stem: expected the 1 -> 32 channel first stage")
    xs = x.float().reshape(b, t, f).contiguous()
    f2 = (f - 1) // 2 + 1
    w1 = conv1.weight.detach().float().reshape(32, 9).contiguous()
    ws = skip.weight.detach().float().reshape(32).contiguous()
    nw = norm.weight.detach().float().contiguous()
    lengths = lengths.to(torch.int64).contiguous()
    h = torch.empty((b, t, f2, 32), device=dev, dtype=torch.bfloat16)
    s = torch.empty_like(h)
    _lib.launch("tf_front_stem_fwd", dev, xs.data_ptr(), w1.data_ptr(), ws.data_ptr(), nw.data_ptr(),
                lengths.data_ptr(), h.data_ptr(), s.data_ptr(), b, t, f, float(norm.eps))
    return h.permute(0, 3, 1, 2), s.permute(0, 3, 1, 2)


def front_residual(h, skip, lengths):
    """Residual tail of a front-end stage: ``silu(h + skip)`` zero past the
    lengths (reference ``front.py:43``), channels-last in and out."""
    h, skip = _nhwc(h), _nhwc(skip.to(h.dtype))
    dev = _lib.require_cuda("front_residual", h, skip, lengths)
    if h.shape != skip.shape:
        raise ValueError("front_residual: h and skip must have the same shape")
    b, c, t, f = h.shape
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty_like(h)
    _lib.launch("tf_front_residual_fwd", dev, h.data_ptr(), skip.data_ptr(),
                _lib.dtype_code(h, "front_residual"), lengths.data_ptr(), y.data_ptr(), b, t, f, c)
    return y


def depthwise_masked(x, layer, lengths, residual=False):
    """Depthwise Conv1d (``layer``: groups = channels, odd kernel, 'same'
    padding) over the time axis of [B, T, C] rows, with bias, zero past the
    lengths; BF16 result (reference ``buffers.py:13-32``). ``residual``: the
    input is added (``bf16(x + conv)``, model.py:188-189)."""
    x = x.contiguous()
    dev = _lib.require_cuda("depthwise_masked", x, lengths, layer.weight)
    b, t, c = x.shape
    k = layer.weight.shape[-1]
    if layer.groups != c or layer.weight.shape[0] != c or 2 * layer.padding[0] + 1 != k:
        raise ValueError("depthwise_masked: expected a depthwise Conv1d with 'same' padding")
    w = _param_bf16(layer.weight, (c, k))
    bias = None if layer.bias is None else _param_bf16(layer.bias, (c,))
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty((b, t, c), device=dev, dtype=torch.bfloat16)
    _lib.launch("tf_depthwise_residual_fwd" if residual else "tf_depthwise_masked_fwd", dev, x.data_ptr(),
                _lib.dtype_code(x, "depthwise_masked"),
                w.data_ptr(), None if bias is None else bias.data_ptr(), lengths.data_ptr(), y.data_ptr(),
                b, t, c, k)
    return y


def glu_depthwise(u, layer, lengths):
    """``depthwise_masked(F.glu(u, -1), layer, lengths)`` in one pass over the BF16
    ``[B, T, 2C]`` up-projection rows ``u`` (reference ``model.py:122-124``): the GLU is
    formed per tap as PyTorch's glu rounds it, never written. BF16 ``[B, T, C]``."""
    u = u.contiguous()
    dev = _lib.require_cuda("glu_depthwise", u, lengths, layer.weight)
    b, t, c2 = u.shape
    c = c2 // 2
    k = layer.weight.shape[-1]
    if u.dtype != torch.bfloat16 or c2 % 2:
        raise ValueError("glu_depthwise: u must be BF16 [B, T, 2C]")
    if layer.groups != c or layer.weight.shape[0] != c or 2 * layer.padding[0] + 1 != k:
        raise ValueError("glu_depthwise: expected a depthwise Conv1d with 'same' padding over C channels")
    w = _param_bf16(layer.weight, (c, k))
    bias = None if layer.bias is None else _param_bf16(layer.bias, (c,))
    lengths = lengths.to(torch.int64).contiguous()
    y = torch.empty((b, t, c), device=dev, dtype=torch.bfloat16)
    _lib.launch("tf_glu_depthwise_fwd", dev, u.data_ptr(), w.data_ptr(), None if bias is None else bias.data_ptr(),
                lengths.data_ptr(), y.data_ptr(), b, t, c, k)
    return y


class RotaryQKV:
    """Rotary q/k of the attention branch (reference ``buffers.py:46-55``):
    x [B, T, 3*H*D] (the qkv projection) -> [3, B, H, T, D], q and k rotated by
    the (cos, sin) table of the pooled grid, v unchanged. The kernel writes FP32
    holding BF16-rounded values — the attention's own operand type; ``out_dtype``
    BF16 gives the reference's return type."""

    @staticmethod
    def apply(x, cos, sin, heads, out_dtype=torch.bfloat16):
        x = x.to(torch.bfloat16).contiguous()
        dev = _lib.require_cuda("RotaryQKV", x, cos, sin)
        b, t, width = x.shape
        d = width // (3 * heads)
        if 3 * heads * d != width or cos.shape[0] < t or cos.shape[-1] != d // 2:
            raise ValueError("RotaryQKV: x must be [B, T, 3*heads*D] and the table [>=T, D/2]")
        cos, sin = cos.float().contiguous(), sin.float().contiguous()
        y = torch.empty((3, b, heads, t, d), device=dev, dtype=torch.float32)
        _lib.launch("tf_rotary_qkv_fwd", dev, x.data_ptr(), cos.data_ptr(), sin.data_ptr(), y.data_ptr(),
                    b, t, heads, d)
        return y if out_dtype == torch.float32 else y.to(out_dtype)
