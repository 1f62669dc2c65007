"""Fused Mamba-3 SISO recurrence on B200 — drop-in for
``trifusion_l4.mamba_fused.fused_mamba`` (reference ``mamba_fused.py:155-191``).

The tensor contract is the reference's (``docs/api.md:61-74``); the work runs
in the CUDA kernels of ``libtrifusion_b200.so`` on the current stream, with no
host synchronisation, so calls can be captured in CUDA graphs.
"""

from __future__ import annotations

import torch

from . import _lib

_BF16_ARGS = ("q", "k", "v", "angles", "z")


def _prep(q, k, v, adt, dt, trap, qb, kb, angles, d, z):
    b, t, h, p = v.shape
    n = q.shape[-1]
    r = angles.shape[-1]
    if n != 128 or p != 64 or r != 32:  # mamba_fused.py:159-160
        raise ValueError(_lib.SHAPE_MESSAGE)
    # The kernel's operands are BF16 (docs/api.md:61-69); FP32/FP16 inputs are
    # rounded to BF16 once, here.
    for x in (q, k, v, angles, z):
        if not x.is_floating_point():
            raise TypeError(f"fused_mamba: expected bfloat16 tensors, got {x.dtype}")
    q, k, v, angles, z = (x if x.dtype == torch.bfloat16 else x.to(torch.bfloat16)
                          for x in (q, k, v, angles, z))
    if q.shape != k.shape or q.shape[:2] != (b, t) or q.dim() != 4:
        raise ValueError("fused_mamba: q and k must be [B,T,Hq,128] matching v")
    if z.shape != v.shape or angles.shape[:3] != (b, t, h):
        raise ValueError("fused_mamba: z must match v and angles must be [B,T,H,32]")
    hq = q.shape[2]
    if hq < 1 or h % hq:
        raise ValueError("fused_mamba: H must be divisible by Hq")
    for name, x in dict(adt=adt, dt=dt, trap=trap).items():
        if tuple(x.shape) != (b, h, t):
            raise ValueError(f"fused_mamba: {name} must be [B,H,T]")
    if trap.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("fused_mamba: trap must be float32 or bfloat16")
    dev = v.device
    tensors = (q, k, v, adt, dt, trap, qb, kb, angles, d, z)
    if dev.type != "cuda" or any(x.device != dev for x in tensors):
        raise RuntimeError("fused_mamba: all tensors must be CUDA tensors on one device")
    # Kernel requirement: unit stride in the innermost dimension of BF16 rows.
    q, k, v, z = (x if x.stride(-1) == 1 else x.contiguous() for x in (q, k, v, z))
    adt, dt = (x if x.dtype == torch.float32 else x.float() for x in (adt, dt))
    qb, kb, d = (x.float().contiguous() for x in (qb, kb, d))
    if qb.shape != (h, 128) or kb.shape != (h, 128) or d.numel() != h:
        raise ValueError("fused_mamba: qb, kb must be [H,128] and d must be [H]")
    return (q, k, v, adt, dt, trap, qb, kb, angles, d, z), (b, t, h, hq)


def _strides(q, k, v, adt, dt, trap, angles, z, out):
    s = []
    for x in (q, k, v, adt, dt, trap, angles, z, out):
        s.extend(x.stride())
    return _lib.int64_array(s)


def fused_mamba(q, k, v, adt, dt, trap, qb, kb, angles, d, z, warps=8):
    """Fused recurrence; returns a fresh contiguous ``[B,T,H,64]`` BF16 tensor.

    ``warps`` is accepted for signature compatibility; the CUDA kernel fixes
    its own launch shape.
    """
    del warps
    (q, k, v, adt, dt, trap, qb, kb, angles, d, z), (b, t, h, hq) = _prep(
        q, k, v, adt, dt, trap, qb, kb, angles, d, z)
    _lib.check_device_error()
    out = torch.empty_like(v, memory_format=torch.contiguous_format)
    stream = torch.cuda.current_stream(v.device).cuda_stream
    with torch.cuda.device(v.device):
        lib = _lib.lib()
        nws = lib.tf_recurrence_workspace_size(b, t, h)
        ws = _lib.workspace(v.device, nws)
        _lib.check(lib.tf_fused_mamba_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), adt.data_ptr(), dt.data_ptr(),
            trap.data_ptr(), _lib.TF_BF16 if trap.dtype == torch.bfloat16 else _lib.TF_F32,
            qb.data_ptr(), kb.data_ptr(), angles.data_ptr(), d.data_ptr(), z.data_ptr(),
            out.data_ptr(), _strides(q, k, v, adt, dt, trap, angles, z, out),
            b, t, h, hq, ws.data_ptr(), ws.numel(), stream))
    return out


def fused_recurrence(q, k, v, adt, dt, trap, qb, kb, angles, d, z, *, q_norm=None,
                     k_norm=None, lengths=None, eps=1e-5, out=None):
    """The recurrence with the work around it fused into the same launch.

    ``q_norm``/``k_norm`` ([128] FP32 weights) apply the C/B RMSNorm of the raw
    q/k rows (reference ``mamba.py:56-57``); ``lengths`` ([B] int64, on the
    device) zeroes output rows ``t >= lengths[b]`` (the length mask of
    ``model.py:174``) and stops the scan there. ``out`` may be given to write
    into a preallocated contiguous buffer.
    """
    (q, k, v, adt, dt, trap, qb, kb, angles, d, z), (b, t, h, hq) = _prep(
        q, k, v, adt, dt, trap, qb, kb, angles, d, z)
    _lib.check_device_error()
    if out is None:
        out = torch.empty_like(v, memory_format=torch.contiguous_format)
    qw = None if q_norm is None else q_norm.float().contiguous()
    kw = None if k_norm is None else k_norm.float().contiguous()
    for w in (qw, kw):
        if w is not None and (w.numel() != 128 or w.device != v.device):
            raise ValueError("fused_recurrence: norm weights must be [128] on the same device")
    if lengths is not None:
        if lengths.dtype != torch.int64 or lengths.numel() != b or lengths.device != v.device:
            raise ValueError("fused_recurrence: lengths must be int64 [B] on the same device")
        lengths = lengths.contiguous()
    stream = torch.cuda.current_stream(v.device).cuda_stream
    with torch.cuda.device(v.device):
        lib = _lib.lib()
        nws = lib.tf_recurrence_workspace_size(b, t, h)
        ws = _lib.workspace(v.device, nws)
        _lib.check(lib.tf_mamba_recurrence_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), adt.data_ptr(), dt.data_ptr(),
            trap.data_ptr(), _lib.TF_BF16 if trap.dtype == torch.bfloat16 else _lib.TF_F32,
            qb.data_ptr(), kb.data_ptr(), angles.data_ptr(), d.data_ptr(), z.data_ptr(),
            out.data_ptr(), _strides(q, k, v, adt, dt, trap, angles, z, out),
            b, t, h, hq, None if qw is None else qw.data_ptr(),
            None if kw is None else kw.data_ptr(), float(eps),
            None if lengths is None else lengths.data_ptr(), ws.data_ptr(), ws.numel(), stream))
    return out


_STAND_INS = {}


def _stand_in(device):
    """A cached one-element FP32 tensor per device (never read or written by the launch)."""
    t = _STAND_INS.get(device)
    if t is None:
        t = _STAND_INS[device] = torch.zeros(1, device=device)
    return t


def fused_recurrence_multi(directions, *, lengths=None, eps=1e-5):
    """One launch for one or two recurrences over the same ``[B, T, H]`` shape —
    the two directions of a bidirectional block — returning their outputs.

    Each direction is a dict with the ``fused_mamba`` tensors (``q k v adt dt
    trap qb kb angles d z``) and optionally:

    * ``a_raw``, ``ddt_raw`` ([B,T,H] projection views), ``dt_bias`` ([H]) and
      ``a_floor`` instead of ``adt``/``dt``: the controls of ``mamba.py:58-63``
      computed inside the launch;
    * ``q_norm``/``k_norm`` (the C/B RMSNorm weights);
    * ``reverse=True``: every row's valid prefix is read and written in reverse
      time order (the backward direction of ``model.py:175-179`` without the
      ``reverse_valid`` copies); rows at or past ``lengths`` come out zero;
    * ``out``: a preallocated contiguous output.
    """
    if not 1 <= len(directions) <= 2:
        raise ValueError("fused_recurrence_multi: one or two directions")
    _lib.check_device_error()
    ios = (_lib.RecurrenceIO * len(directions))()
    keep, outs, shape = [], [], None
    for i, d_ in enumerate(directions):
        raw = d_.get("a_raw") is not None
        adt = d_.get("adt")
        dt = d_.get("dt")
        if raw:  # adt/dt are computed in the launch: pass a one-element stand-in
            b_, t_, h_ = d_["a_raw"].shape
            adt = dt = _stand_in(d_["v"].device).expand(b_, h_, t_)
        (q, k, v, adt_, dt_, trap, qb, kb, angles, d, z), dims = _prep(
            d_["q"], d_["k"], d_["v"], adt, dt, d_["trap"], d_["qb"], d_["kb"], d_["angles"], d_["d"],
            d_["z"])
        if shape is None:
            shape = dims
        elif dims != shape:
            raise ValueError("fused_recurrence_multi: both directions need the same [B,T,H] and groups")
        b, t, h, hq = dims
        out = d_.get("out")
        if out is None:
            out = torch.empty_like(v, memory_format=torch.contiguous_format)
        elif (tuple(out.shape) != tuple(v.shape) or out.dtype != torch.bfloat16 or out.device != v.device
              or out.stride(-1) != 1):
            raise ValueError("fused_recurrence_multi: out must be BF16 [B,T,H,64] on v's device with a "
                             "contiguous last dimension")
        io = ios[i]
        io.q, io.k, io.v, io.z, io.angles = (x.data_ptr() for x in (q, k, v, z, angles))
        io.qb, io.kb, io.d = qb.data_ptr(), kb.data_ptr(), d.data_ptr()
        io.trap = trap.data_ptr()
        io.trap_dtype = _lib.TF_BF16 if trap.dtype == torch.bfloat16 else _lib.TF_F32
        st = list(_strides(q, k, v, adt_, dt_, trap, angles, z, out))
        if raw:
            a_raw, ddt_raw = d_["a_raw"], d_["ddt_raw"]
            if a_raw.dtype != torch.bfloat16 or ddt_raw.dtype != torch.bfloat16:
                a_raw, ddt_raw = a_raw.to(torch.bfloat16), ddt_raw.to(torch.bfloat16)
            if tuple(a_raw.shape) != (b, t, h) or tuple(ddt_raw.shape) != (b, t, h):
                raise ValueError("fused_recurrence_multi: a_raw/ddt_raw must be [B,T,H]")
            bias = d_["dt_bias"].detach().float().contiguous()
            io.a_raw, io.ddt_raw, io.dt_bias = a_raw.data_ptr(), ddt_raw.data_ptr(), bias.data_ptr()
            io.a_floor = float(d_.get("a_floor", 1e-4))
            st += [*a_raw.stride(), *ddt_raw.stride()]
            keep += [a_raw, ddt_raw, bias]
        else:
            io.adt, io.dt = adt_.data_ptr(), dt_.data_ptr()
            st += [0] * 6
        for j, val in enumerate(st):
            io.strides[j] = val
        for name, field in (("q_norm", "q_norm_w"), ("k_norm", "k_norm_w")):
            w = d_.get(name)
            if w is not None:
                w = w.detach().float().contiguous()
                if w.numel() != 128:
                    raise ValueError("fused_recurrence_multi: norm weights must be [128]")
                setattr(io, field, w.data_ptr())
                keep.append(w)
        io.out = out.data_ptr()
        io.reverse = 1 if d_.get("reverse") else 0
        keep += [q, k, v, adt_, dt_, trap, qb, kb, angles, d, z]
        outs.append(out)
    b, t, h, hq = shape
    dev = outs[0].device
    if lengths is not None:
        if lengths.dtype != torch.int64 or lengths.numel() != b or lengths.device != dev:
            raise ValueError("fused_recurrence_multi: lengths must be int64 [B] on the same device")
        lengths = lengths.contiguous()
    with torch.cuda.device(dev):
        lib = _lib.lib()
        n = len(directions)
        ws = _lib.workspace(dev, lib.tf_recurrence_workspace_size_multi(n, b, t, h))
        _lib.check(lib.tf_mamba_recurrence_multi_fwd(
            ios, n, b, t, h, hq, float(eps), None if lengths is None else lengths.data_ptr(),
            ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream))
    del keep
    return outs
