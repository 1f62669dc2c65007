"""Valid-row ("ragged") layouts for batches of clips of different lengths.

A batch is padded to its longest clip (reference ``audio.py:52-66``); the rows
of a clip at or past its length carry nothing the recurrence reads, and its
output there is zero. Between host and device only the valid rows need to move.
The packed layout (``tf_ragged_copy_fwd`` in include/trifusion_b200.h) holds,
tensor after tensor, for each clip b and group g the valid steps of (b, g)
back to back, each tensor's region starting at a 16-byte-aligned offset.

Two kinds of tensors occur on the recurrence path:

* ``"time_major"`` — ``[B, T, ...]`` (q, k, v, z, angles, the output): one group
  per clip, a step is one row of ``prod(shape[2:])`` elements;
* ``"time_minor"`` — ``[B, G, T]`` (adt, dt, trap): ``G`` groups per clip, a step
  is one element.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

KINDS = ("time_major", "time_minor")


@dataclass(frozen=True)
class RaggedSpec:
    """Layout of one dense tensor: ``[batch][groups][steps][step_bytes]``."""

    groups: int
    steps: int
    step_bytes: int

    @staticmethod
    def of(x: torch.Tensor, kind: str) -> "RaggedSpec":
        if kind not in KINDS:
            raise ValueError(f"kind must be one of {KINDS}")
        if x.dim() < (2 if kind == "time_major" else 3):
            raise ValueError("tensor has too few dimensions for its kind")
        es = x.element_size()
        if kind == "time_major":
            return RaggedSpec(1, x.shape[1], es * (x[0, 0].numel() if x.shape[1] else 0))
        if x.dim() != 3:
            raise ValueError("a time_minor tensor is [B, G, T]")
        return RaggedSpec(x.shape[1], x.shape[2], es)


def region_bytes(spec: RaggedSpec, lengths) -> int:
    """Bytes of one tensor's packed region (rounded up to 16)."""
    rows = sum(min(max(int(n), 0), spec.steps) for n in lengths)
    return (rows * spec.groups * spec.step_bytes + 15) // 16 * 16


def packed_bytes(specs, lengths) -> int:
    return sum(region_bytes(s, lengths) for s in specs)


def pack_host(tensors, kinds, lengths, out: torch.Tensor) -> int:
    """Write the valid steps of host ``tensors`` into the uint8 host buffer ``out``
    in the packed layout; returns the bytes written (the CPU counterpart of
    ``ragged_copy(..., to_dense=False)``)."""
    off = 0
    lens = [int(n) for n in lengths]
    for x, kind in zip(tensors, kinds):
        spec = RaggedSpec.of(x, kind)
        flat = x.contiguous().view(torch.uint8).reshape(x.shape[0], spec.groups, spec.steps * spec.step_bytes)
        pos = off
        for b, n in enumerate(lens):
            n = min(max(n, 0), spec.steps) * spec.step_bytes
            for g in range(spec.groups):
                out[pos:pos + n] = flat[b, g, :n]
                pos += n
        off += region_bytes(spec, lens)
    return off


def unpack_host(packed: torch.Tensor, like, kinds, lengths):
    """Dense host tensors (shapes and dtypes of ``like``) from a packed buffer; rows
    past each clip's length are zero."""
    outs = []
    off = 0
    lens = [int(n) for n in lengths]
    for x, kind in zip(like, kinds):
        spec = RaggedSpec.of(x, kind)
        y = torch.zeros_like(x, device="cpu").contiguous()
        flat = y.view(torch.uint8).reshape(x.shape[0], spec.groups, spec.steps * spec.step_bytes)
        pos = off
        for b, n in enumerate(lens):
            n = min(max(n, 0), spec.steps) * spec.step_bytes
            for g in range(spec.groups):
                flat[b, g, :n] = packed[pos:pos + n]
                pos += n
        off += region_bytes(spec, lens)
        outs.append(y)
    return outs


class RaggedCopier:
    """``ragged_copy`` bound to fixed dense tensors: the argument arrays of
    ``tf_ragged_copy_fwd`` are built once, so a per-step call costs one C call."""

    def __init__(self, dense, kinds):
        if not dense:
            raise ValueError("RaggedCopier needs at least one tensor")
        dev = dense[0].device
        if dev.type != "cuda" or any(x.device != dev or not x.is_contiguous() for x in dense):
            raise ValueError("RaggedCopier: contiguous tensors on one CUDA device")
        self.batch = dense[0].shape[0]
        if any(x.shape[0] != self.batch for x in dense):
            raise ValueError("RaggedCopier: every tensor shares the batch size")
        specs = [RaggedSpec.of(x, k) for x, k in zip(dense, kinds)]
        n = len(dense)
        self.device = dev
        self._keep = list(dense)
        self._args = ((ctypes.c_void_p * n)(*[x.data_ptr() for x in dense]),
                      (ctypes.c_int64 * n)(*[sp.groups for sp in specs]),
                      (ctypes.c_int64 * n)(*[sp.steps for sp in specs]),
                      (ctypes.c_int64 * n)(*[sp.step_bytes for sp in specs]), n)

    def __call__(self, packed: torch.Tensor, lengths: torch.Tensor, to_dense: bool) -> None:
        """Copy on the current stream; ``lengths`` int64 [B] on the tensors' device."""
        if packed.device != self.device or lengths.device != self.device or lengths.numel() != self.batch:
            raise ValueError("RaggedCopier: packed and lengths on the tensors' device, one length per clip")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib().tf_ragged_copy_fwd(packed.data_ptr(), *self._args, lengths.data_ptr(),
                                                     self.batch, 1 if to_dense else 0, stream))


def ragged_copy(packed: torch.Tensor, dense, kinds, lengths: torch.Tensor, to_dense: bool) -> None:
    """Device copy between ``packed`` (uint8) and the contiguous ``dense`` tensors, on
    the current stream (``tf_ragged_copy_fwd``). ``lengths``: int64 [B] on the device."""
    if not dense:
        return
    if packed.dtype != torch.uint8 or lengths.dtype != torch.int64 or not lengths.is_contiguous():
        raise ValueError("ragged_copy: packed is uint8 and lengths int64 contiguous")
    RaggedCopier(dense, kinds)(packed, lengths, to_dense)
