"""Host-buffer pipeline: steps fed from pinned host memory with the copies of
one step overlapping the kernels of its neighbours.

The reference's entry points take CUDA tensors (``docs/api.md:61-74``); a caller
holding its inputs in host memory copies them in, launches, and copies the result
back. Done on one stream, the kernel waits for the copies and the copy engines
wait for the kernel. ``HostPipeline`` keeps ``depth`` device buffer sets and
three streams: copy-in, compute and copy-out. Step i copies into set ``i % depth``
while step i-1 computes and step i-2's result goes back, which leaves the
larger of the copy-in time, the copy-out time and the kernel time per step.
(Host-to-device and device-to-host copies use separate copy engines.)

Ordering, per buffer set j:

* copy-in waits until the previous compute on set j has read its inputs;
* compute waits for its copy-in and for the previous copy-out of set j's output;
* copy-out waits for the compute.

The caller may rewrite a step's host inputs once ``inputs_consumed(handle)`` has
fired, and read its host output once ``done(handle)`` has fired (or after
``synchronize()``).

With ``packed=True`` every buffer set keeps all inputs in one device block (each
input at a 256-byte-aligned offset), and ``host_block()`` returns a pinned host
block of the same layout with views to fill; ``submit(block, host_out)`` then moves
a step's inputs with a single copy instead of one per tensor (many small copies
each pay a fixed cost on the host link).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class StepHandle:
    """Events of one submitted step."""

    consumed: torch.cuda.Event  # the host inputs have been copied
    finished: torch.cuda.Event  # the host output holds the result


class HostPipeline:
    """Runs ``fn`` over steps whose inputs and outputs live in pinned host memory.

    ``fn(*device_inputs)`` returns the step's device result. With
    ``writes_out=True`` it is called as ``fn(*device_inputs, out=device_out)``
    and writes the set's own output buffer (no extra copy); otherwise its result
    is copied into that buffer on the compute stream, so a function that
    returns a reused static buffer (a CUDA-graph engine) stays correct.
    """

    def __init__(self, fn, example_inputs, out_shape, out_dtype, device=None, depth=2, writes_out=False,
                 packed=False):
        if depth < 1:
            raise ValueError("depth must be at least 1")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        if device.type != "cuda":
            raise ValueError("HostPipeline runs on a CUDA device")
        self.fn = fn
        self.device = device
        self.depth = depth
        self.writes_out = writes_out
        self.packed = packed
        self._layout = []  # (offset, nbytes, dtype, shape) per input
        offset = 0
        for x in example_inputs:
            nbytes = x.numel() * x.element_size()
            self._layout.append((offset, nbytes, x.dtype, tuple(x.shape)))
            offset += (nbytes + 255) // 256 * 256
        self.block_bytes = offset
        self.sets = []
        for _ in range(depth):
            if packed:
                block = torch.empty(self.block_bytes, dtype=torch.uint8, device=device)
                inputs = self._views(block)
            else:
                block = None
                inputs = [torch.empty(x.shape, dtype=x.dtype, device=device) for x in example_inputs]
            out = torch.empty(tuple(out_shape), dtype=out_dtype, device=device)
            self.sets.append((inputs, out, block))
        self.copy_in = torch.cuda.Stream(device)
        self.compute = torch.cuda.Stream(device)
        self.copy_out = torch.cuda.Stream(device)
        current = torch.cuda.current_stream(device)
        self._read = [torch.cuda.Event() for _ in range(depth)]      # compute has read set j's inputs
        self._returned = [torch.cuda.Event() for _ in range(depth)]  # set j's output is back on the host
        for j in range(depth):
            self._read[j].record(current)
            self._returned[j].record(current)
        self._n = 0

    def _views(self, block):
        return [block[o:o + n].view(dt).view(shape) for o, n, dt, shape in self._layout]

    def host_block(self):
        """A pinned host block in the packed layout and its per-input views (to fill)."""
        if not self.packed:
            raise ValueError("host_block() needs packed=True")
        block = torch.empty(self.block_bytes, dtype=torch.uint8).pin_memory()
        return block, self._views(block)

    def submit(self, host_inputs, host_out) -> StepHandle:
        """Queue one step: copy ``host_inputs`` in (a list of tensors, or with
        ``packed=True`` the block from ``host_block()``), run, copy the result to
        ``host_out``."""
        j = self._n % self.depth
        self._n += 1
        inputs, out, block = self.sets[j]
        single = isinstance(host_inputs, torch.Tensor)
        if single and (not self.packed or host_inputs.numel() != self.block_bytes
                       or host_inputs.dtype != torch.uint8):
            raise ValueError("a single host tensor must be the packed block from host_block()")
        if not single and len(host_inputs) != len(inputs):
            raise ValueError(f"expected {len(inputs)} inputs, got {len(host_inputs)}")
        arrived = torch.cuda.Event()
        consumed = torch.cuda.Event()
        finished = torch.cuda.Event()
        with torch.cuda.stream(self.copy_in):
            self.copy_in.wait_event(self._read[j])
            if single:
                block.copy_(host_inputs, non_blocking=True)
            else:
                for src, dst in zip(host_inputs, inputs):
                    dst.copy_(src, non_blocking=True)
            arrived.record(self.copy_in)
            consumed.record(self.copy_in)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(arrived)
            self.compute.wait_event(self._returned[j])
            if self.writes_out:
                self.fn(*inputs, out=out)
            else:
                out.copy_(self.fn(*inputs))
            self._read[j].record(self.compute)
        with torch.cuda.stream(self.copy_out):
            self.copy_out.wait_event(self._read[j])
            host_out.copy_(out, non_blocking=True)
            self._returned[j].record(self.copy_out)
            finished.record(self.copy_out)
        return StepHandle(consumed, finished)

    @staticmethod
    def inputs_consumed(handle: StepHandle) -> bool:
        return handle.consumed.query()

    @staticmethod
    def done(handle: StepHandle) -> bool:
        return handle.finished.query()

    def synchronize(self) -> None:
        for s in (self.copy_in, self.compute, self.copy_out):
            s.synchronize()
