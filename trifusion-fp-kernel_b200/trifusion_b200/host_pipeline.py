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


class RaggedHostPipeline:
    """``HostPipeline`` for batches of clips of different lengths whose inputs and
    output cross the host link as valid rows only (``trifusion_b200.ragged``).

    ``example_inputs`` are dense host tensors in ``fn``'s argument order and
    ``kinds`` their layout kinds (``"time_major"``, ``"time_minor"``, or ``None``
    for a tensor copied whole, e.g. per-head parameters). A step's host block
    (``host_block()``) holds the clip lengths (int64, padded to 256 bytes), the
    whole tensors, then the valid rows of the others; ``pack(block, inputs,
    lengths)`` fills it and returns its used size. On the device every buffer set
    keeps dense tensors; each step copies the used bytes in, scatters the rows
    (``tf_ragged_copy_fwd``), calls ``fn(*dense_inputs, lengths, out=dense_out)``,
    gathers the output's valid rows (``out_kind``) and copies only those back.
    Rows at or past a clip's length keep whatever an earlier step left there on
    the device, so ``fn`` must not read them (the recurrence with ``lengths``
    does not); the output there is not transferred (zero by the length mask).
    Streams and ordering are those of ``HostPipeline``. With ``graphs=True`` each
    buffer set's device work (scatter, ``fn``, gather) is captured in a CUDA graph
    after its first step and replayed afterwards (``fn`` must then be capturable and
    read its arguments only on the device).
    """

    def __init__(self, fn, example_inputs, kinds, out_shape, out_dtype, out_kind="time_major", device=None,
                 depth=2, graphs=False):
        from . import ragged

        self.graphs = graphs
        self._graph = [None] * depth
        if depth < 1 or len(kinds) != len(example_inputs):
            raise ValueError("depth >= 1 and one kind per input")
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.fn, self.device, self.depth = fn, device, depth
        self.kinds = list(kinds)
        self.out_kind = out_kind
        self.batch = example_inputs[0].shape[0]
        self._whole = [i for i, k in enumerate(kinds) if k is None]
        self._rows = [i for i, k in enumerate(kinds) if k is not None]
        self._header = (self.batch * 8 + 255) // 256 * 256
        off = self._header
        self._whole_layout = []
        for i in self._whole:
            n = example_inputs[i].numel() * example_inputs[i].element_size()
            self._whole_layout.append((i, off, n))
            off += (n + 255) // 256 * 256
        self._rows_offset = off
        full = [example_inputs[i].shape[1] if kinds[i] == "time_major" else example_inputs[i].shape[-1]
                for i in self._rows]
        self.capacity = off + ragged.packed_bytes(
            [ragged.RaggedSpec.of(example_inputs[i], kinds[i]) for i in self._rows], [max(full, default=0)] * self.batch)
        out_like = torch.empty(tuple(out_shape), dtype=out_dtype, device="meta")
        self.out_capacity = ragged.packed_bytes([ragged.RaggedSpec.of(out_like, out_kind)],
                                                [out_like.shape[1] if out_kind == "time_major" else out_like.shape[-1]]
                                                * self.batch)
        self.sets = []
        for _ in range(depth):
            block = torch.empty(self.capacity, dtype=torch.uint8, device=device)
            dense = [torch.empty(x.shape, dtype=x.dtype, device=device) for x in example_inputs]
            for i, o, n in self._whole_layout:
                dense[i] = block[o:o + n].view(example_inputs[i].dtype).view(example_inputs[i].shape)
            lengths = block[:self.batch * 8].view(torch.int64)
            out = torch.empty(tuple(out_shape), dtype=out_dtype, device=device)
            out_packed = torch.empty(self.out_capacity, dtype=torch.uint8, device=device)
            copiers = (ragged.RaggedCopier([dense[i] for i in self._rows], [kinds[i] for i in self._rows]),
                       ragged.RaggedCopier([out], [out_kind]))
            self.sets.append((block, dense, lengths, out, out_packed, copiers))
        self.copy_in = torch.cuda.Stream(device)
        self.compute = torch.cuda.Stream(device)
        self.copy_out = torch.cuda.Stream(device)
        current = torch.cuda.current_stream(device)
        self._read = [torch.cuda.Event() for _ in range(depth)]
        self._returned = [torch.cuda.Event() for _ in range(depth)]
        for j in range(depth):
            self._read[j].record(current)
            self._returned[j].record(current)
        self._n = 0
        self._out_like = out_like
        self._rows_view = [st[0][self._rows_offset:] for st in self.sets]

    def host_block(self):
        """A pinned host block able to hold any step's packed inputs."""
        return torch.empty(self.capacity, dtype=torch.uint8).pin_memory()

    def host_out(self):
        """A pinned host buffer able to hold any step's packed output rows."""
        return torch.empty(self.out_capacity, dtype=torch.uint8).pin_memory()

    def pack(self, block, host_inputs, lengths) -> int:
        """Fill ``block`` with one step's lengths, whole tensors and valid rows; returns
        the bytes a step moves in."""
        from . import ragged

        lengths = torch.as_tensor(lengths, dtype=torch.int64)
        if lengths.numel() != self.batch:
            raise ValueError("one length per clip")
        block[:self.batch * 8] = lengths.contiguous().view(torch.uint8)
        for i, o, n in self._whole_layout:
            block[o:o + n] = host_inputs[i].contiguous().view(torch.uint8).reshape(-1)
        used = ragged.pack_host([host_inputs[i] for i in self._rows], [self.kinds[i] for i in self._rows],
                                lengths.tolist(), block[self._rows_offset:])
        return self._rows_offset + used

    def out_bytes(self, lengths) -> int:
        """Bytes of a step's packed output rows."""
        from . import ragged

        return ragged.packed_bytes([ragged.RaggedSpec.of(self._out_like, self.out_kind)], [int(n) for n in lengths])

    def unpack_out(self, host_out, lengths):
        """The dense output of a step (zero past each clip's length) from its packed rows."""
        from . import ragged

        like = torch.empty(self._out_like.shape, dtype=self._out_like.dtype)
        return ragged.unpack_host(host_out, [like], [self.out_kind], lengths)[0]

    def submit(self, block, in_bytes, host_out, out_bytes) -> StepHandle:
        """Queue one step: the first ``in_bytes`` of ``block`` in, run, the first
        ``out_bytes`` of the packed output back to ``host_out``."""
        if not (0 < in_bytes <= self.capacity and 0 <= out_bytes <= self.out_capacity):
            raise ValueError("step sizes out of range")
        j = self._n % self.depth
        self._n += 1
        dev_block, dense, lengths, out, out_packed, (unpack_rows, pack_out) = self.sets[j]
        arrived, consumed, finished = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
        with torch.cuda.stream(self.copy_in):
            self.copy_in.wait_event(self._read[j])
            dev_block[:in_bytes].copy_(block[:in_bytes], non_blocking=True)
            arrived.record(self.copy_in)
            consumed.record(self.copy_in)
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(arrived)
            self.compute.wait_event(self._returned[j])
            def work():
                unpack_rows(self._rows_view[j], lengths, to_dense=True)
                self.fn(*dense, lengths, out=out)
                pack_out(out_packed, lengths, to_dense=False)

            if self._graph[j] is not None:
                self._graph[j].replay()
            else:
                work()
                if self.graphs:  # captured after its first eager run (which did this step's work)
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(graph, stream=self.compute):
                        work()
                    self._graph[j] = graph
            self._read[j].record(self.compute)
        with torch.cuda.stream(self.copy_out):
            self.copy_out.wait_event(self._read[j])
            host_out[:out_bytes].copy_(out_packed[:out_bytes], non_blocking=True)
            self._returned[j].record(self.copy_out)
            finished.record(self.copy_out)
        return StepHandle(consumed, finished)

    def synchronize(self) -> None:
        for s in (self.copy_in, self.compute, self.copy_out):
            s.synchronize()
