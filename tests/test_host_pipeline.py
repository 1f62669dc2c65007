"""HostPipeline: steps fed from pinned host memory, copies overlapping kernels.

GPU cases check that pipelined steps return exactly what direct calls return,
including a step function that reuses one static output buffer (a CUDA-graph
engine behaves like that) and inputs rewritten between steps.
"""

import pytest
import torch

from trifusion_b200.host_pipeline import HostPipeline


def test_rejects_a_cpu_device():
    with pytest.raises(ValueError):
        HostPipeline(lambda x: x, [torch.zeros(4)], (4,), torch.float32, device="cpu")


gpu = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA GPU")


@gpu
@needs_cuda
def test_recurrence_steps_equal_direct_calls():
    from trifusion_b200 import fused_recurrence
    from trifusion_b200.synthetic import lengths_uniform, norm_weight, recurrence_inputs

    b, t, h = 4, 150, 12
    qw, kw = norm_weight(128, 1).cuda(), norm_weight(128, 2).cuda()
    steps = []
    for s in range(5):
        args = [x.contiguous().pin_memory() for x in recurrence_inputs(b, t, h, kind="baseline", seed=s, device="cpu")]
        steps.append(args + [lengths_uniform(b, 20, t, seed=s).pin_memory()])

    def run(*xs, out):
        return fused_recurrence(*xs[:11], q_norm=qw, k_norm=kw, lengths=xs[11], out=out)

    pipe = HostPipeline(run, steps[0], (b, t, h, 64), torch.bfloat16, writes_out=True)
    outs = [torch.empty(b, t, h, 64, dtype=torch.bfloat16).pin_memory() for _ in steps]
    for x, o in zip(steps, outs):
        pipe.submit(x, o)
    pipe.synchronize()
    for x, o in zip(steps, outs):
        dev = [y.cuda() for y in x]
        ref = fused_recurrence(*dev[:11], q_norm=qw, k_norm=kw, lengths=dev[11])
        assert torch.equal(o, ref.cpu())


@gpu
@needs_cuda
def test_packed_block_equals_separate_copies():
    """packed=True: one host block per step, one copy; same results as the direct calls."""
    from trifusion_b200 import fused_recurrence
    from trifusion_b200.synthetic import lengths_uniform, norm_weight, recurrence_inputs

    b, t, h = 3, 130, 12
    qw, kw = norm_weight(128, 1).cuda(), norm_weight(128, 2).cuda()
    example = list(recurrence_inputs(b, t, h, kind="baseline", seed=0, device="cpu")) + [lengths_uniform(b, 5, t)]
    example = [x.contiguous() for x in example]

    def run(*xs, out):
        return fused_recurrence(*xs[:11], q_norm=qw, k_norm=kw, lengths=xs[11], out=out)

    pipe = HostPipeline(run, example, (b, t, h, 64), torch.bfloat16, writes_out=True, packed=True)
    blocks, outs, refs = [], [], []
    for s in range(4):
        xs = [x.contiguous() for x in recurrence_inputs(b, t, h, kind="baseline", seed=s, device="cpu")]
        xs.append(lengths_uniform(b, 5, t, seed=s))
        block, views = pipe.host_block()
        for v, x in zip(views, xs):
            v.copy_(x)
        dev = [x.cuda() for x in xs]
        refs.append(fused_recurrence(*dev[:11], q_norm=qw, k_norm=kw, lengths=dev[11]).cpu())
        blocks.append(block)
        outs.append(torch.empty(b, t, h, 64, dtype=torch.bfloat16).pin_memory())
    for block, o in zip(blocks, outs):
        pipe.submit(block, o)
    pipe.synchronize()
    for o, r in zip(outs, refs):
        assert torch.equal(o, r)
    with pytest.raises(ValueError):
        pipe.submit(torch.zeros(7, dtype=torch.uint8), outs[0])


@gpu
@needs_cuda
def test_static_output_buffer_and_reused_host_inputs():
    static = torch.empty(1 << 20, device="cuda")

    def engine(x):
        torch.mul(x, 3.0, out=static)  # every call overwrites the same buffer
        return static

    host_in = torch.empty(1 << 20).pin_memory()
    pipe = HostPipeline(engine, [host_in], (1 << 20,), torch.float32, depth=2)
    outs = []
    for i in range(6):
        handle_prev = None if not outs else outs[-1][1]
        if handle_prev is not None:
            handle_prev.consumed.synchronize()  # inputs copied: the host buffer may be rewritten
        host_in.fill_(float(i))
        o = torch.empty(1 << 20).pin_memory()
        outs.append((o, pipe.submit([host_in], o)))
    pipe.synchronize()
    for i, (o, h) in enumerate(outs):
        assert HostPipeline.done(h)
        assert torch.all(o == 3.0 * i)


@gpu
@needs_cuda
def test_wrong_input_count_raises():
    pipe = HostPipeline(lambda x: x, [torch.zeros(4)], (4,), torch.float32)
    with pytest.raises(ValueError):
        pipe.submit([torch.zeros(4), torch.zeros(4)], torch.zeros(4))


# ---- valid-row (ragged) transfers ------------------------------------------------

RECURRENCE_KINDS = ["time_major", "time_major", "time_major", "time_minor", "time_minor", "time_minor",
                    None, None, "time_major", None, "time_major"]  # q k v adt dt trap qb kb angles d z


def _ragged_example(b=5, t=70, h=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(b, t, 1, 128, generator=g).to(torch.bfloat16),   # time_major, 256-byte rows
            torch.randn(b, t, h, 64, generator=g).to(torch.bfloat16),    # time_major
            torch.randn(b, h, t, generator=g),                            # time_minor FP32
            torch.randn(b, t, 1, 3, generator=g).to(torch.bfloat16)]     # time_major, 6-byte rows


def test_ragged_pack_unpack_round_trip():
    from trifusion_b200 import ragged

    xs = _ragged_example()
    kinds = ["time_major", "time_major", "time_minor", "time_major"]
    lengths = [70, 0, 13, 71, 1]  # clamped to [0, T]
    specs = [ragged.RaggedSpec.of(x, k) for x, k in zip(xs, kinds)]
    assert specs[2] == ragged.RaggedSpec(3, 70, 4) and specs[0] == ragged.RaggedSpec(1, 70, 256)
    buf = torch.zeros(ragged.packed_bytes(specs, lengths), dtype=torch.uint8)
    used = ragged.pack_host(xs, kinds, lengths, buf)
    assert used == buf.numel()
    for s in specs:
        assert ragged.region_bytes(s, lengths) % 16 == 0
    back = ragged.unpack_host(buf, xs, kinds, lengths)
    for x, y, k in zip(xs, back, kinds):
        for bi, n in enumerate(lengths):
            n = min(n, 70)
            if k == "time_major":
                assert torch.equal(y[bi, :n], x[bi, :n]) and not y[bi, n:].any()
            else:
                assert torch.equal(y[bi, :, :n], x[bi, :, :n]) and not y[bi, :, n:].any()


@gpu
@needs_cuda
def test_ragged_device_copy_is_bit_exact_and_leaves_padding():
    from trifusion_b200 import ragged

    xs = _ragged_example()
    kinds = ["time_major", "time_major", "time_minor", "time_major"]
    lengths = [70, 0, 13, 71, 1]
    specs = [ragged.RaggedSpec.of(x, k) for x, k in zip(xs, kinds)]
    host = torch.zeros(ragged.packed_bytes(specs, lengths), dtype=torch.uint8)
    ragged.pack_host(xs, kinds, lengths, host)
    dense = [torch.full_like(x, 7.0, device="cuda") for x in xs]
    lens = torch.tensor(lengths, device="cuda")
    ragged.ragged_copy(host.cuda(), dense, kinds, lens, to_dense=True)
    for x, d, k in zip(xs, dense, kinds):
        d = d.cpu()
        for bi, n in enumerate(lengths):
            n = min(n, 70)
            valid, pad = (d[bi, :n], d[bi, n:]) if k == "time_major" else (d[bi, :, :n], d[bi, :, n:])
            ref = x[bi, :n] if k == "time_major" else x[bi, :, :n]
            assert torch.equal(valid, ref) and bool((pad == 7.0).all())
    packed = torch.zeros_like(host, device="cuda")
    ragged.ragged_copy(packed, dense, kinds, lens, to_dense=False)
    assert torch.equal(packed.cpu(), host)


@gpu
@needs_cuda
def test_ragged_pipeline_equals_direct_calls():
    """Only valid rows cross the host link; the outputs' valid rows equal the direct
    call's, bit for bit, over steps with different lengths, with and without the
    CUDA graphs of the device work."""
    from trifusion_b200 import fused_recurrence
    from trifusion_b200.synthetic import norm_weight, recurrence_inputs

    b, t, h = 4, 150, 12
    qw, kw = norm_weight(128, 1).cuda(), norm_weight(128, 2).cuda()

    def run(*xs, out):
        xs = list(xs)
        xs[8] = xs[8].expand(b, t, h, 32)
        return fused_recurrence(*xs[:11], q_norm=qw, k_norm=kw, lengths=xs[11], out=out)

    def step_inputs(s):
        xs = [x.contiguous() for x in recurrence_inputs(b, t, h, kind="baseline", seed=s, device="cpu")]
        xs[8] = xs[8][:, :, :1].contiguous()
        return xs

    for graphs in (False, True):
        _ragged_steps(run, step_inputs, b, t, h, qw, kw, graphs)


def _ragged_steps(run, step_inputs, b, t, h, qw, kw, graphs):
    from trifusion_b200 import fused_recurrence
    from trifusion_b200.host_pipeline import RaggedHostPipeline
    from trifusion_b200.synthetic import lengths_uniform

    pipe = RaggedHostPipeline(run, step_inputs(0), RECURRENCE_KINDS, (b, t, h, 64), torch.bfloat16, graphs=graphs)
    cases = []
    for s in range(5):
        xs = step_inputs(s)
        lens = lengths_uniform(b, 1, t, seed=s)
        block, out = pipe.host_block(), pipe.host_out()
        cases.append((xs, lens, block, pipe.pack(block, xs, lens), out, pipe.out_bytes(lens)))
    for xs, lens, block, nin, out, nout in cases:
        pipe.submit(block, nin, out, nout)
    pipe.synchronize()
    for xs, lens, block, nin, out, nout in cases:
        got = pipe.unpack_out(out, lens.tolist())
        dev = [x.cuda() for x in xs]
        dev[8] = dev[8].expand(b, t, h, 32)
        ref = fused_recurrence(*dev, q_norm=qw, k_norm=kw, lengths=lens.cuda()).cpu()
        assert torch.equal(got, ref)
        assert nin < pipe.capacity and nout < pipe.out_capacity
