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
