"""InferenceEngine's fallbacks, on the host with no GPU (reference runtime.py:116-128).

A capture that runs out of memory, or leaves more reserved than the engine's
limit, drops the graph, blacklists the shape and runs it eagerly from then on.
The CUDA calls of the capture path are replaced by fakes; the failure is a
``torch.cuda.OutOfMemoryError`` raised from the fake capture.
"""

import contextlib

import pytest
import torch

from trifusion_b200 import runtime


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.calls = 0

    def forward(self, audio, lengths, channels):
        self.calls += 1
        return {"logits": audio.sum(-1)[:, :1].repeat(1, 5) + lengths[:, None]}


class _FakeGraph:
    def replay(self):
        pass


@pytest.fixture
def fake_cuda(monkeypatch):
    state = {"oom": False, "reserved": 0, "captures": 0}

    @contextlib.contextmanager
    def graph(g, *a, **k):
        state["captures"] += 1
        if state["oom"]:
            raise torch.cuda.OutOfMemoryError("fake capture OOM")
        yield

    class _Stream:
        def wait_stream(self, other):
            pass

    monkeypatch.setattr(torch.cuda, "Stream", lambda *a, **k: _Stream())
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "synchronize", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    monkeypatch.setattr(torch.cuda, "CUDAGraph", _FakeGraph)
    monkeypatch.setattr(torch.cuda, "graph", graph)
    monkeypatch.setattr(torch.cuda, "memory_reserved", lambda *a, **k: state["reserved"])
    monkeypatch.setattr(runtime._lib, "check_device_error", lambda: None)
    return state


def _inputs(b=2, n=8):
    return torch.randn(b, 1, n), torch.tensor([n, n - 2][:b]), torch.ones(b, dtype=torch.int64)


def test_capture_oom_falls_back_to_eager_and_blacklists_the_shape(fake_cuda):
    model = _Model()
    engine = runtime.InferenceEngine(model, graphs=True)
    fake_cuda["oom"] = True
    x = _inputs()
    out = engine(*x)
    assert torch.equal(out, model(*x)["logits"])
    key = (tuple(x[0].shape), x[0].dtype)
    assert key in engine.disabled_shapes and key not in engine.cache
    captures = fake_cuda["captures"]
    fake_cuda["oom"] = False
    engine(*x)  # the shape stays eager: no second capture
    assert fake_cuda["captures"] == captures and engine.graph_hits == 0


def test_reserved_memory_limit_falls_back_to_eager(fake_cuda):
    engine = runtime.InferenceEngine(_Model(), graphs=True, max_reserved_gib=1.0)
    fake_cuda["reserved"] = 2 * 2**30
    x = _inputs()
    engine(*x)
    assert (tuple(x[0].shape), x[0].dtype) in engine.disabled_shapes and not engine.cache


def test_capture_within_limits_is_cached_and_replayed(fake_cuda):
    engine = runtime.InferenceEngine(_Model(), graphs=True, max_graphs=1)
    x = _inputs()
    engine(*x)
    engine(*x)
    assert len(engine.cache) == 1 and engine.graph_hits == 2 and fake_cuda["captures"] == 1
    y = _inputs(1, 16)
    engine(*y)  # LRU of one: the first shape is evicted
    assert list(engine.cache) == [(tuple(y[0].shape), y[0].dtype)]
