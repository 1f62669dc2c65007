"""Checkpoint loading, runtime settings and CUDA-graph inference (reference
``runtime.py``), for B200.

``load_student`` reads the reference's checkpoint format
(``{"model_config": dict, "model": state_dict}``) with a strict key check;
``InferenceEngine(graphs=True)`` captures one CUDA graph per input shape in a
bounded LRU cache and replays it, falling back to eager execution for shapes
whose capture runs out of memory or exceeds the reserved-memory limit.
"""

from __future__ import annotations

import gc
import time
from collections import OrderedDict
from dataclasses import fields

import torch

from . import _lib
from .model import ModelConfig, TriFusion

B200_CAPABILITY = (10, 0)


def load_student(path, optimized=True, device="cuda"):
    """Build the student from a saved checkpoint (reference ``runtime.py:11-48``).

    ``optimized=True`` selects the B200 kernels (backend ``"l4"``), fused
    recurrence launches and BF16 GEMM/convolution weights; ``optimized=False``
    keeps FP32 weights and the reference's PyTorch formulas around the
    recurrence. Unknown configuration fields and any key mismatch raise.
    """
    saved = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
    config = dict(saved["model_config"])
    known = {f.name for f in fields(ModelConfig)}
    if set(config) - known:
        raise ValueError("Unsupported model configuration fields")
    config.update(
        backend="l4" if optimized else "reference",
        checkpoint_blocks=False,
        checkpoint_frontend=False,
        buffer_fusion=optimized,
        native_kernels=optimized,
        paired_mamba=False,
    )
    # Shapes only: the checkpoint's tensors are attached below (assign=True).
    with torch.device("meta"):
        model = TriFusion(ModelConfig(**config))
    del model.memory_head  # training-only head, absent from deployed weights
    state = {k: v for k, v in saved["model"].items()
             if not k.startswith(("kd_features.", "memory_head."))}
    model.load_state_dict(state, strict=True, assign=True)
    # The STFT window is a non-persistent buffer: materialise it.
    model.front.window = torch.hann_window(400, periodic=True)
    model.eval().requires_grad_(False)
    for block in model.blocks:
        block.forward_mamba.fused_recurrence = optimized
        block.backward_mamba.fused_recurrence = optimized
    if optimized:
        prepare_static_weights(model)
    return model.to(device)


def prepare_static_weights(model):
    """Cast GEMM/convolution weights to BF16 once; norms and controls stay FP32."""
    for module in model.modules():
        if isinstance(module, (torch.nn.Linear, torch.nn.Conv1d, torch.nn.Conv2d)):
            module.to(dtype=torch.bfloat16)
        if isinstance(module, torch.nn.Conv2d):  # the front end runs channels-last
            module.to(memory_format=torch.channels_last)


def configure_runtime(threads=2, enforce_l4=True):
    """Process-wide settings for validated inference (reference ``runtime.py:59-67``).

    The device check is for the B200 (sm_100) this build targets; the keyword
    keeps its reference name so existing callers run unchanged.
    """
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA GPU is required")
    if enforce_l4 and torch.cuda.get_device_capability() != B200_CAPABILITY:
        raise RuntimeError("This runtime is validated for B200/SM100")
    torch.set_num_threads(threads)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cudnn.benchmark = False


class InferenceEngine:
    """Eager or CUDA-graph inference (reference ``runtime.py:70-138``).

    ``max_reserved_gib`` bounds the caching allocator's reservation after a
    capture (a capture that leaves more reserved is dropped and its shape runs
    eagerly); the default is the reference's 19.5 GiB. Callers that batch many
    seconds of audio per call on a 180 GB B200 pass a larger bound.
    """

    def __init__(self, model, graphs=False, max_graphs=2, max_reserved_gib=19.5):
        self.model = model
        self.graphs = graphs
        self.max_graphs = max_graphs
        self.limit = int(max_reserved_gib * 2**30)
        self.cache = OrderedDict()
        self.disabled_shapes = set()
        self.graph_build_seconds = 0.0
        self.graph_hits = 0

    @torch.inference_mode()
    def eager(self, audio, lengths, channels):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            return self.model(audio, lengths, channels)["logits"]

    def clear(self):
        self.cache.clear()
        gc.collect()
        torch.cuda.empty_cache()

    def _capture(self, key, audio, lengths, channels):
        while len(self.cache) >= self.max_graphs:
            self.cache.popitem(last=False)
        gc.collect()
        torch.cuda.empty_cache()
        start = time.perf_counter()
        x, l, c = audio.clone(), lengths.clone(), channels.clone()
        # Warm up on a side stream: loads cuFFT/cuBLAS plans and sizes the
        # recurrence workspace before capture.
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                self.eager(x, l, c)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph):
                out = self.eager(x, l, c)
        except torch.cuda.OutOfMemoryError:
            del graph, x, l, c
            self.clear()
            self.disabled_shapes.add(key)
            return None
        self.graph_build_seconds += time.perf_counter() - start
        if torch.cuda.memory_reserved() > self.limit:
            del graph, out, x, l, c
            self.clear()
            self.disabled_shapes.add(key)
            return None
        entry = (graph, x, l, c, out)
        self.cache[key] = entry
        return entry

    @torch.inference_mode()
    def __call__(self, audio, lengths, channels):
        # A device-side timeout of an earlier call surfaces here (host-mapped word, no sync).
        _lib.check_device_error()
        key = (tuple(audio.shape), audio.dtype)
        if not self.graphs or key in self.disabled_shapes:
            return self.eager(audio, lengths, channels)
        entry = self.cache.get(key)
        if entry is None:
            entry = self._capture(key, audio, lengths, channels)
            if entry is None:
                return self.eager(audio, lengths, channels)
        graph, x, l, c, out = entry
        self.cache.move_to_end(key)
        x.copy_(audio)
        l.copy_(lengths)
        c.copy_(channels)
        graph.replay()
        self.graph_hits += 1
        # A later replay overwrites the graph's output buffer: return a copy.
        return out.clone()
