"""Host logic of the data-parallel runner: length buckets, LPT partition and
the final logits gather (world size 2 over gloo on the CPU)."""

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from trifusion_b200.audio import BUCKET_SECONDS, SAMPLE_RATE, AudioFile, bucket_samples, plan_batches
from trifusion_b200.sharding import batch_cost, gather_logits, lpt_partition
from trifusion_b200.synthetic import batch_audio, clip_set


def test_buckets_follow_reference_rule():
    assert bucket_samples(1) == 4 * SAMPLE_RATE
    assert bucket_samples(4 * SAMPLE_RATE) == 4 * SAMPLE_RATE
    assert bucket_samples(4 * SAMPLE_RATE + 1) == 8 * SAMPLE_RATE
    assert bucket_samples(72 * SAMPLE_RATE) == 72 * SAMPLE_RATE
    with pytest.raises(ValueError):
        bucket_samples(72 * SAMPLE_RATE + 1)


def test_plan_batches_groups_and_sizes():
    recs = clip_set(300, seed=1)
    plan = plan_batches(recs, padded_seconds=120, max_batch=32)
    seen = [r.index for _, rows in plan for r in rows]
    assert sorted(seen) == list(range(300))  # every clip exactly once
    for limit, rows in plan:
        assert limit // SAMPLE_RATE in BUCKET_SECONDS
        assert len({r.channels for r in rows}) == 1
        assert all(r.samples <= limit for r in rows)
        assert 1 <= len(rows) <= max(1, min(32, 120 * SAMPLE_RATE // limit))
    # groups come out in (channels, length) order
    keys = [(rows[0].channels, limit) for limit, rows in plan]
    assert keys == sorted(keys)


def test_lpt_partition_is_complete_deterministic_and_balanced():
    costs = [batch_cost(limit, rows) for limit, rows in plan_batches(clip_set(1024), max_batch=32)]
    for world in (1, 2, 4, 8):
        parts = lpt_partition(costs, world)
        assert sorted(i for p in parts for i in p) == list(range(len(costs)))
        assert parts == lpt_partition(costs, world)
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) <= max(sum(costs) / world, max(costs)) * 4 / 3


def test_batch_audio_padding_and_channels():
    rows = [AudioFile(0, None, 1000, 2), AudioFile(1, None, 300, 1)]
    audio, lengths, channels = batch_audio(1600, rows)
    assert audio.shape == (2, 2, 1600)
    assert lengths.tolist() == [1000, 300] and channels.tolist() == [2, 1]
    assert (audio[0, :, 1000:] == 0).all() and (audio[1, 1] == 0).all() and (audio[1, 0, 300:] == 0).all()
    assert audio[0, 1, :1000].abs().sum() > 0


def _gather_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        costs = [5, 3, 8, 1, 1, 4]
        mine = lpt_partition(costs, world)[rank]
        # each batch i holds clip indices [10*i, 10*i+1]; logits encode the clip index
        idx = torch.tensor([10 * i + j for i in mine for j in range(2)], dtype=torch.int64)
        logits = idx.double().unsqueeze(1).repeat(1, 5).float() + torch.arange(5).float()
        all_idx, all_logits = gather_logits(idx, logits)
        # One collective round when every rank knows a bound on the others' rows.
        cap = max(2 * len(p) for p in lpt_partition(costs, world))
        one_idx, one_logits = gather_logits(idx, logits, capacity=cap)
        assert torch.equal(one_idx, all_idx) and torch.equal(one_logits, all_logits)
        out[rank] = (all_idx.tolist(), all_logits.tolist())
    finally:
        dist.destroy_process_group()


def test_gather_logits_two_ranks_gloo():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_gather_worker, args=(2, port, out), nprocs=2, join=True)
    expect = sorted(10 * i + j for i in range(6) for j in range(2))
    for rank in range(2):
        idx, logits = out[rank]
        assert idx == expect
        assert logits == [[float(i) + k for k in range(5)] for i in expect]
