"""bench.py's micro-batches on the CPU: every timed micro-batch is full (max_batch
distinct symbols owned by the rank), so per-GPU work does not shrink as the GPU
count grows, and when the Zipf stream yields fewer full micro-batches than a run
needs they are reused in stream order."""

import numpy as np

import bench
from hackathon_b200 import batcher as B


def test_micro_batches_are_full_distinct_owned_and_reused_in_order():
    wl = dict(bench.WORKLOADS["scaleout"], max_batch=256)
    n_sym, world, rank, count = 4096, 4, 1, 60
    info = {}
    batches, capacity = bench.make_batches(wl, n_sym, world, rank, count, backlog=100_000, info=info)
    mine, _ = B.shard_slots(n_sym, world, rank)
    assert capacity == len(mine) and len(batches) == count
    for b in batches:
        assert len(b) == 256 and len(set(b.tolist())) == 256
        assert b.min() >= 0 and b.max() < capacity
    d = info["distinct"]
    assert 1 <= d < count  # this stream runs out of full micro-batches for this rank
    for i in range(count):
        assert np.array_equal(batches[i], batches[i % d])
    # with a deep enough stream nothing is reused
    info2 = {}
    b2, _ = bench.make_batches(wl, n_sym, world, rank, 8, backlog=100_000, info=info2)
    assert info2["distinct"] == 8 and all(np.array_equal(x, y) for x, y in zip(b2, batches[:8]))
