"""The multi-GPU host logic of bench.py on CPU: two ranks over gloo.

Symbols are sharded over ranks by splitmix64 (no collective on the data path);
each rank forms its own micro-batches from the shared arrival stream; the
timing reduction takes the max over ranks and the request count the sum.
"""

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2
N_SYMBOLS = 4096


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        import bench
        from hackathon_b200 import batcher as B

        wl = dict(bench.WORKLOADS["scaleout"], max_batch=256)
        batches, capacity = bench.make_batches(wl, N_SYMBOLS, WORLD, rank, 8, backlog=200_000)
        mine, slot_of = B.shard_slots(N_SYMBOLS, WORLD, rank)
        owned = [None] * WORLD
        dist.all_gather_object(owned, mine.tolist())
        cpu = torch.device("cpu")
        t_max = bench.allreduce(float(10 + rank), "max", WORLD, cpu)
        rows = bench.allreduce(float(sum(len(b) for b in batches)), "sum", WORLD, cpu)
        bench.barrier(WORLD)
        q.put((rank, capacity, len(mine), [b.tolist() for b in batches], owned, t_max, rows,
               slot_of[mine].tolist()))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_symbols_and_reduce_timings():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(WORLD):
        r = q.get(timeout=120)
        out[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    owned = out[0][4]
    assert owned == out[1][4]  # every rank gathered the same ownership
    a, b = set(owned[0]), set(owned[1])
    assert not a & b and a | b == set(range(N_SYMBOLS))  # disjoint, complete
    sent = 0
    for rank in range(WORLD):
        _, capacity, n_mine, batches, _, t_max, rows, slots = out[rank]
        assert capacity == n_mine == len(owned[rank])
        assert slots == list(range(n_mine))  # owned symbols get slots 0..n-1
        assert t_max == 10.0 + (WORLD - 1)
        assert len(batches) == 8
        for bt in batches:
            assert 0 < len(bt) <= 256
            assert len(set(bt)) == len(bt)  # one request per symbol per micro-batch
            assert min(bt) >= 0 and max(bt) < capacity
        sent += sum(len(bt) for bt in batches)
    assert out[0][6] == out[1][6] == float(sent)
