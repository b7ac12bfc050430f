"""Request streams, symbol sharding and micro-batch formation for the scale-out path.

* ``zipf_stream``: synthetic arrivals - symbol ids drawn from a Zipf(s) law over
  ``n_symbols`` ranks (rank r has weight r^-s), the ranks scattered over the ids
  by a seeded permutation so hot symbols do not cluster on one shard.
* ``owner``: stable shard of a symbol key across GPUs (splitmix64 mod N; a
  name's key is its crc32). Each GPU holds only its own symbols' state; no
  collective is needed on the path.
* ``micro_batches``: the reference's round rule (example_model.py:885-899) over a
  backlog - the k-th pending request of every symbol goes to round k, so a
  symbol appears at most once per batch and its requests stay in order - with
  each round cut into micro-batches of at most ``max_batch`` requests.
"""

from __future__ import annotations

import zlib
from typing import List, Tuple

import numpy as np

_M64 = (1 << 64) - 1


def splitmix64(x: np.ndarray) -> np.ndarray:
    z = (x.astype(np.uint64) + np.uint64(0x9E3779B97F4A7C15)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)) & np.uint64(_M64)
    z = ((z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)) & np.uint64(_M64)
    return z ^ (z >> np.uint64(31))


def owner(symbol_ids: np.ndarray, n_shards: int) -> np.ndarray:
    """Shard of each symbol key: splitmix64(key) mod n_shards. The one sharding
    rule of the package: the bench's keys are the dense symbol ids, the client's
    the crc32 of the symbol name (``symbol_key``)."""
    if n_shards <= 1:
        return np.zeros(len(symbol_ids), np.int64)
    with np.errstate(over="ignore"):
        return (splitmix64(np.asarray(symbol_ids)) % np.uint64(n_shards)).astype(np.int64)


def symbol_key(name: str) -> int:
    """Integer key of a symbol name for ``owner``: crc32 of its UTF-8 bytes."""
    return zlib.crc32(name.encode("utf-8"))


def zipf_stream(n_symbols: int, n_requests: int, s: float = 1.1, seed: int = 0) -> np.ndarray:
    """Symbol ids (int64) of n_requests arrivals, Zipf(s) over n_symbols ranks."""
    rng = np.random.default_rng(seed)
    w = np.arange(1, n_symbols + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    ranks = np.searchsorted(cdf, rng.random(n_requests), side="right")
    ranks = np.minimum(ranks, n_symbols - 1)
    perm = rng.permutation(n_symbols)
    return perm[ranks].astype(np.int64)


def micro_batches(stream: np.ndarray, max_batch: int, limit: int | None = None) -> List[np.ndarray]:
    """Indices into `stream` per micro-batch, by the round rule (module docstring)."""
    order = np.argsort(stream, kind="stable")
    sorted_ids = stream[order]
    starts = np.r_[0, np.flatnonzero(np.diff(sorted_ids)) + 1]
    occ = np.empty(len(stream), np.int64)  # occurrence index of each request within its symbol
    occ[order] = np.arange(len(stream)) - np.repeat(starts, np.diff(np.r_[starts, len(stream)]))
    batches: List[np.ndarray] = []
    by_round = np.argsort(occ, kind="stable")  # round-major, arrival order inside a round
    rounds = occ[by_round]
    bounds = np.r_[0, np.flatnonzero(np.diff(rounds)) + 1, len(by_round)]
    for a, b in zip(bounds[:-1], bounds[1:]):
        for c in range(a, b, max_batch):
            batches.append(by_round[c:min(b, c + max_batch)])
            if limit is not None and len(batches) >= limit:
                return batches
    return batches


def continuous_batches(stream: np.ndarray, max_batch: int, limit: int | None = None) -> List[np.ndarray]:
    """Indices into `stream` per micro-batch, batching continuously across rounds.

    Each micro-batch takes the oldest pending request of up to `max_batch`
    distinct symbols, oldest head first. A symbol still appears at most once per
    batch and its requests keep their order (its next request can only join a
    later batch), but a batch does not stop at a round boundary, so it stays full
    while at least `max_batch` symbols have work queued.
    """
    import heapq

    order = np.argsort(stream, kind="stable")
    ids = stream[order]
    starts = np.r_[0, np.flatnonzero(np.diff(ids)) + 1]
    ends = np.r_[starts[1:], len(ids)]
    # heap of (arrival index of the symbol's head request, symbol group)
    heap = [(int(order[a]), g) for g, a in enumerate(starts)]
    heapq.heapify(heap)
    pos = starts.copy()
    batches: List[np.ndarray] = []
    while heap and (limit is None or len(batches) < limit):
        take = [heapq.heappop(heap) for _ in range(min(max_batch, len(heap)))]
        batches.append(np.fromiter((h for h, _ in take), np.int64, len(take)))
        for _, g in take:
            pos[g] += 1
            if pos[g] < ends[g]:
                heapq.heappush(heap, (int(order[pos[g]]), g))
    return batches


def shard_slots(n_symbols: int, n_shards: int, shard: int) -> Tuple[np.ndarray, np.ndarray]:
    """(symbol ids owned by `shard`, slot of every symbol id or -1 when not owned)."""
    ids = np.arange(n_symbols, dtype=np.int64)
    mine = ids[owner(ids, n_shards) == shard]
    slot = np.full(n_symbols, -1, np.int64)
    slot[mine] = np.arange(len(mine))
    return mine, slot
