"""Frame-grid bucketing, execution chunks and the per-rank shard of a batch of utterances.

Restates the reference's dispatch of encoder inputs:

* ``FRAME_GRID``: the padded frame count of a batch is rounded up to a multiple of the grid
  (``script/bench_asr.py:352-356``, ``script/fast/fast_asr.py:113-123``);
* ``EXEC_BATCH``: a logical batch is split into chunks of at most ``exec_batch`` utterances, each trimmed to its own
  longest utterance rounded up to the grid (``script/bench_asr.py:383-390``, ``:413-420``);
* the serving engine sorts utterances by duration before chunking (``serve/engine.py:78-86``).

Multi-GPU (the reference runs independent serving replicas, ``serve/ray_app.py:36-37``, each sorting and chunking
its own requests): ranks share no data.  Two ways to split one set of utterances over ranks:

* :func:`shard_utterances` deals the length-sorted utterances round robin, and each rank plans its own chunks from
  its share (the replica model).  Every rank gets the same length mix, so the padded work balances even when a rank
  holds only a couple of chunks (512 lognormal utterances over 8 ranks: the busiest rank carries 1.01x the mean);
* :func:`shard_chunks` plans the chunks once and assigns whole chunks greedily, longest padded work first, to the
  rank with the least padded frames so far (the same 512 utterances: 12 chunks, 1.24x the mean at 8 ranks).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

FRAME_GRID = 128
EXEC_BATCH = 48
LOGICAL_BATCH = 128


def bucket_frames(n: int, grid: int = FRAME_GRID) -> int:
    """Round a frame count up to the grid (grid <= 0 disables bucketing)."""
    n = int(n)
    if grid <= 0:
        return n
    return ((n + grid - 1) // grid) * grid


@dataclass
class Chunk:
    """One execution chunk: utterance indices (into the caller's list), their lengths and the padded T."""

    index: np.ndarray
    lengths: np.ndarray
    T: int

    @property
    def B(self) -> int:
        return int(self.index.size)

    @property
    def padded_frames(self) -> int:
        return self.B * self.T

    @property
    def valid_frames(self) -> int:
        return int(self.lengths.sum())


def plan_chunks(lengths, exec_batch: int = EXEC_BATCH, logical_batch: int = LOGICAL_BATCH,
                frame_grid: int = FRAME_GRID, sort: bool = True) -> list[Chunk]:
    """Sort utterances by length (stable), cut logical batches of ``logical_batch``, split each into chunks of at
    most ``exec_batch`` and give every chunk ``T = bucket(max length in chunk)``."""
    lengths = np.asarray(lengths, dtype=np.int64)
    if lengths.ndim != 1:
        raise ValueError("lengths must be 1-D")
    if np.any(lengths < 0):
        raise ValueError("negative utterance length")
    order = np.argsort(lengths, kind="stable") if sort else np.arange(lengths.size)
    chunks: list[Chunk] = []
    lb = logical_batch if logical_batch > 0 else max(1, lengths.size)
    eb = exec_batch if exec_batch > 0 else lb
    for s in range(0, order.size, lb):
        batch = order[s:s + lb]
        for c in range(0, batch.size, eb):
            idx = batch[c:c + eb]
            lens = lengths[idx]
            T = bucket_frames(max(int(lens.max()), 1), frame_grid)
            chunks.append(Chunk(index=idx.copy(), lengths=lens.astype(np.int32), T=T))
    return chunks


@dataclass
class Shard:
    rank: int
    chunks: list = field(default_factory=list)

    @property
    def padded_frames(self) -> int:
        return sum(c.padded_frames for c in self.chunks)

    @property
    def valid_frames(self) -> int:
        return sum(c.valid_frames for c in self.chunks)


def shard_chunks(chunks: list[Chunk], world_size: int) -> list[Shard]:
    """Greedy longest-processing-time assignment of chunks to ranks by padded frames (B*T); ties go to the lower
    rank.  Deterministic, so every rank computes the same plan without communicating."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    shards = [Shard(rank=r) for r in range(world_size)]
    load = [0] * world_size
    order = sorted(range(len(chunks)), key=lambda i: (-chunks[i].padded_frames, i))
    for i in order:
        r = min(range(world_size), key=lambda k: (load[k], k))
        shards[r].chunks.append(chunks[i])
        load[r] += chunks[i].padded_frames
    return shards


def shard_utterances(lengths, world_size: int) -> list[np.ndarray]:
    """Indices of each rank's utterances: sorted by length (stable), dealt round robin (utterance i of the sorted
    order to rank i mod world_size).  Deterministic, so every rank computes the same split without communicating;
    each rank then plans its chunks with :func:`plan_chunks` on its own share."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    order = np.argsort(np.asarray(lengths, dtype=np.int64), kind="stable")
    return [order[r::world_size].copy() for r in range(world_size)]
