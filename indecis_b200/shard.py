"""Sequences across GPUs, one process per GPU.

Sequences are independent in the encoder: the per-row GEMMs do not depend on
the batch (linalg/int8_test.go:149) and attention runs per (sequence, head)
(internal/modernbert/infer.go:490-517). So a batch is split into contiguous
ranges of sequences, one per rank, balanced by cost, each rank encodes its
range on its own GPU, and each writes its rows into a disjoint slice of one
host output. No data crosses between GPUs; the ranks only agree on the split,
which every rank computes from the same offsets.

Cost of a sequence of n tokens: the GEMMs and row work grow with n; attention
with n * keys per query, where a global layer sees n keys and a local one at
most local_attention + 1 (Window, internal/modernbert/model.go:60-80).
"""
from __future__ import annotations

from multiprocessing import shared_memory

import numpy as np


def seq_costs(offs, layers: int, global_every: int, local_attention: int, hidden: int) -> np.ndarray:
    """Relative cost of each sequence (operations, up to a constant)."""
    n = np.diff(np.asarray(offs, np.int64)).astype(np.float64)
    n_global = sum(1 for l in range(layers) if l % global_every == 0)
    n_local = layers - n_global
    gemm = 2.0 * n * (12.0 * hidden * hidden)  # QKV, Wo, Wi, WoMLP at I ~ 1.5 H: about 12 H^2 MACs per token
    attn = 4.0 * (hidden) * n * (n_global * n + n_local * np.minimum(n, local_attention + 1))
    return gemm * layers + attn


def shard_ranges(offs, world: int, costs=None) -> list[tuple[int, int]]:
    """Contiguous sequence ranges [s0, s1), one per rank, splitting the
    cumulative cost at the rank quantiles. Empty ranges are allowed (fewer
    sequences than ranks)."""
    nseq = len(offs) - 1
    if world < 1:
        raise ValueError("world must be >= 1")
    if costs is None:
        costs = np.diff(np.asarray(offs, np.int64)).astype(np.float64)
    costs = np.asarray(costs, np.float64)
    if len(costs) != nseq:
        raise ValueError("one cost per sequence")
    cum = np.concatenate([[0.0], np.cumsum(costs)])
    total = cum[-1]
    bounds = [0]
    for r in range(1, world):
        # first sequence whose cumulative cost start reaches r/world of the total
        b = int(np.searchsorted(cum, total * r / world, side="left"))
        b = min(max(b, bounds[-1]), nseq)
        bounds.append(b)
    bounds.append(nseq)
    return [(bounds[r], bounds[r + 1]) for r in range(world)]


def local_batch(ids, offs, s0: int, s1: int):
    """ids and offsets of sequences [s0, s1), offsets rebased to 0."""
    offs = np.asarray(offs, np.int64)
    t0, t1 = int(offs[s0]), int(offs[s1])
    return np.ascontiguousarray(np.asarray(ids)[t0:t1], np.int32), offs[s0:s1 + 1] - t0


class HostOutput:
    """A float32 [rows][width] host array in shared memory that every rank
    maps and writes its own rows of (the host gather)."""

    def __init__(self, name: str, rows: int, width: int, create: bool):
        size = max(1, rows * width * 4)
        self.shm = shared_memory.SharedMemory(name=name, create=create, size=size)
        self.array = np.ndarray((rows, width), np.float32, buffer=self.shm.buf)
        self.owner = create

    def write(self, row0: int, rows: np.ndarray):
        self.array[row0:row0 + len(rows)] = rows

    def close(self):
        self.array = None
        self.shm.close()
        if self.owner:
            self.shm.unlink()


def encode_shard(encode, ids, offs, rank: int, world: int, out: HostOutput, costs=None, mode: str = "pooled"):
    """Encodes this rank's range with encode(ids, offs) -> rows and writes
    them into the host output: pooled rows at the sequence index, token rows
    at the token index. Returns the range."""
    s0, s1 = shard_ranges(offs, world, costs)[rank]
    if s1 > s0:
        lid, loffs = local_batch(ids, offs, s0, s1)
        rows = encode(lid, loffs)
        out.write(s0 if mode == "pooled" else int(np.asarray(offs)[s0]), rows)
    return s0, s1
