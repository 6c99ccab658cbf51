"""Host-side partitioning of the decode-attention work across GPUs (one process per GPU).

The reference runs on one GPU only (engine/m1_engine.cpp:2165, ggml_backend_cuda_init(0)); these
two partitions are the multi-GPU extension of its split-K decomposition (m4-kqkv.cu:204-218):

* ``kv_slabs`` -- long context: every layer's KV cache is cut into contiguous sequence slabs, one
  per rank.  Each rank computes split-K partial records over its slab; the only exchange is an
  all-gather of those records (32 heads x 516 floats per split), then every rank merges them
  (PHASE selector 2).  The merge is the same online-softmax rule for local and remote splits.
* ``lpt_assign`` -- ragged batched decode: whole sequences per rank, balanced by total keys with
  the longest-processing-time greedy rule.  No exchange at all.
"""
from __future__ import annotations

import heapq


def kv_slabs(n_keys: int, world: int, align: int = 128) -> list[tuple[int, int]]:
    """Contiguous [begin, end) key ranges, one per rank, boundaries on ``align``-key tiles where
    possible, sizes differing by at most one tile."""
    if world < 1 or n_keys < 0:
        raise ValueError("world must be >= 1 and n_keys >= 0")
    tiles = (n_keys + align - 1) // align
    base, rem = divmod(tiles, world)
    out, t = [], 0
    for r in range(world):
        nt = base + (1 if r < rem else 0)
        b, e = min(t * align, n_keys), min((t + nt) * align, n_keys)
        out.append((b, e))
        t += nt
    return out


def lpt_assign(lengths: list[int], world: int) -> list[list[int]]:
    """Sequence indices per rank: longest first, each to the currently least-loaded rank
    (ties to the lowest rank).  Deterministic."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + lengths[i], r))
    for r in range(world):
        out[r].sort()
    return out


def ragged_lengths(seed: int = 5, n: int = 16, lo: int = 512, hi: int = 65536) -> list[int]:
    """The ragged decode batch: n sequence lengths uniform on [lo, hi]."""
    import numpy as np
    return [int(x) for x in np.random.default_rng(seed).integers(lo, hi + 1, n)]


def packed_bases(lengths: list[int]) -> list[int]:
    """First cache row of each sequence when the sequences are packed back to back."""
    out, r = [], 0
    for n in lengths:
        out.append(r)
        r += n
    return out


def rank_loads(lengths: list[int], assignment: list[list[int]]) -> list[int]:
    return [sum(lengths[i] for i in seqs) for seqs in assignment]
