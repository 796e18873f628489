"""Sequence-slot sharding across the GPUs of one box.

Sequences (and the state slots they own) are independent units of the decode path, so a
multi-GPU deployment partitions them: sequence s of N goes to rank floor(s * G / N).  Each rank
holds its own slot pool (slot 0 reserved as the null slot) and the activations of its
sequences; no data-path collective exists.  Only timing is combined across ranks (max of the
per-rank device times, sum of per-rank bytes).
"""

from __future__ import annotations


def owner(sequence: int, total: int, world: int) -> int:
    """Rank that owns `sequence` out of `total` sequences over `world` ranks."""
    if not 0 <= sequence < total:
        raise ValueError("sequence out of range")
    return sequence * world // total


def shard_range(total: int, rank: int, world: int) -> range:
    """The contiguous block of sequences owned by `rank`: {s : owner(s) == rank}."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    start = -(-rank * total // world)          # ceil(rank * total / world)
    stop = -(-(rank + 1) * total // world)
    return range(start, stop)


def local_slot(sequence: int, total: int, world: int, slots_per_sequence: int = 1, candidate: int = 0) -> int:
    """Slot of (sequence, candidate) inside its owner's pool; slot 0 stays the null slot."""
    rank = owner(sequence, total, world)
    first = shard_range(total, rank, world).start
    return 1 + (sequence - first) * slots_per_sequence + candidate
