"""Placement of attention work on the GPUs of one box (one process per GPU).

The reference runs attention on the host with OpenMP over (batch, head) pairs
(csrc/gt_ops_nn.cpp:2468) and has no multi-device path. Here the independent units are
(batch, kv head) pairs: a kv head carries its H/Hkv query heads, so dK/dV of a unit never need a
cross-GPU reduction and the forward, backward and decode shard with no collective on the data path.

* prefill / training: contiguous ranges of the B*Hkv units, sizes differing by at most one;
* decode: whole sequences, balanced by cached length (the work is proportional to it) with a
  longest-first greedy assignment.
"""

from __future__ import annotations


def unit_range(n_units: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of the units rank `rank` of `world` owns: contiguous, sizes differ by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_head_units(B: int, Hkv: int, world: int, rank: int) -> list[tuple[int, int]]:
    """The (batch, kv head) pairs of one rank, in row-major order of (b, hk)."""
    start, stop = unit_range(B * Hkv, world, rank)
    return [(u // Hkv, u % Hkv) for u in range(start, stop)]


def balance_sequences(lengths, world: int) -> list[list[int]]:
    """Assign sequences to ranks so the summed lengths are balanced (longest first, each to the
    currently lightest rank; ties go to the lower rank). Returns per-rank sorted index lists."""
    if world <= 0:
        raise ValueError("world must be positive")
    load = [0] * world
    owned = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owned[r].append(i)
        load[r] += max(int(lengths[i]), 0)
    return [sorted(o) for o in owned]
