"""By-tensor sharding of a parameter set over data-parallel ranks.

Every 128-element block of the step is independent except two per-tensor
reductions (alpha and the ratio thresholds), so assigning whole tensors to
ranks makes the step collective-free. The assignment is a greedy LPT
(largest tensor first, to the least-loaded rank; ties to the lowest rank), a
pure function of the tensor sizes, so every rank computes the same owners
without communication.

Each rank steps only its own tensors with a ``TurboAdam`` built over them,
passing their global indices as ``tensor_ids`` so the stochastic-rounding
streams -- keyed by (seed, tensor id, step, element) -- and hence the packed
state are identical for every world size.
"""
from __future__ import annotations

from typing import Sequence


def lpt_owners(numels: Sequence[int], world: int) -> list[int]:
    """Owner rank of each tensor (greedy longest-processing-time)."""
    if world < 1:
        raise ValueError(f"world size must be >= 1, got {world}")
    order = sorted(range(len(numels)), key=lambda i: (-int(numels[i]), i))
    load = [0] * world
    owner = [0] * len(numels)
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        owner[i] = r
        load[r] += int(numels[i])
    return owner


def shard_by_tensor(params: Sequence, world: int, rank: int):
    """(local params, their global indices) owned by ``rank``.

    ``params`` is the full, identically ordered parameter list on every rank
    (tensors or anything with ``numel()``).
    """
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    owners = lpt_owners([p.numel() for p in params], world)
    ids = [i for i, o in enumerate(owners) if o == rank]
    return [params[i] for i in ids], ids


def rank_loads(numels: Sequence[int], world: int) -> list[int]:
    """Elements per rank under :func:`lpt_owners`."""
    load = [0] * world
    for n, r in zip(numels, lpt_owners(numels, world)):
        load[r] += int(n)
    return load


ALIGN_BLOCKS = 4096  # TA_SHARD_ALIGN_BLOCKS: one alpha reduction chunk


def zero1_partition(numels: Sequence[int], world: int, block_size: int = 128):
    """ZeRO-1 flat partition of a parameter set (all tensors concatenated in
    order) into ``world`` contiguous ranges of about equal size. A cut inside a
    tensor is moved to the nearest multiple of ALIGN_BLOCKS blocks of that
    tensor (or to its start / end), so no alpha reduction chunk straddles two
    ranks. Returns, per rank, a list of shards
    ``(tensor_index, elem_lo, elem_hi, block_offset, global_numel)``."""
    if world < 1:
        raise ValueError(f"world size must be >= 1, got {world}")
    numels = [int(n) for n in numels]
    starts = [0]
    for n in numels:
        starts.append(starts[-1] + n)
    total = starts[-1]
    align = ALIGN_BLOCKS * block_size
    cuts = [0]
    for r in range(1, world):
        x = (total * r) // world
        t = max(i for i in range(len(numels)) if starts[i] <= x) if numels else 0
        off = x - starts[t]
        snapped = min(numels[t], int(round(off / align)) * align) if numels else 0
        cuts.append(max(cuts[-1], starts[t] + snapped))
    cuts.append(total)
    out = []
    for r in range(world):
        lo, hi = cuts[r], cuts[r + 1]
        mine = []
        for t, n in enumerate(numels):
            a, b = max(lo, starts[t]), min(hi, starts[t] + n)
            if a < b:
                e0, e1 = a - starts[t], b - starts[t]
                mine.append((t, e0, e1, e0 // block_size, n))
        out.append(mine)
    return out


def zero1_spanning(partition):
    """The job's tensors that a zero1_partition splits over ranks, as
    ``(tensor_index, global_numel)`` in tensor order (the same on every
    rank): the ``spanning`` argument of TurboAdam."""
    count, numel = {}, {}
    for shards in partition:
        for t, _, _, _, gn in shards:
            count[t] = count.get(t, 0) + 1
            numel[t] = gn
    return [(t, numel[t]) for t in sorted(count) if count[t] > 1]
