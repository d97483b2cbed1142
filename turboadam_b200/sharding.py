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
