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


class Zero1ParamGather:
    """ZeRO-1 around TurboAdam: every rank holds the full parameters, steps
    the ``zero1_partition`` range it owns, and gathers the others' updated
    ranges after the step (the post-step parameter all-gather).

    ``params`` is the full parameter list, identically ordered and shaped on
    every rank. :meth:`optimizer_args` gives this rank's shard parameters --
    views into the full tensors, so the step updates them in place -- with
    the ``tensor_ids`` / ``shards`` / ``spanning`` arguments of TurboAdam.
    :meth:`gather` then broadcasts each rank's updated ranges to all ranks
    (``torch.distributed``; NCCL on GPUs, gloo on CPU). When the parameters
    are consecutive views of one flat buffer (the usual ZeRO layout) each
    rank's range is one contiguous span and the gather is one broadcast per
    rank; otherwise one broadcast per shard. Each rank receives the
    (world - 1) / world of the parameter bytes it does not own -- the
    NVLink-bound part of ZeRO-1, which no fusion with the step reduces.
    The step needs every shard to start 16-byte aligned: in a flat buffer,
    pad each tensor to a multiple of 4 (fp32) or 8 (bf16) elements.
    """

    def __init__(self, params, world: int | None = None, rank: int | None = None,
                 process_group=None, block_size: int = 128):
        import torch.distributed as dist

        self.params = list(params)
        self.group = process_group
        self.world = dist.get_world_size(process_group) if world is None else int(world)
        self.rank = dist.get_rank(process_group) if rank is None else int(rank)
        numels = [p.numel() for p in self.params]
        self.partition = zero1_partition(numels, self.world, block_size)
        self.spanning = zero1_spanning(self.partition)
        self._flat = self._flat_spans(numels)

    def _flat_spans(self, numels):
        """(base tensor, [(lo, hi)] per rank) when the parameters are
        consecutive slices of one contiguous storage, else None."""
        ps = self.params
        if not ps or any(not p.is_contiguous() for p in ps):
            return None
        esz = ps[0].element_size()
        if any(p.dtype != ps[0].dtype or p.device != ps[0].device for p in ps):
            return None
        for a, b in zip(ps, ps[1:]):
            if b.data_ptr() != a.data_ptr() + a.numel() * esz:
                return None
        starts = [0]
        for n in numels:
            starts.append(starts[-1] + n)
        base = ps[0].detach().view(-1)
        base = base.as_strided((starts[-1],), (1,), base.storage_offset())
        spans = []
        for shards in self.partition:
            if not shards:
                spans.append((0, 0))
                continue
            t0, e0 = shards[0][0], shards[0][1]
            t1, e1 = shards[-1][0], shards[-1][2]
            spans.append((starts[t0] + e0, starts[t1] + e1))
        return base, spans

    def optimizer_args(self):
        """(shard params, kwargs for TurboAdam) of this rank."""
        import torch

        mine = self.partition[self.rank]
        shard_params = [torch.nn.Parameter(self.params[t].detach().view(-1)[e0:e1])
                        for t, e0, e1, _, _ in mine]
        kw = dict(tensor_ids=[t for t, *_ in mine],
                  shards=[(boff, gn) for _, _, _, boff, gn in mine],
                  spanning=self.spanning, process_group=self.group)
        return shard_params, kw

    def gather(self) -> None:
        """Broadcast every rank's updated ranges to all ranks."""
        import torch.distributed as dist

        work = []
        if self._flat is not None:
            base, spans = self._flat
            for r, (lo, hi) in enumerate(spans):
                if hi > lo:
                    work.append(dist.broadcast(base[lo:hi], src=self._global_rank(r),
                                               group=self.group, async_op=True))
        else:
            for r, shards in enumerate(self.partition):
                for t, e0, e1, _, _ in shards:
                    work.append(dist.broadcast(self.params[t].detach().view(-1)[e0:e1],
                                               src=self._global_rank(r), group=self.group,
                                               async_op=True))
        for w in work:
            w.wait()

    def _global_rank(self, r: int) -> int:
        import torch.distributed as dist

        if self.group is None:
            return r
        return dist.get_global_rank(self.group, r)
