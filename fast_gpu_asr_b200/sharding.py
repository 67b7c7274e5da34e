"""Data-parallel sharding of utterance batches over GPUs (one process per GPU).

Both attention variants are independent per utterance: the reference has no
cross-utterance term in any plugin (``parakeet_relative_attention_plugin.cu`` and
``zipformer_relative_attention_plugin.cu`` index every tensor by batch row first), so the
batch dimension shards with no collective on the data path. The plan here is the one the
benchmark configuration describes for the ragged whole-box run:

* utterances are sorted by length and cut into batches of ``batch_size`` (similar lengths
  per batch keep the padded frame count low);
* batches are dealt to ranks either round-robin (batch ``b`` to rank ``b % world``) or,
  by default in the ragged benchmark, longest processing time first: batches in order
  of decreasing estimated cost, each to the rank with the least estimated work so far.
  Round-robin over a length-sorted plan gives rank 0 the longest batch of every round,
  which grows the slowest rank's share with the number of ranks; the greedy deal keeps
  the estimated loads within one batch's cost of each other;
* or dynamically (``DynamicDeal``): the ranks take batches one at a time, longest first,
  from a shared counter in a key-value store, each as soon as its GPU has finished the
  previous one, so measured rather than estimated times balance the ranks;
* each rank runs its batches on its own GPU and stream;
* at the end the per-batch outputs are gathered to rank 0 with point-to-point sends
  (NCCL over NVLink on GPUs, gloo in the CPU tests), outside the timed kernels.

Every rank derives the same plan from the same seed, so only tensor data crosses ranks.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class Batch:
    index: int               # position in the length-sorted plan
    utterances: np.ndarray   # utterance ids (indices into the input list), longest first
    lengths: np.ndarray      # their lengths, same order

    @property
    def max_length(self) -> int:
        return int(self.lengths.max()) if self.lengths.size else 0


def length_sorted_batches(lengths, batch_size: int) -> list[Batch]:
    """Cut utterances into batches of ``batch_size`` after a stable longest-first sort."""
    lengths = np.asarray(lengths)
    if lengths.ndim != 1:
        raise ValueError("lengths must be one-dimensional")
    if batch_size < 1:
        raise ValueError("batch_size must be positive")
    order = np.argsort(-lengths, kind="stable")
    return [Batch(i // batch_size, order[i : i + batch_size], lengths[order[i : i + batch_size]])
            for i in range(0, len(order), batch_size)]


def shard_round_robin(num_batches: int, world: int, rank: int) -> list[int]:
    """Batch indices that ``rank`` of ``world`` runs: b with b % world == rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return list(range(rank, num_batches, world))


def batch_costs(plan: list[Batch]) -> np.ndarray:
    """Estimated relative cost of each batch: utterances x (longest length)^2, the work of
    attention over a batch padded to its longest utterance."""
    return np.array([len(b.lengths) * float(b.max_length) ** 2 for b in plan])


def shard_longest_first(costs, world: int) -> list[list[int]]:
    """Longest-processing-time deal: batch indices per rank. Batches are taken in order of
    decreasing cost (ties by index) and each goes to the rank with the least total cost so
    far (ties to the lower rank). Deterministic, so every rank derives the same deal.
    Each rank's list is in increasing batch order."""
    if world < 1:
        raise ValueError("world must be positive")
    costs = np.asarray(costs, dtype=np.float64)
    loads = np.zeros(world)
    shards: list[list[int]] = [[] for _ in range(world)]
    for b in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        r = int(np.argmin(loads))
        shards[r].append(b)
        loads[r] += costs[b]
    return [sorted(s) for s in shards]


class DynamicDeal:
    """Batches taken one at a time from a counter shared by all ranks.

    ``store`` is a ``torch.distributed`` key-value store reachable by every rank (for
    example a ``TCPStore`` hosted by rank 0); ``order`` is the sequence in which batches are
    handed out (longest first: ``np.argsort(-costs, kind="stable")``). Each ``next()`` is one
    atomic increment of ``key`` in the store and returns the next batch index, or None when
    every batch is taken; every batch goes to exactly one rank. ``taken`` lists this rank's
    batches in the order it took them. After the last ``next()``, ``assignment()`` (a
    collective over the default process group) returns every rank's list for the gather.
    """

    def __init__(self, store, order, key: str = "fga_deal_next"):
        self.store = store
        self.order = [int(b) for b in order]
        self.key = key
        self.taken: list[int] = []

    def next(self) -> int | None:
        i = int(self.store.add(self.key, 1)) - 1
        if i >= len(self.order):
            return None
        self.taken.append(self.order[i])
        return self.order[i]

    def assignment(self, world: int) -> list[list[int]]:
        if world == 1:
            return [sorted(self.taken)]
        import torch.distributed as dist

        lists: list = [None] * world
        dist.all_gather_object(lists, sorted(self.taken))
        return [list(x) for x in lists]


def gather_to_rank0(outputs: dict, plan_shapes: dict, world: int, rank: int, device,
                    dtype, assignment: list[list[int]] | None = None) -> dict | None:
    """Gather every rank's per-batch outputs to rank 0.

    ``outputs`` maps this rank's batch indices to a tensor or a list of tensors;
    ``plan_shapes`` maps every batch index of the plan to the shape, or list of shapes, of
    those tensors (all ranks know the plan). ``assignment[r]`` lists rank r's batches
    (default: round-robin). Each rank sends its batches' tensors, flattened in batch order,
    as one buffer; rank 0 receives the buffers of the other ranks and returns {batch index:
    tensor or list of tensors} for the whole plan. The other ranks return None.
    Collective: every rank must call it. A rank that fails before its send makes rank 0's
    receive fail (gloo: closed connection; NCCL: the process group's timeout) instead of
    waiting for ever.
    """
    import torch
    import torch.distributed as dist

    if assignment is None:
        assignment = [shard_round_robin(len(plan_shapes), world, r) for r in range(world)]
    mine = assignment[rank]
    if sorted(outputs) != sorted(mine):
        raise ValueError("outputs must cover exactly this rank's batches")
    single = {b: not isinstance(plan_shapes[b], list) for b in plan_shapes}
    shapes = {b: [plan_shapes[b]] if single[b] else list(plan_shapes[b]) for b in plan_shapes}
    if world == 1:
        return dict(outputs)

    def tensors(b):
        return [outputs[b]] if single[b] else list(outputs[b])

    if rank != 0:
        parts = [t.reshape(-1).to(dtype) for b in mine for t in tensors(b)]
        flat = torch.cat(parts) if parts else torch.empty(0, dtype=dtype, device=device)
        dist.send(flat.contiguous(), dst=0)
        return None
    gathered = dict(outputs)
    for src in range(1, world):
        theirs = assignment[src]
        sizes = [[int(np.prod(sh)) for sh in shapes[b]] for b in theirs]
        buf = torch.empty(sum(map(sum, sizes)), dtype=dtype, device=device)
        dist.recv(buf, src=src)
        off = 0
        for b, bsizes in zip(theirs, sizes):
            got = []
            for sh, n in zip(shapes[b], bsizes):
                got.append(buf[off : off + n].reshape(sh))
                off += n
            gathered[b] = got[0] if single[b] else got
    return gathered
