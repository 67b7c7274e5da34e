"""Data-parallel sharding of utterance batches over GPUs (one process per GPU).

Both attention variants are independent per utterance: the reference has no
cross-utterance term in any plugin (``parakeet_relative_attention_plugin.cu`` and
``zipformer_relative_attention_plugin.cu`` index every tensor by batch row first), so the
batch dimension shards with no collective on the data path. The plan here is the one the
benchmark configuration describes for the ragged whole-box run:

* utterances are sorted by length and cut into batches of ``batch_size`` (similar lengths
  per batch keep the padded frame count low);
* batch ``b`` goes to rank ``b % world`` (round-robin, so every rank gets a mix of long
  and short batches);
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


def gather_to_rank0(outputs: dict, plan_shapes: dict, world: int, rank: int, device,
                    dtype) -> dict | None:
    """Gather every rank's per-batch outputs to rank 0.

    ``outputs`` maps this rank's batch indices to tensors; ``plan_shapes`` maps every
    batch index of the plan to its output shape (all ranks know the plan). Each rank sends
    its batches' tensors, flattened in batch order, as one buffer; rank 0 receives the
    buffers of the other ranks and returns {batch index: tensor} for the whole plan. The
    other ranks return None. Collective: every rank must call it.
    """
    import torch
    import torch.distributed as dist

    mine = shard_round_robin(len(plan_shapes), world, rank)
    if sorted(outputs) != mine:
        raise ValueError("outputs must cover exactly this rank's batches")
    if world == 1:
        return dict(outputs)
    if rank != 0:
        flat = (torch.cat([outputs[b].reshape(-1).to(dtype) for b in mine])
                if mine else torch.empty(0, dtype=dtype, device=device))
        dist.send(flat.contiguous(), dst=0)
        return None
    gathered = dict(outputs)
    for src in range(1, world):
        theirs = shard_round_robin(len(plan_shapes), world, src)
        sizes = [int(np.prod(plan_shapes[b])) for b in theirs]
        buf = torch.empty(sum(sizes), dtype=dtype, device=device)
        dist.recv(buf, src=src)
        off = 0
        for b, n in zip(theirs, sizes):
            gathered[b] = buf[off : off + n].reshape(plan_shapes[b])
            off += n
    return gathered
