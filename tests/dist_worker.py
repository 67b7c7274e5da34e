"""Worker for the multi-process sharding tests (gloo on CPU; imported by spawned ranks).

Each rank runs the length-sorted plan's batches assigned to it round-robin, computing
every batch with the CPU oracle on small seeded inputs (the kernels themselves need a
GPU), and the per-batch outputs are gathered to rank 0, which saves them for the test.
"""

from __future__ import annotations

import os
from datetime import timedelta

import numpy as np


def batch_inputs(batch_index: int, batch_lengths: np.ndarray, heads: int = 2, qd: int = 4):
    """Seeded Zipformer-weights inputs for one batch, padded to its longest utterance."""
    rng = np.random.default_rng(1000 + batch_index)
    n, t = len(batch_lengths), int(batch_lengths.max())
    projection = rng.normal(0.0, 0.5, (n, t, heads * (2 * qd + 4))).astype(np.float32)
    position = rng.normal(0.0, 0.5, (1, 2 * t - 1, heads, 4)).astype(np.float32)
    mask = np.arange(t)[None, :] >= np.asarray(batch_lengths)[:, None]
    return projection, position, mask


def batch_output(batch_index: int, batch_lengths: np.ndarray) -> np.ndarray:
    from oracle import zipformer_relative_attention

    return zipformer_relative_attention(*batch_inputs(batch_index, batch_lengths))


def run_rank(rank: int, world: int, port: int, lengths: list, batch_size: int, out_path: str):
    import torch
    import torch.distributed as dist

    from fast_gpu_asr_b200.sharding import gather_to_rank0, length_sorted_batches, shard_round_robin

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        plan = length_sorted_batches(np.asarray(lengths), batch_size)
        shapes = {}
        for b in plan:
            n, t = len(b.lengths), b.max_length
            shapes[b.index] = (n, 2, t, t)
        outputs = {}
        for idx in shard_round_robin(len(plan), world, rank):
            outputs[idx] = torch.from_numpy(batch_output(idx, plan[idx].lengths))
        gathered = gather_to_rank0(outputs, shapes, world, rank, "cpu", torch.float32)
        if rank == 0:
            np.savez(out_path, **{str(k): v.numpy() for k, v in gathered.items()})
    finally:
        dist.destroy_process_group()
