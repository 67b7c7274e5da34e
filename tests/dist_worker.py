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


def run_rank(rank: int, world: int, port: int, lengths: list, batch_size: int, out_path: str,
             deal: str = "round_robin", fail_rank: int = -1):
    """One rank of the sharded run. ``deal``: "round_robin", "longest_first" (then every
    batch's output is a pair: the weights and their row sums, to exercise multi-tensor
    gathers) or "dynamic" (batches taken from a counter in a TCPStore hosted by rank 0, each
    after a short sleep standing in for the batch's work; rank 0 records every rank's list in
    ``out_path`` + ".deal.json"). ``fail_rank``: that rank raises after its compute, before the gather; rank 0
    then records the error its gather raised in ``out_path`` + ".error"."""
    import torch
    import torch.distributed as dist

    from fast_gpu_asr_b200.sharding import (DynamicDeal, batch_costs, gather_to_rank0,
                                            length_sorted_batches, shard_longest_first,
                                            shard_round_robin)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        plan = length_sorted_batches(np.asarray(lengths), batch_size)
        dynamic = None
        if deal == "longest_first":
            assignment = shard_longest_first(batch_costs(plan), world)
        elif deal == "dynamic":
            store = dist.TCPStore("127.0.0.1", port + 1, world, rank == 0,
                                  timeout=timedelta(seconds=20))
            costs = batch_costs(plan)
            dynamic = DynamicDeal(store, np.argsort(-costs, kind="stable"))
            import time

            # Every rank starts pulling together, and each batch takes a few milliseconds of
            # "work", so no rank can drain the counter before the others begin.
            dist.barrier()
            while (idx := dynamic.next()) is not None:
                time.sleep(0.01 * (1 + idx % 3))
            assignment = dynamic.assignment(world)
            if rank == 0:
                import json

                with open(out_path + ".deal.json", "w") as f:
                    json.dump(assignment, f)
        else:
            assignment = [shard_round_robin(len(plan), world, r) for r in range(world)]
        shapes = {}
        for b in plan:
            n, t = len(b.lengths), b.max_length
            shapes[b.index] = (n, 2, t, t) if deal != "longest_first" else [(n, 2, t, t), (n, 2, t)]
        outputs = {}
        for idx in assignment[rank]:
            w = torch.from_numpy(batch_output(idx, plan[idx].lengths))
            outputs[idx] = w if deal != "longest_first" else [w, w.sum(dim=3)]
        if rank == fail_rank:
            raise RuntimeError(f"rank {rank} fails before the gather (injected)")
        try:
            gathered = gather_to_rank0(outputs, shapes, world, rank, "cpu", torch.float32,
                                       assignment)
        except Exception as e:  # noqa: BLE001 - recorded for the test
            if rank == 0:
                with open(out_path + ".error", "w") as f:
                    f.write(f"{type(e).__name__}: {e}")
            raise
        if rank == 0:
            flat = {}
            for k, v in gathered.items():
                if isinstance(v, list):
                    flat[f"{k}"] = v[0].numpy()
                    flat[f"{k}_sum"] = v[1].numpy()
                else:
                    flat[str(k)] = v.numpy()
            np.savez(out_path, **flat)
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
