"""Batch sharding and the final gather (host logic; gloo world-size 2 and 3 on CPU)."""

from __future__ import annotations

import socket

import numpy as np
import pytest

from fast_gpu_asr_b200.sharding import (batch_costs, length_sorted_batches,
                                        shard_longest_first, shard_round_robin)
from fast_gpu_asr_b200.workloads import ragged_durations


def test_length_sorted_batches_cover_every_utterance_once():
    lengths = np.random.default_rng(0).integers(1, 500, size=1037)
    plan = length_sorted_batches(lengths, 256)
    assert [len(b.utterances) for b in plan] == [256, 256, 256, 256, 13]
    ids = np.concatenate([b.utterances for b in plan])
    assert sorted(ids.tolist()) == list(range(1037))
    flat = np.concatenate([b.lengths for b in plan])
    assert (np.diff(flat) <= 0).all()  # longest first, across batch boundaries
    assert all((lengths[b.utterances] == b.lengths).all() for b in plan)


def test_length_sorted_batches_is_stable_and_validates():
    plan = length_sorted_batches([5, 7, 5, 7], 3)
    assert plan[0].utterances.tolist() == [1, 3, 0] and plan[1].utterances.tolist() == [2]
    with pytest.raises(ValueError):
        length_sorted_batches([[1, 2]], 2)
    with pytest.raises(ValueError):
        length_sorted_batches([1, 2], 0)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_round_robin_partitions_the_plan(world):
    n = 79  # 20,000 utterances in batches of 256
    shards = [shard_round_robin(n, world, r) for r in range(world)]
    flat = sorted(b for s in shards for b in s)
    assert flat == list(range(n))
    assert max(map(len, shards)) - min(map(len, shards)) <= 1
    with pytest.raises(ValueError):
        shard_round_robin(n, world, world)


def test_ragged_box_plan_matches_the_configuration():
    durations = ragged_durations()
    assert durations.shape == (20000,) and durations.min() >= 1.0 and durations.max() <= 35.0
    assert abs(durations.mean() - 8.0) < 0.3
    assert len(length_sorted_batches(durations, 256)) == 79


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,count,batch", [(2, 23, 4), (3, 5, 4)])
def test_gather_to_rank0_equals_single_process(tmp_path, world, count, batch):
    import torch.multiprocessing as mp

    import dist_worker

    lengths = np.random.default_rng(world).integers(3, 12, size=count).tolist()
    out = tmp_path / "gathered.npz"
    mp.start_processes(dist_worker.run_rank, args=(world, _free_port(), lengths, batch, str(out)),
                       nprocs=world, join=True, start_method="spawn")
    got = np.load(out)
    plan = length_sorted_batches(np.asarray(lengths), batch)
    assert sorted(int(k) for k in got.files) == [b.index for b in plan]
    for b in plan:
        np.testing.assert_array_equal(got[str(b.index)], dist_worker.batch_output(b.index, b.lengths))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_longest_first_deal_balances_the_ragged_plan(world):
    """On the ragged plan, the greedy deal keeps every rank within one batch's cost of the
    others, and its slowest rank is no slower than round-robin's."""
    plan = length_sorted_batches(ragged_durations(), 256)
    costs = batch_costs(plan)
    shards = shard_longest_first(costs, world)
    assert sorted(b for s in shards for b in s) == list(range(len(plan)))
    loads = [costs[s].sum() for s in shards]
    assert max(loads) - min(loads) <= costs.max()
    rr = [costs[shard_round_robin(len(plan), world, r)].sum() for r in range(world)]
    assert max(loads) <= max(rr)
    # Within 3 % of a perfect split, unless one batch alone is more than a rank's share.
    assert max(loads) <= max(1.03 * costs.sum() / world, costs.max())
    assert shard_longest_first(costs, world) == shards  # deterministic


@pytest.mark.parametrize("world,count,batch", [(2, 23, 4), (3, 14, 3)])
def test_gather_with_longest_first_deal_and_tensor_lists(tmp_path, world, count, batch):
    import torch.multiprocessing as mp

    import dist_worker

    lengths = np.random.default_rng(10 + world).integers(3, 12, size=count).tolist()
    out = tmp_path / "gathered.npz"
    mp.start_processes(dist_worker.run_rank,
                       args=(world, _free_port(), lengths, batch, str(out), "longest_first"),
                       nprocs=world, join=True, start_method="spawn")
    got = np.load(out)
    plan = length_sorted_batches(np.asarray(lengths), batch)
    for b in plan:
        w = dist_worker.batch_output(b.index, b.lengths)
        np.testing.assert_array_equal(got[str(b.index)], w)
        np.testing.assert_allclose(got[f"{b.index}_sum"], w.sum(axis=3), rtol=1e-6)


@pytest.mark.parametrize("world,count,batch", [(2, 31, 3), (3, 20, 2)])
def test_dynamic_deal_takes_every_batch_once_and_gathers(tmp_path, world, count, batch):
    """Ranks pull batches from a shared counter (longest first): every batch is taken by
    exactly one rank, every rank takes some, and the gather over that assignment equals the
    single-process result."""
    import json

    import torch.multiprocessing as mp

    import dist_worker

    lengths = np.random.default_rng(20 + world).integers(3, 12, size=count).tolist()
    out = tmp_path / "gathered.npz"
    mp.start_processes(dist_worker.run_rank,
                       args=(world, _free_port(), lengths, batch, str(out), "dynamic"),
                       nprocs=world, join=True, start_method="spawn")
    plan = length_sorted_batches(np.asarray(lengths), batch)
    assignment = json.loads((tmp_path / "gathered.npz.deal.json").read_text())
    taken = sorted(b for r in assignment for b in r)
    assert taken == list(range(len(plan)))
    assert all(len(r) > 0 for r in assignment)
    got = np.load(out)
    for b in plan:
        np.testing.assert_array_equal(got[str(b.index)], dist_worker.batch_output(b.index, b.lengths))


def test_dynamic_deal_in_one_process():
    """The counter hands out the order once, then None; with one rank it takes all."""
    from torch.distributed import HashStore

    from fast_gpu_asr_b200.sharding import DynamicDeal

    deal = DynamicDeal(HashStore(), [3, 0, 2, 1])
    assert [deal.next() for _ in range(6)] == [3, 0, 2, 1, None, None]
    assert deal.assignment(1) == [[0, 1, 2, 3]]


def test_rank_failing_before_the_gather_is_reported_not_hung(tmp_path):
    """A rank that raises after its compute, before its send: rank 0's gather fails with an
    error well within the process group's timeout (no hang), and it records the error."""
    import time

    import torch.multiprocessing as mp

    import dist_worker

    lengths = np.random.default_rng(3).integers(3, 12, size=12).tolist()
    out = tmp_path / "gathered.npz"
    ctx = mp.start_processes(dist_worker.run_rank,
                             args=(2, _free_port(), lengths, 3, str(out), "round_robin", 1),
                             nprocs=2, join=False, start_method="spawn")
    t0 = time.monotonic()
    for proc in ctx.processes:
        proc.join(timeout=90)
    elapsed = time.monotonic() - t0
    assert all(not p.is_alive() for p in ctx.processes)
    assert all(p.exitcode != 0 for p in ctx.processes)
    assert elapsed < 60, elapsed
    assert not out.exists()
    err = (tmp_path / "gathered.npz.error").read_text()
    assert err  # the receive from the failed rank raised on rank 0
