"""Host logic of the multi-GPU path: the length-balanced record partition,
its agreement across ranks (world_size-2 gloo on the CPU), the host-side
reductions, and the gather of per-device outputs into the caller's order."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from fast_forced_aligner_b200.alignment import AlignmentBatch
from fast_forced_aligner_b200.sharding import (Shard, ShardedAlignment, partition_records,
                                               record_costs, reduce_over_ranks, shard_of_rank)


def _cfg4_like_lengths(count=8256, seed=7):
    """Lengths with the multi-GPU configuration's shape (lognormal, median 600)."""
    rng = np.random.default_rng(seed)
    T = np.clip(np.round(rng.lognormal(np.log(600.0), 0.6, count)), 50, 6000).astype(np.int64)
    return T, (0.3 * T).astype(np.int64)


@pytest.mark.parametrize("shards", [1, 2, 3, 4, 8])
def test_partition_is_a_balanced_cover(shards):
    T, U = _cfg4_like_lengths()
    costs = record_costs(T, U)
    parts = partition_records(costs, shards)
    assert len(parts) == shards
    allx = np.concatenate(parts)
    assert np.array_equal(np.sort(allx), np.arange(T.size))  # disjoint and complete
    for p in parts:
        assert np.all(np.diff(p) > 0)
    loads = np.array([costs[p].sum() for p in parts])
    # LPT bound: the heaviest bin exceeds the mean by at most one record.
    assert loads.max() <= costs.sum() / shards + costs.max()
    if shards > 1:
        assert loads.max() / loads.mean() < 1.01


def test_partition_edge_cases():
    assert [p.tolist() for p in partition_records([5], 3)] == [[0], [], []]
    assert [p.tolist() for p in partition_records([], 2)] == [[], []]
    # Equal costs: deterministic round-robin by index.
    assert [p.tolist() for p in partition_records([1, 1, 1, 1], 2)] == [[0, 2], [1, 3]]
    # Decreasing cost, each to the lightest bin: 7->b0, 5->b1, 4->b1 (9),
    # 3->b0 (10), 2->b1 (11).
    parts = partition_records([3, 7, 5, 4, 2], 2)
    assert [p.tolist() for p in parts] == [[0, 1], [2, 3, 4]]
    with pytest.raises(ValueError):
        partition_records([1], 0)
    with pytest.raises(ValueError):
        record_costs([1, 2], [1])
    with pytest.raises(ValueError):
        shard_of_rank([1], [0], 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, U = _cfg4_like_lengths()
        mine = shard_of_rank(T.tolist(), U.tolist(), rank, world)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine.tolist())
        mx = reduce_over_ranks(float(rank + 1), "max")
        sm = reduce_over_ranks(float(len(mine)), "sum")
        np.save(os.path.join(out_dir, f"rank{rank}.npy"),
                np.array([mx, sm] + [len(g) for g in gathered], dtype=np.float64))
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            for g in gathered:
                f.write(",".join(map(str, g)) + "\n")
    finally:
        dist.destroy_process_group()


def test_ranks_agree_on_partition_over_gloo(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    texts = [(tmp_path / f"rank{r}.txt").read_text() for r in range(world)]
    assert texts[0] == texts[1]  # every rank computed the same partition
    parts = [np.array([int(x) for x in line.split(",") if x]) for line in texts[0].splitlines()]
    T, U = _cfg4_like_lengths()
    assert np.array_equal(np.sort(np.concatenate(parts)), np.arange(T.size))
    expect = partition_records(record_costs(T, U), world)
    for p, e in zip(parts, expect):
        assert np.array_equal(p, e)
    for r in range(world):
        mx, sm = np.load(tmp_path / f"rank{r}.npy")[:2]
        assert mx == world and sm == T.size


def test_reduce_without_process_group_is_identity():
    assert reduce_over_ranks(3.5, "max") == 3.5
    assert reduce_over_ranks(2.0, "sum") == 2.0


def _fake_batch(lengths, base, reuse):
    """A CPU AlignmentBatch whose every field encodes the record it belongs to."""
    B = len(lengths)
    rec = torch.tensor(base, dtype=torch.int64)
    labels = torch.cat([torch.full((n,), int(r), dtype=torch.int64) for n, r in zip(lengths, base)])
    return AlignmentBatch(
        tuple(lengths), labels, labels.float() * 0.5, rec.int(), rec.float(), rec.int() % 2,
        rec.int() % 3, rec * 10, rec[:, None].repeat(1, 3), rec.int()[:, None].repeat(1, 3),
        rec[:, None].repeat(1, 4) if reuse else torch.zeros((0, 4), dtype=torch.int64))


@pytest.mark.parametrize("reuse", [False, True])
def test_gather_restores_caller_order(reuse):
    lengths = (3, 1, 4, 2, 5)
    shards_ix = [np.array([1, 3]), np.array([0, 2, 4])]
    shards = tuple(
        Shard(torch.device("cpu"), ix, _fake_batch([lengths[i] for i in ix], ix.tolist(),
                                                   reuse and k == 1))
        for k, ix in enumerate(shards_ix))
    result = ShardedAlignment(len(lengths), lengths, shards)
    g = result.gather("cpu")
    want = torch.cat([torch.full((n,), r, dtype=torch.int64) for r, n in enumerate(lengths)])
    assert torch.equal(g.labels, want)
    assert torch.equal(g.scores, want.float() * 0.5)
    assert g.status.tolist() == list(range(5))
    assert g.objective.tolist() == [0.0, 1.0, 2.0, 3.0, 4.0]
    assert g.repaired_frames.tolist() == [0, 10, 20, 30, 40]
    assert g.shortcut_stats[:, 2].tolist() == list(range(5))
    if reuse:  # rows of shards without reuse statistics are zero
        assert g.reuse_stats[:, 0].tolist() == [0, 0, 2, 0, 4]
    else:
        assert g.reuse_stats.shape == (0, 4)
    assert result.status().tolist() == list(range(5))
    assert [p.tolist() for p in result.paths()] == [[r] * n for r, n in enumerate(lengths)]
    with pytest.raises(ValueError, match=r"batch indices \[1\]"):
        result.raise_for_status()  # status 1 at record 1 (failed path)
