"""Sequence sharding on the CPU: shard plans, the range generator, the merge
rule, and the all-gather plumbing across two gloo ranks."""

import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from seoulkv_b200 import synthetic
from seoulkv_b200.sharded import Exchange, ShardPlan
from tests.helpers import ShardCase


def test_shard_plan_covers_the_context():
    for total, n in ((1 << 20, 8), (100_003, 3), (65536, 1)):
        plans = [ShardPlan(total, n, r) for r in range(n)]
        assert plans[0].begin == 0 and plans[-1].end == total
        assert all(a.end == b.begin for a, b in zip(plans, plans[1:]))
        assert plans[0].shard_sink == 128 and plans[-1].shard_local == 256
        assert all(p.shard_sink == 0 for p in plans[1:]) and all(p.shard_local == 0 for p in plans[:-1])
    with pytest.raises(ValueError):
        ShardPlan(1024, 2, 2)
    with pytest.raises(ValueError):
        ShardPlan(300, 2, 1, local=256)  # the local window does not fit the last shard


def test_range_generator_slices_agree():
    k, v, _ = synthetic.make_kv_range(150_000, 0, 150_000, seed=9, components=8, block=32768)
    k2, v2, _ = synthetic.make_kv_range(150_000, 40_000, 100_000, seed=9, components=8, block=32768)
    assert torch.equal(k[:, 40_000:100_000], k2) and torch.equal(v[:, 40_000:100_000], v2)


def test_merge_rule_orders_by_score_rank_then_id():
    keys = np.zeros((2, 4, 4, 100), np.uint32)
    ids = np.zeros((2, 4, 4, 100), np.int32)
    # shard 0 rank 0 and shard 1 rank 0 tie on the score: the lower global id wins
    keys[0, 0, 0, 0] = (0x9000 << 16) | 7
    ids[0, 0, 0, 0] = 50
    keys[1, 0, 0, 0] = (0x9000 << 16) | 9
    ids[1, 0, 0, 0] = 3
    keys[0, 0, 0, 1] = (0x9100 << 16) | 1  # higher score, later rank
    ids[0, 0, 0, 1] = 60
    g = O.merge_shards(keys, ids, [0, 1000])
    assert list(g[0, 0, :3]) == [60, 50, 1003]
    assert g[0, 0, 3] == -1 and (g[1:] == -1).all()


def _worker(rank, world, port, total, q_bits, out_path):
    import sys

    sys.path.insert(0, str(__import__("pathlib").Path(__file__).resolve().parents[1]))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(max(1, (os.cpu_count() or 2) // world))  # ranks share the cores
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ShardPlan(total, world, rank)
        cells = ShardCase(plan).cells()
        res = [O.run_cell(cells[g], q_bits[4 * g:4 * g + 4]) for g in range(4)]
        keys = torch.from_numpy(np.stack([O.stage2_rank_keys(r) for r in res]).view(np.int32))
        ids = torch.from_numpy(np.stack([r["final_ids"] for r in res]).astype(np.int32))
        ex = Exchange()
        assert (ex.size, ex.rank) == (world, rank)
        keys_all = torch.empty(world, 4, 4, 100, dtype=torch.int32)
        ids_all = torch.empty_like(keys_all)
        ex.gather(keys_all, keys)
        ex.gather(ids_all, ids)
        begin = [ShardPlan(total, world, r).begin for r in range(world)]
        gids = O.merge_shards(keys_all.numpy().view(np.uint32), ids_all.numpy(), begin)
        np.save(out_path.format(rank), gids)
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_agree_with_one_process(tmp_path):
    total, world = 16384, 2
    q = synthetic.make_query(total, synthetic.make_kv_range(total, 0, 1, seed=31, components=64)[2], seed=77)
    q_bits = q.reshape(16, 256).contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    port = 29500 + os.getpid() % 1000
    out = str(tmp_path / "gids_{}.npy")
    mp.start_processes(_worker, args=(world, port, total, q_bits, out), nprocs=world, start_method="spawn")
    got = [np.load(out.format(r)) for r in range(world)]
    assert np.array_equal(got[0], got[1]), "every rank merges the same global top-100"
    # the same step in one process
    shards = []
    for r in range(world):
        plan = ShardPlan(total, world, r)
        shards.append(dict(cells=ShardCase(plan).cells(), begin=plan.begin))
    keys = np.zeros((world, 4, 4, 100), np.uint32)
    ids = np.zeros((world, 4, 4, 100), np.int32)
    for s, sh in enumerate(shards):
        for g in range(4):
            res = O.run_cell(sh["cells"][g], q_bits[4 * g:4 * g + 4])
            keys[s, g] = O.stage2_rank_keys(res)
            ids[s, g] = res["final_ids"]
    want = O.merge_shards(keys, ids, [sh["begin"] for sh in shards])
    assert np.array_equal(got[0], want)
    assert (want >= 0).all() and want.max() < total


def test_sharded_grow_validation():
    """ShardedSeoulKV4 rejects a bad growth allowance and mismatched zones
    before it touches a device."""
    from seoulkv_b200.sharded import ShardedSeoulKV4

    plan = ShardPlan(8192, 1, 0)
    case = ShardCase(plan)
    for bad in (-1, 1.5, True):
        with pytest.raises(ValueError, match="grow"):
            ShardedSeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index, plan=plan, grow=bad)
    with pytest.raises(ValueError, match="zones"):
        ShardedSeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index, plan=ShardPlan(8192, 1, 0, local=128))
