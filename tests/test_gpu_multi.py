"""Sequence-sharded decode across GPUs: one process per GPU, the default
peer-memory transport (every shard's top-100 lists written into every
peer's exchange region by the fused kernel, the global merge inside the
kernel, the winners' FP8 records read from the owning GPU) and the NCCL
transport, against the CPU oracle's sharded restatement (global ids
bit-exact, output within tolerance, the same output on every GPU).

Needs two or more GPUs; skipped otherwise.  (Running the shards as separate
launches on ONE GPU is not done: their kernels wait on one another's flags,
and nothing makes separate launches run at the same time.)
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import oracle as O
from seoulkv_b200 import synthetic
from seoulkv_b200.sharded import ShardPlan
from tests.helpers import ShardCase, bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
PER_SHARD = 16384
QSEEDS = (501, 502)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import datetime
    import sys
    import time

    import torch.distributed as dist

    from seoulkv_b200.sharded import ShardedSeoulKV4

    t0 = time.time()
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        total = PER_SHARD * world
        plan = ShardPlan(total, world, rank)
        case = ShardCase(plan)
        t1 = time.time()
        for transport in ("p2p", "nccl"):
            with ShardedSeoulKV4(device=dev, k=case.k, v=case.v, index=case.index, plan=plan,
                                 transport=transport) as sh:
                for qs in QSEEDS:
                    q = synthetic.make_query(total, case.mixes, seed=qs)
                    out = sh.run(q).cpu()
                    gids = sh.selected_ids().cpu()
                    np.save(os.path.join(out_dir, f"{transport}_{qs}_{rank}_out.npy"), bits(out).reshape(16, 256))
                    np.save(os.path.join(out_dir, f"{transport}_{qs}_{rank}_gids.npy"), gids.numpy())
                sh.attn.synchronize()  # every step's status words clear (no timeout, no capacity error)
            dist.barrier()
        print(f"rank {rank}: setup {t1 - t0:.1f} s, steps {time.time() - t1:.1f} s", file=sys.stderr)
    finally:
        dist.destroy_process_group()


def _shard_groups():
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    return [w for w in (2, 3) if w <= n]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2+ GPUs")
def test_sharded_across_gpus_matches_oracle(tmp_path):
    for world in _shard_groups():
        mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
        total = PER_SHARD * world
        cases = [ShardCase(ShardPlan(total, world, r)) for r in range(world)]
        for qs in QSEEDS:
            q = synthetic.make_query(total, cases[0].mixes, seed=qs)
            gids_ref, out_ref, _ = O.sharded_reference([c.reference_view() for c in cases], bits(q).reshape(16, 256))
            for transport in ("p2p", "nccl"):
                outs = [np.load(tmp_path / f"{transport}_{qs}_{r}_out.npy") for r in range(world)]
                gids = [np.load(tmp_path / f"{transport}_{qs}_{r}_gids.npy") for r in range(world)]
                for r in range(world):
                    assert np.array_equal(gids[r], gids_ref), (world, transport, qs, r, "global top-100")
                    assert np.array_equal(outs[r], outs[0]), (world, transport, qs, r, "same output on every GPU")
                err = np.abs(O.bf16_to_f32(outs[0]).astype(np.float64) - O.bf16_to_f32(out_ref).astype(np.float64))
                assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (world, transport, err.max(), err.mean())
