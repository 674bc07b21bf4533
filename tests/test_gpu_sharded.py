"""Sequence-sharded decode on one GPU: N shard engines in one process, the
merge / partial-attention / combine kernels through the C ABI, against the
CPU oracle (global ids bit-exact, BF16 output within tolerance)."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import SeoulKV4, SeoulKV4Config, _native, synthetic
from seoulkv_b200.sharded import PART, ShardedSeoulKV4, ShardPlan, _Dev
from tests.helpers import AppendCase, ShardCase, bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _check_out(got_bits, want_bits):
    err = np.abs(O.bf16_to_f32(got_bits).astype(np.float64) - O.bf16_to_f32(want_bits).astype(np.float64))
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


@pytest.mark.parametrize("n", [2, 3])
def test_sharded_step_matches_oracle(cuda, n):
    total = 8192 * n
    plans = [ShardPlan(total, n, r) for r in range(n)]
    cases = [ShardCase(p) for p in plans]
    q = synthetic.make_query(total, cases[0].mixes, seed=88)
    qb = bits(q).reshape(16, 256)
    gids_ref, out_ref, per_shard = O.sharded_reference([c.reference_view() for c in cases], qb)
    attns = [SeoulKV4(device=cuda, k=c.k, v=c.v, index=c.index, config=SeoulKV4Config(debug=True)) for c in cases]
    try:
        st = torch.cuda.current_stream(cuda).cuda_stream
        for a in attns:
            a.run(q)
        torch.cuda.synchronize(cuda)
        # each shard's local funnel equals the oracle's
        for s, a in enumerate(attns):
            want = np.stack([r["final_ids"] for r in per_shard[s]])
            assert np.array_equal(a.debug_snapshot()["selected_ids"].numpy(), want), f"shard {s} local top-100"
        keys_all = torch.empty(n, 4, 4, 100, dtype=torch.int32, device=cuda)
        ids_all = torch.empty_like(keys_all)
        for s, a in enumerate(attns):
            kp, ip = a._engine.shard_outputs(0)
            keys_all[s].copy_(torch.as_tensor(_Dev(kp, (4, 4, 100), "<i4", st), device=cuda))
            ids_all[s].copy_(torch.as_tensor(_Dev(ip, (4, 4, 100), "<i4", st), device=cuda))
        want_keys = np.stack([np.stack([O.stage2_rank_keys(r) for r in res]) for res in per_shard])
        assert np.array_equal(keys_all.cpu().numpy().view(np.uint32), want_keys), "Stage-II rank keys"
        begin = torch.tensor([p.begin for p in plans], dtype=torch.int32, device=cuda)
        gids = torch.empty(4, 4, 100, dtype=torch.int32, device=cuda)
        _native.shard_merge(keys_all.data_ptr(), ids_all.data_ptr(), begin.data_ptr(), n, 4, gids.data_ptr(), st)
        part = torch.empty(n, 4, 4, PART, dtype=torch.float32, device=cuda)
        for s, a in enumerate(attns):
            a._engine.shard_attention(gids.data_ptr(), plans[s].begin, part[s].data_ptr(), st)
        out = torch.empty(16, 256, dtype=torch.int16, device=cuda)
        _native.shard_combine(part.data_ptr(), n, 4, out.data_ptr(), st)
        torch.cuda.synchronize(cuda)
        assert np.array_equal(gids.cpu().numpy(), gids_ref), "global top-100"
        _check_out(out.cpu().numpy().view(np.uint16), out_ref)
    finally:
        for a in attns:
            a.close()


def test_single_shard_equals_plain_decode(cuda):
    plan = ShardPlan(8192, 1, 0)
    case = ShardCase(plan)
    q = synthetic.make_query(plan.total, case.mixes, seed=5)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=SeoulKV4Config(debug=True)) as plain:
        want = plain.run(q).to_torch()
        want_ids = plain.debug_snapshot()["selected_ids"]
    with ShardedSeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, plan=plan) as sh:
        got = sh.run(q).cpu()
        gids = sh.selected_ids().cpu()
    assert torch.equal(gids.long(), want_ids)
    _check_out(bits(got).reshape(16, 256), bits(want).reshape(16, 256))


def test_single_shard_group_over_peer_memory(cuda):
    """The in-kernel exchange path (a one-shard group maps only itself) equals the plain decode."""
    plan = ShardPlan(8192, 1, 0)
    case = ShardCase(plan)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=SeoulKV4Config(debug=True)) as plain:
        outs, ids = [], []
        for s in (11, 12, 13):
            q = synthetic.make_query(plan.total, case.mixes, seed=s)
            outs.append(plain.run(q).to_torch())
            ids.append(plain.debug_snapshot()["selected_ids"])
    with ShardedSeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, plan=plan, transport="p2p") as sh:
        assert sh.attn._engine.fused
        for i, s in enumerate((11, 12, 13)):  # several steps: the per-step flags advance
            q = synthetic.make_query(plan.total, case.mixes, seed=s)
            got = sh.run(q).cpu()
            assert torch.equal(sh.selected_ids().cpu().long(), ids[i])
            _check_out(bits(got).reshape(16, 256), bits(outs[i]).reshape(16, 256))
        sh.attn.synchronize()  # status: no exchange timed out


def test_merge_rejects_bad_shapes(cuda):
    x = torch.zeros(11, 4, 4, 100, dtype=torch.int32, device=cuda)
    g = torch.zeros(4, 4, 100, dtype=torch.int32, device=cuda)
    b = torch.zeros(11, dtype=torch.int32, device=cuda)
    with pytest.raises(_native.NativeError):
        _native.shard_merge(x.data_ptr(), x.data_ptr(), b.data_ptr(), 11, 4, g.data_ptr())
    with pytest.raises(_native.NativeError):
        _native.shard_merge(x.data_ptr(), x.data_ptr(), b.data_ptr(), 2, 3, g.data_ptr())


def _grown_layer(n, total, m, seed=31):
    """An n-shard layer of `total` tokens whose last shard will grow by m:
    every shard's slice of one (total + m)-token sequence, as AppendCases."""
    plans = [ShardPlan(total, n, r) for r in range(n)]
    grown = total + m
    cases = []
    for p in plans:
        last = p.shard == n - 1
        end = grown if last else p.end
        kv = synthetic.make_kv_range(grown, p.begin, end, seed=seed, components=64)
        cases.append(AppendCase(context=p.context, total=end - p.begin, nprobe=128, sink=p.shard_sink,
                                local=p.shard_local, kv=kv))
    return plans, cases


def test_sharded_append_matches_oracle(cuda):
    """Two shards decoded through the merge / attention / combine kernels after
    the last shard (which holds the local window) grew by 300 tokens."""
    n, total, m = 2, 16384, 300
    plans, cases = _grown_layer(n, total, m)
    last = cases[-1]
    cfgs = [SeoulKV4Config(debug=True, max_context=(p.context + m) if p.shard == n - 1 else None) for p in plans]
    attns = [SeoulKV4(device=cuda, k=c.k, v=c.v, index=c.index, config=cf) for c, cf in zip(cases, cfgs)]
    try:
        attns[-1].append(*last.appended(last.context, last.total))
        views = [c.reference_view(c.total, p.begin) for c, p in zip(cases, plans)]
        q = synthetic.make_query(total + m, last.mixes, seed=91)
        qb = bits(q).reshape(16, 256)
        gids_ref, out_ref, _ = O.sharded_reference(views, qb)
        st = torch.cuda.current_stream(cuda).cuda_stream
        for a in attns:
            a.run(q)
        keys_all = torch.empty(n, 4, 4, 100, dtype=torch.int32, device=cuda)
        ids_all = torch.empty_like(keys_all)
        for s, a in enumerate(attns):
            kp, ip = a._engine.shard_outputs(0)
            keys_all[s].copy_(torch.as_tensor(_Dev(kp, (4, 4, 100), "<i4", st), device=cuda))
            ids_all[s].copy_(torch.as_tensor(_Dev(ip, (4, 4, 100), "<i4", st), device=cuda))
        begin = torch.tensor([p.begin for p in plans], dtype=torch.int32, device=cuda)
        gids = torch.empty(4, 4, 100, dtype=torch.int32, device=cuda)
        _native.shard_merge(keys_all.data_ptr(), ids_all.data_ptr(), begin.data_ptr(), n, 4, gids.data_ptr(), st)
        part = torch.empty(n, 4, 4, PART, dtype=torch.float32, device=cuda)
        for s, a in enumerate(attns):
            a._engine.shard_attention(gids.data_ptr(), plans[s].begin, part[s].data_ptr(), st)
        out = torch.empty(16, 256, dtype=torch.int16, device=cuda)
        _native.shard_combine(part.data_ptr(), n, 4, out.data_ptr(), st)
        torch.cuda.synchronize(cuda)
        assert np.array_equal(gids.cpu().numpy(), gids_ref), "global top-100 after the append"
        _check_out(out.cpu().numpy().view(np.uint16), out_ref)
    finally:
        for a in attns:
            a.close()


def test_single_shard_group_append_over_peer_memory(cuda):
    """A one-shard peer-memory group grown by appends decodes as a plain
    instance grown by the same tokens (the group's length grows on the device)."""
    m = 300
    plans, cases = _grown_layer(1, 8192, m, seed=33)
    plan, c = plans[0], cases[0]
    k1, v1 = c.appended(8192, 8192 + 7)
    k2, v2 = c.appended(8192 + 7, 8192 + m)
    with SeoulKV4(device=cuda, k=c.k, v=c.v, index=c.index,
                  config=SeoulKV4Config(debug=True, max_context=8192 + m)) as plain:
        plain.append(k1, v1)
        plain.append(k2, v2)
        q = synthetic.make_query(8192 + m, c.mixes, seed=14)
        want = plain.run(q).to_torch()
        want_ids = plain.debug_snapshot()["selected_ids"]
    with ShardedSeoulKV4(device=cuda, k=c.k, v=c.v, index=c.index, plan=plan, transport="p2p", grow=m,
                         config=SeoulKV4Config(debug=True)) as sh:
        sh.append(k1, v1)
        sh.append(k2.cuda(), v2.cuda())
        assert sh.total == 8192 + m
        got = sh.run(q).cpu()
        assert torch.equal(sh.selected_ids().cpu().long(), want_ids)
        _check_out(bits(got).reshape(16, 256), bits(want).reshape(16, 256))
        with pytest.raises(ValueError, match="room to grow"):
            sh.append(k1[:, :1], v1[:, :1])
        sh.attn.synchronize()
