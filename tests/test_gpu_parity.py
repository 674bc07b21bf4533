"""CUDA engine vs the CPU oracle, stage by stage (bit-exact) and output (tolerance)."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import SeoulKV4, SeoulKV4Config, _native
from tests.helpers import Case, bits

pytestmark = pytest.mark.gpu

# north_star tolerance for the BF16 attention output
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


@pytest.fixture(scope="module")
def case():
    return Case(context=8192, nprobe=128, seed=11)


@pytest.fixture(params=["fused", "staged"])
def path(request, monkeypatch):
    """Both device paths: the single cluster kernel and the 14 staged kernels."""
    monkeypatch.setattr(_native, "FORCE_STAGED", request.param == "staged")
    return request.param


def _compare(eng, res, nc, capacity):
    counts = eng.read_stage(0, "counts", np.int32, (4, 8))
    lohi = eng.read_stage(0, "lohi", np.uint16, (4, 2, 4, nc))
    thresh = eng.read_stage(0, "thresh", np.uint16, (4, 4))
    tags = eng.read_stage(0, "tags", np.uint32, (4, nc))
    sel = eng.read_stage(0, "selected", np.int32, (4, 2048))
    pool = eng.read_stage(0, "pool", np.int32, (4, capacity))
    u15 = eng.read_stage(0, "u15", np.int32, (4, 6400))
    cand = eng.read_stage(0, "cand", np.int32, (4, 1024))
    fpos = eng.read_stage(0, "final_pos", np.int32, (4, 4, 100))
    for g, r in enumerate(res):
        assert np.array_equal(lohi[g, 0], r["lo"]), f"cell {g}: coarse lower bounds"
        assert np.array_equal(lohi[g, 1], r["hi"]), f"cell {g}: coarse upper bounds"
        assert np.array_equal(thresh[g], r["thresh"]), f"cell {g}: coarse thresholds"
        n = counts[g, 0]
        assert n == len(r["tags"]) and np.array_equal(tags[g, :n], r["tags"]), f"cell {g}: survivors"
        n = counts[g, 1]
        assert n == len(r["selected"]) and np.array_equal(sel[g, :n], r["selected"]), f"cell {g}: fine union"
        n = counts[g, 2]
        assert n == len(r["pool"]) and np.array_equal(pool[g, :n], r["pool"]), f"cell {g}: pool"
        n = counts[g, 3]
        assert n == len(r["u15"]) and np.array_equal(u15[g, :n], r["u15"]), f"cell {g}: stage-1.5 union"
        n = counts[g, 4]
        assert n == len(r["cand"]) and np.array_equal(cand[g, :n], r["cand"]), f"cell {g}: stage-1.6 union"
        assert np.array_equal(fpos[g], r["final_pos"]), f"cell {g}: stage-II ranks"
        assert counts[g, 5] == 0, f"cell {g}: status"


def test_funnel_parity_and_output(case, cuda, path):
    cfg = SeoulKV4Config(debug=True, trace_stages=True)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=cfg) as attn:
        attn.run(case.query(100))
        assert attn._engine.fused == (path == "fused")
        for qseed in (101, 102, 103):
            q = case.query(qseed)
            y = attn.run(q).to_torch()
            res, ref_out = case.oracle(q)
            eng = attn._engine
            _compare(eng, res, case.index.cells()[0]["centroids"].shape[0], 13056)
            ids = attn.debug_snapshot()["selected_ids"].numpy()
            want = np.stack([r["final_ids"] for r in res])
            assert np.array_equal(ids, want), "selected token ids"
            got = O.bf16_to_f32(bits(y).reshape(16, 256)).astype(np.float64)
            ref = O.bf16_to_f32(ref_out).astype(np.float64)
            err = np.abs(got - ref)
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


def test_device_query_and_replay(case, cuda, path):
    q = case.query(201)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=SeoulKV4Config(debug=True)) as attn:
        a = attn.run(q).to_torch()
        b = attn.run(q.to(cuda)).to_torch()
        assert torch.equal(a, b)
        ids1 = attn.debug_snapshot()["selected_ids"]
        attn.run(case.query(202))
        attn.run(q)
        assert torch.equal(attn.debug_snapshot()["selected_ids"], ids1)


@pytest.mark.parametrize("context,nprobe,capacity,staged", [
    (6400, 256, 13056, False),                    # the smallest context the profile accepts
    (16384, (128, 192, 256, 512), 13056, False),  # a different nprobe per KV head
    (32768, 512, 15360, False),                   # the largest nprobe, a larger Stage-1.5 capacity
    (32768, 512, 15360, True),
], ids=["6400-256", "16384-perhead", "32768-512-fused", "32768-512-staged"])
def test_parity_sweep(cuda, monkeypatch, context, nprobe, capacity, staged):
    """Every stage bit-exact and the output within tolerance across contexts,
    per-head nprobe and capacities."""
    monkeypatch.setattr(_native, "FORCE_STAGED", staged)
    case = Case(context=context, nprobe=64, seed=61)
    cfg = SeoulKV4Config(debug=True, nprobe=nprobe, stage15_capacity=capacity, trace_stages=True)
    per_head = [nprobe] * 4 if isinstance(nprobe, int) else list(nprobe)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=cfg) as attn:
        for qseed in (1, 2):
            q = case.query(qseed)
            y = attn.run(q).to_torch()
            assert attn._engine.fused == (not staged)
            res, ref_out = case.oracle(q, capacity=capacity, nprobe=per_head)
            _compare(attn._engine, res, case.index.cells()[0]["centroids"].shape[0], capacity)
            ids = attn.debug_snapshot()["selected_ids"].numpy()
            assert np.array_equal(ids, np.stack([r["final_ids"] for r in res])), "selected token ids"
            got = O.bf16_to_f32(bits(y).reshape(16, 256)).astype(np.float64)
            err = np.abs(got - O.bf16_to_f32(ref_out).astype(np.float64))
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


@pytest.mark.parametrize("staged", [False, True], ids=["fused", "staged"])
def test_large_attention_zones(cuda, monkeypatch, staged):
    """A sink of 512 and a local window of 8192 keys: more dense keys than a
    warp folds in one pass (8,704 keys over 256 warps)."""
    monkeypatch.setattr(_native, "FORCE_STAGED", staged)
    case = Case(context=32768, nprobe=384, seed=71, sink=512, local=8192)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=SeoulKV4Config(debug=True)) as attn:
        q = case.query(3)
        y = attn.run(q).to_torch()
        res, ref_out = case.oracle(q)
        ids = attn.debug_snapshot()["selected_ids"].numpy()
        assert np.array_equal(ids, np.stack([r["final_ids"] for r in res])), "selected token ids"
        got = O.bf16_to_f32(bits(y).reshape(16, 256)).astype(np.float64)
        err = np.abs(got - O.bf16_to_f32(ref_out).astype(np.float64))
        assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


@pytest.fixture(scope="module")
def headline():
    """T=131072, nprobe 384, sink 128, local 256."""
    return Case(context=131072, nprobe=384, seed=1000)


@pytest.mark.parametrize("staged", [False, True], ids=["fused", "staged"])
def test_headline_config_parity(cuda, monkeypatch, headline, staged):
    """The benchmarked configuration itself: every stage bit-exact, ids
    bit-exact and the output within tolerance, on three fresh queries."""
    monkeypatch.setattr(_native, "FORCE_STAGED", staged)
    case = headline
    nc = case.index.cells()[0]["centroids"].shape[0]
    cfg = SeoulKV4Config(debug=True, trace_stages=True)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=cfg) as attn:
        for qseed in (1000 * 7919 + 3, 1000 * 7919 + 4, 1000 * 7919 + 5):
            q = case.query(qseed)
            y = attn.run(q).to_torch()
            assert attn._engine.fused == (not staged)
            res, ref_out = case.oracle(q)
            _compare(attn._engine, res, nc, 13056)
            ids = attn.debug_snapshot()["selected_ids"].numpy()
            assert np.array_equal(ids, np.stack([r["final_ids"] for r in res])), "selected token ids"
            got = O.bf16_to_f32(bits(y).reshape(16, 256)).astype(np.float64)
            err = np.abs(got - O.bf16_to_f32(ref_out).astype(np.float64))
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


def test_l2_window_changes_nothing(cuda, headline):
    """The centroid planes held in persisting L2 give the same bits as without
    the window (and the window really is set on a B200)."""
    case = headline
    nc = case.index.cells()[0]["centroids"].shape[0]
    outs = []
    for resident in (True, False):
        cfg = SeoulKV4Config(debug=True, l2_resident=resident)
        with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=cfg) as attn:
            got = []
            for qseed in (11, 12):
                y = attn.run(case.query(qseed)).to_torch()
                got.append((bits(y), attn.debug_snapshot()["selected_ids"].numpy()))
            meta = attn.metadata()
            if resident:
                assert meta["l2_resident_bytes"] == 4 * nc * 128, meta["l2_resident_bytes"]
            else:
                assert meta["l2_resident_bytes"] == 0
            outs.append(got)
    for (ya, ia), (yb, ib) in zip(*outs):
        assert np.array_equal(ya, yb) and np.array_equal(ia, ib)


def test_above_the_fused_limit(cuda):
    """T = 262,144 (nc = 65,440 > 32,768): the staged kernels carry it; every
    stage bit-exact against the oracle."""
    case = Case(context=262144, nprobe=384, seed=62)
    nc = case.index.cells()[0]["centroids"].shape[0]
    assert nc > 32768
    cfg = SeoulKV4Config(debug=True, trace_stages=True)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=cfg) as attn:
        for qseed in (1, 2):
            q = case.query(qseed)
            y = attn.run(q).to_torch()
            res, ref_out = case.oracle(q)
            _compare(attn._engine, res, nc, 13056)
            ids = attn.debug_snapshot()["selected_ids"].numpy()
            assert np.array_equal(ids, np.stack([r["final_ids"] for r in res])), "selected token ids"
            got = O.bf16_to_f32(bits(y).reshape(16, 256)).astype(np.float64)
            err = np.abs(got - O.bf16_to_f32(ref_out).astype(np.float64))
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())
