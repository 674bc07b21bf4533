"""CUDA engine through the C ABI: reference-built index, codec planes, batching, errors."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import _native
from seoulkv_b200.index import device_view
from tests.helpers import GOLDEN_FILES, Case, Golden, bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _engine(n_slots, context, nc, capacity=13056, sink=128, local=256, staged=None):
    return _native.Engine(n_slots=n_slots, context=context, sink=sink, local=local, nc=nc,
                          capacity=capacity, device=0, staged=staged)


def _upload_kv(eng, slot, k, v):
    eng.upload_kv(slot, bits(k).ctypes.data, bits(v).ctypes.data, False)


def _run(eng, qs):
    q = np.ascontiguousarray(np.stack([bits(x).reshape(16, 256) for x in qs]))
    eng.bind_query(q.ctypes.data, False, 0)
    eng.run(0)
    eng.sync()
    return eng.debug_ids(), eng.output_host()


def _check_out(got_bits, want_bits):
    err = np.abs(O.bf16_to_f32(got_bits).astype(np.float64) - O.bf16_to_f32(want_bits).astype(np.float64))
    assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (err.max(), err.mean())


@pytest.fixture(scope="module", params=GOLDEN_FILES)
def gold(request):
    return Golden(request.param)


@pytest.mark.parametrize("staged", [False, True], ids=["fused", "staged"])
def test_reference_built_index(gold, cuda, staged):
    """Engine on the index the reference itself built: ids equal the pinned oracle."""
    views = gold.views()
    eng = _engine(1, gold.context, views[0]["nc"], sink=gold.sink, local=gold.local, staged=staged)
    try:
        eng.upload_index(0, views)
        _upload_kv(eng, 0, gold.k, gold.v)
        for qi, q in enumerate(gold.queries):
            ids, out = _run(eng, [q])
            assert np.array_equal(ids[0], gold.z[f"q{qi}_final_ids"]), f"query {qi}: selected ids"
            _check_out(out[0], gold.z[f"q{qi}_out"])
    finally:
        eng.close()


def test_upload_codec_and_fp8_records(gold, cuda):
    views = gold.views()
    T = gold.context
    eng = _engine(1, T, views[0]["nc"], sink=gold.sink, local=gold.local)
    try:
        eng.upload_index(0, views)
        _upload_kv(eng, 0, gold.k, gold.v)
        scales, p2, r2, r4 = O.key_codec(bits(gold.k))
        assert np.array_equal(eng.read_stage(0, "key_scale", np.float32, (4, 256)), scales)
        assert np.array_equal(eng.read_stage(0, "prefix2", np.uint8, (4, T, 64)), p2)
        assert np.array_equal(eng.read_stage(0, "residual2", np.uint8, (4, T, 64)), r2)
        assert np.array_equal(eng.read_stage(0, "residual4", np.uint8, (4, T, 128)), r4)
        kv8 = eng.read_stage(0, "kv8", np.uint8, (4, T, 512))
        want_k = gold.k.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        want_v = gold.v.to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert np.array_equal(kv8[..., :256], want_k)
        assert np.array_equal(kv8[..., 256:], want_v)
    finally:
        eng.close()


def test_fp8_conversion_edge_values(cuda):
    """Saturation/NaN/subnormal/tie behaviour of the record conversion equals torch's cast."""
    T = 8192
    vals = torch.tensor([0.0, -0.0, 1e-9, 2.0 ** -10, 1.5 * 2.0 ** -9, 0.001953125, 447.0, 448.0, 449.0,
                         463.9, 464.0, 465.0, -465.0, 1e30, 240.0, 3.14159, -2.71828], dtype=torch.float32)
    k = torch.zeros(4, T, 256)
    k[0, 0, :len(vals)] = vals
    k[1, 5, 10:10 + len(vals)] = -vals
    k = k.bfloat16()
    v = k.flip(1).contiguous()
    case = Case(context=T, nprobe=128, seed=3)
    eng = _engine(1, T, case.index.cells()[0]["centroids"].shape[0])
    try:
        eng.upload_index(0, [device_view(c) for c in case.index.cells()])
        _upload_kv(eng, 0, k, v)
        kv8 = eng.read_stage(0, "kv8", np.uint8, (4, T, 512))
        assert np.array_equal(kv8[..., :256], k.to(torch.float8_e4m3fn).view(torch.uint8).numpy())
        assert np.array_equal(kv8[..., 256:], v.to(torch.float8_e4m3fn).view(torch.uint8).numpy())
    finally:
        eng.close()


@pytest.mark.parametrize("staged", [False, True], ids=["fused", "staged"])
def test_batched_slots_match_single(cuda, staged):
    """Three independent caches in one engine (one launch per step or stage) vs the oracle."""
    cases = [Case(context=8192, nprobe=128, seed=s) for s in (21, 22, 23)]
    nc = cases[0].index.cells()[0]["centroids"].shape[0]
    eng = _engine(3, 8192, nc, staged=staged)
    try:
        for s, c in enumerate(cases):
            eng.upload_index(s, [device_view(x) for x in c.index.cells()])
            _upload_kv(eng, s, c.k, c.v)
        qs = [c.query(500 + s) for s, c in enumerate(cases)]
        ids, out = _run(eng, qs)
        for s, (c, q) in enumerate(zip(cases, qs)):
            res, ref = c.oracle(q)
            assert np.array_equal(ids[s], np.stack([r["final_ids"] for r in res])), f"slot {s}"
            _check_out(out[s], ref)
    finally:
        eng.close()


@pytest.mark.parametrize("staged", [False, True], ids=["fused", "staged"])
def test_capacity_overflow_is_reported(cuda, staged):
    """A pool above the configured capacity sets the status word; sync raises."""
    case = Case(context=8192, nprobe=128, seed=11)
    nc = case.index.cells()[0]["centroids"].shape[0]
    eng = _engine(1, 8192, nc, capacity=2048, staged=staged)
    try:
        eng.upload_index(0, [device_view(c) for c in case.index.cells()])
        _upload_kv(eng, 0, case.k, case.v)
        q = bits(case.query(7)).reshape(1, 16, 256).copy()
        eng.bind_query(q.ctypes.data, False, 0)
        eng.run(0)
        with pytest.raises(_native.NativeError) as exc:
            eng.sync()
        assert exc.value.code == _native.SKV_E_CAPACITY
        assert eng.status().flags & _native.SKV_STATUS_POOL_OVER
        # the engine stays usable: a later run with a smaller nprobe is rejected
        # by validation, and output memory is still readable
        assert eng.output_host().shape == (1, 16, 256)
    finally:
        eng.close()


def test_small_pool_is_reported(cuda):
    """nprobe too small for the 2048-key Stage-1.5 minimum raises like the reference."""
    from seoulkv_b200 import SeoulKV4, SeoulKV4Config

    case = Case(context=8192, nprobe=16, seed=11)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=SeoulKV4Config()) as attn:
        with pytest.raises(ValueError, match="outside"):
            attn.run(case.query(1))
