"""Public API validation (mirrors the reference's errors); no GPU needed."""

import pytest
import torch

from seoulkv_b200 import DecodeResult, SeoulKV4, SeoulKV4Config, SeoulKV4Index
from seoulkv_b200.config import validate_nprobe
from tests.helpers import Case


@pytest.fixture(scope="module")
def case():
    return Case(context=8192, nprobe=128, seed=31)


def test_config_validation():
    assert SeoulKV4Config().stage15_capacity == 13056
    SeoulKV4Config(stage15_capacity=24576, debug=True, nprobe=64)
    for bad in (12287, 24577, 13000, 12288.0, True):
        with pytest.raises(ValueError):
            SeoulKV4Config(stage15_capacity=bad)
    with pytest.raises(TypeError):
        SeoulKV4Config(debug=1)
    with pytest.raises(ValueError):
        SeoulKV4Config(nprobe=24)
    assert SeoulKV4Config(nprobe=[16, 32, 48, 64]).nprobe == (16, 32, 48, 64)
    with pytest.raises(Exception):
        SeoulKV4Config().debug = True  # frozen
    cfg = SeoulKV4Config()
    assert cfg.l2_resident and cfg.lead_cluster and not cfg.trace_stages
    for field in ("l2_resident", "lead_cluster", "trace_stages"):
        with pytest.raises(TypeError):
            SeoulKV4Config(**{field: 1})


def test_nprobe_rules():
    assert validate_nprobe(64, 1000) == (64,) * 4
    assert validate_nprobe((16, 32, 48, 512), 1000) == (16, 32, 48, 512)
    for bad in (8, 520, 17, "64", (16, 16, 16), 64.0):
        with pytest.raises(ValueError):
            validate_nprobe(bad, 1000)
    with pytest.raises(ValueError):
        validate_nprobe(512, 500)


def test_build_validation(case):
    k, v = case.k, case.v
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k.float())
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k[:3])
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, v[:, :100])
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k[:, :6000])           # context below 6400
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k[:, :8190])           # not a multiple of 4
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, sink=4000, local=3000)  # retrieval zone < 2048
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, lam=-1.0)
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, lam=float("nan"))
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, seed=-1)
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, build_device="meta")
    with pytest.raises(ValueError):
        SeoulKV4Index.build(k, sink=1.5)


def test_index_metadata_and_zones(case):
    m = case.index.metadata()
    assert m["context"] == 8192 and m["sink"] == 128 and m["local"] == 256
    assert m["nprobe"] == [128] * 4 and m["summary_codec"] == "group-scale-32-v1"
    assert m["attention_tokens"] == 128 + 256 + 100
    assert len(m["key_hashes"]) == 4


def test_constructor_validation(case):
    idx = case.index
    with pytest.raises(TypeError):
        SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=idx, config=object())
    with pytest.raises(TypeError):
        SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=None)
    with pytest.raises(ValueError):
        SeoulKV4(device=None, k=case.k, v=case.v, index=idx)
    with pytest.raises(ValueError):
        SeoulKV4(device="cpu", k=case.k, v=case.v, index=idx)
    with pytest.raises(ValueError):
        SeoulKV4(device="cuda:0", k=case.k.float(), v=case.v, index=idx)
    with pytest.raises(ValueError):
        SeoulKV4(device="cuda:0", k=case.k, v=case.v[:, :4096], index=idx)
    bad = case.k.clone()
    bad[2, 7, 3] += 1
    with pytest.raises(ValueError, match="fingerprint"):
        SeoulKV4(device="cuda:0", k=bad, v=case.v, index=idx)


def test_lifecycle_without_run(case):
    attn = SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index)
    assert not attn.initialized
    meta = attn.metadata()
    assert meta["initialized"] is False and meta["cache_layout"] == "flat"
    with pytest.raises(RuntimeError):
        attn.debug_snapshot()
    with pytest.raises(ValueError):
        attn.run(torch.zeros(1, 1, 16, 255, dtype=torch.bfloat16))
    attn.close()
    attn.close()  # idempotent
    with pytest.raises(RuntimeError):
        attn.run(torch.zeros(1, 1, 16, 256, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError):
        attn.metadata()
    with SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index) as a2:
        assert not a2.initialized
    assert a2._closed


def test_result_liveness():
    class Owner:
        _closed = False
        _generation = 2

    o = Owner()
    r = DecodeResult(o, 1)
    with pytest.raises(RuntimeError):
        r.to_torch()


def test_batch_validation_and_lifecycle(case):
    """SeoulKV4Batch: the per-cache checks of SeoulKV4, plus shared shapes across caches."""
    from seoulkv_b200 import SeoulKV4Batch

    with pytest.raises(ValueError):
        SeoulKV4Batch(device="cuda:0", caches=[])
    with pytest.raises(TypeError):
        SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v, None)])
    with pytest.raises(ValueError):
        SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v[:, :4096], case.index)])
    other = Case(context=12288, nprobe=64, seed=32)
    with pytest.raises(ValueError, match="share the context"):
        SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v, case.index), (other.k, other.v, other.index)])
    bad = case.k.clone()
    bad[1, 5, 9] += 1
    with pytest.raises(ValueError, match="fingerprint"):
        SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v, case.index), (bad, case.v, case.index)])
    b = SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v, case.index)] * 2,
                      config=SeoulKV4Config(nprobe=64))
    meta = b.metadata()
    assert meta["caches"] == 2 and meta["initialized"] is False and meta["nprobe"] == [[64] * 4, [64] * 4]
    with pytest.raises(ValueError):
        b.run(torch.zeros(1, 1, 16, 256, dtype=torch.bfloat16))  # one query per cache
    with pytest.raises(RuntimeError):
        b.debug_snapshot()
    b.close()
    b.close()
    with pytest.raises(RuntimeError):
        b.run(torch.zeros(2, 1, 16, 256, dtype=torch.bfloat16))
