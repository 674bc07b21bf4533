"""Index build and the NPZ file format (load-compatible with the reference)."""

import os
import sys

import numpy as np
import pytest
import torch

from seoulkv_b200 import SeoulKV4Index, _codecs
from tests.helpers import Case

# the reference's source directory (holding seoulkv4/), only from the environment
REF = os.environ.get("SEOULKV_REFERENCE", "")
HAVE_REF = bool(REF) and os.path.isdir(os.path.join(REF, "seoulkv4"))


@pytest.fixture(scope="module")
def case():
    return Case(context=8192, nprobe=64, seed=41)


def _cells_equal(a, b):
    assert a.keys() == b.keys()
    for k in a:
        x, y = a[k], b[k]
        if isinstance(x, torch.Tensor):
            assert x.dtype == y.dtype and torch.equal(x.view(torch.uint8) if x.dtype == torch.bfloat16 else x,
                                                       y.view(torch.uint8) if y.dtype == torch.bfloat16 else y), k
        else:
            assert x == y, k


def test_build_produces_valid_spill2_index(case):
    for c in case.index.cells():
        _codecs.validate_static_cell(c)
        _codecs.require_group_scale_cell(c)
        nc = c["centroids"].shape[0]
        assert nc == 1952 and c["upper"].shape == (nc, 64)


def test_build_is_deterministic(case):
    again = SeoulKV4Index.build(case.k, case.v, nprobe=64)
    for a, b in zip(case.index.cells(), again.cells()):
        _cells_equal(a, b)


def test_dump_load_roundtrip(case, tmp_path):
    p = tmp_path / "idx.npz"
    case.index.dump(p)
    back = SeoulKV4Index.load(p)
    for a, b in zip(case.index.cells(), back.cells()):
        _cells_equal(a, b)
    assert back.metadata() == case.index.metadata()
    over = SeoulKV4Index.load(p, nprobe=[16, 32, 48, 64])
    assert over.nprobe == (16, 32, 48, 64)
    assert over.metadata()["nprobe_source"] == "load override"
    with pytest.raises(ValueError):
        SeoulKV4Index.load(p, nprobe=7)


def test_load_rejects_corrupt_files(case, tmp_path):
    p = tmp_path / "idx.npz"
    case.index.dump(p)
    z = dict(np.load(p))
    z["0_values"] = z["0_values"].copy()
    z["0_values"][0] = z["0_values"][1]  # breaks spill-2 invariants
    bad = tmp_path / "bad.npz"
    np.savez(bad, **z)
    with pytest.raises(ValueError):
        SeoulKV4Index.load(bad)
    (tmp_path / "junk.npz").write_bytes(b"not a zip")
    with pytest.raises(Exception):
        SeoulKV4Index.load(tmp_path / "junk.npz")


@pytest.mark.skipif(not HAVE_REF, reason="reference package not importable here")
@pytest.mark.skipif(not HAVE_REF, reason="needs the reference package")
def test_reference_loads_our_dump_and_we_load_theirs(case, tmp_path):
    sys.path.insert(0, REF)
    from seoulkv4 import SeoulKV4Index as RefIndex

    ours = tmp_path / "ours.npz"
    case.index.dump(ours)
    ref = RefIndex.load(ours)
    for a, b in zip(case.index.cells(), ref._cells):
        _cells_equal(a, b)
    built = RefIndex.build(case.k, case.v, nprobe=64)
    theirs = tmp_path / "theirs.npz"
    built.dump(theirs)
    back = SeoulKV4Index.load(theirs)
    for a, b in zip(built._cells, back.cells()):
        _cells_equal(a, b)
    assert back.metadata() == built.metadata()


@pytest.mark.skipif(not HAVE_REF, reason="needs the reference package (its fixture writer)")
def test_legacy_v3_grouped_fixture_loads(case, tmp_path):
    """A version-3 grouped fixture (the index cells plus a diagnostic replay
    query), written by the reference's own ``save_fixture``, opens as an index:
    the query fields are dropped and every index array equals the source's."""
    sys.path.insert(0, REF)
    from seoulkv4._codecs import index as ref_codec

    cells = []
    g = torch.Generator().manual_seed(5)
    for c in case.index.cells():
        nc = int(c["centroids"].shape[0])
        f = dict(c)
        f["q"] = torch.randn(4, 256, generator=g).bfloat16()
        f["coarse_ids"] = torch.arange(nc, dtype=torch.int32)
        f["head_mask"] = torch.full((nc,), 15, dtype=torch.int32)
        cells.append(f)
    path = tmp_path / "grouped_v3.npz"
    ref_codec.save_fixture(path, cells, {"source": "test"})
    loaded, meta = _codecs.load_index(path)
    assert meta["version"] == 3
    for src, got in zip(case.index.cells(), loaded):
        assert not ({"q", "coarse_ids", "head_mask"} & got.keys())
        for name, value in src.items():
            if isinstance(value, torch.Tensor):
                ref = value.float() if value.dtype == torch.bfloat16 else value  # v3 stores BF16 as FP32
                assert torch.equal(got[name].to(ref.dtype), ref), name
            else:
                assert got[name] == value, name
    idx = SeoulKV4Index.load(path, nprobe=64)
    assert idx.nprobe == (64, 64, 64, 64)
