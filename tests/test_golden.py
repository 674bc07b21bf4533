"""The CPU oracle against fixtures produced by the reference's own code.

See tests/golden/make_golden.py: the index, the key codec and every offline
oracle helper output stored there come from the reference package.
"""

import hashlib

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import _codecs
from seoulkv_b200.index import posting_mates
from tests.helpers import GOLDEN_FILES, Golden, bits


@pytest.fixture(scope="module", params=GOLDEN_FILES)
def gold(request):
    return Golden(request.param)


@pytest.fixture(scope="module")
def runs(gold):
    cells = gold.oracle_cells()
    return [[O.run_cell(c, bits(q).reshape(16, 256)[4 * g:4 * g + 4]) for g, c in enumerate(cells)]
            for q in gold.queries]


def test_regenerated_cache_matches_fingerprints(gold):
    for h in range(4):
        assert _codecs.fingerprint(gold.k[h]) == gold.meta["key_hashes"][h]


def test_key_codec_matches_reference(gold):
    scales, p2, r2, r4 = O.key_codec(bits(gold.k))
    assert np.array_equal(scales, gold.z["key_scales"])
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()  # noqa: E731
    want = gold.meta["plane_sha256"]
    assert sha(p2.reshape(-1, 64)) == want["prefix2_token"]
    assert sha(r2.reshape(-1, 64)) == want["residual2"]
    assert sha(r4.reshape(-1, 128)) == want["residual4"]


def test_query_operands_match_reference(gold, runs):
    for qi, res in enumerate(runs):
        q15 = np.stack([r["q15"] for r in res])
        qs = np.stack([r["qs"] for r in res])
        assert np.array_equal(q15, gold.z[f"q{qi}_ref_q15"])
        assert np.array_equal(qs, gold.z[f"q{qi}_ref_qs"])
        # the reference's host oracle multiplies by lambda in float64; the
        # device (and this restatement) in float32
        np.testing.assert_allclose(np.stack([r["qn"] for r in res]), gold.z[f"q{qi}_ref_norm"], rtol=1e-6)
        np.testing.assert_allclose(np.stack([r["qsum"] for r in res]), gold.z[f"q{qi}_ref_qsum"],
                                   rtol=1e-5, atol=1e-5)


def test_fine_selection_matches_reference_tree(gold, runs):
    for qi, res in enumerate(runs):
        for g, r in enumerate(res):
            assert np.array_equal(np.sort(r["fine_top"], axis=1), gold.z[f"q{qi}_{g}_ref_tree_top_p"])
            assert np.array_equal(r["selected"], gold.z[f"q{qi}_{g}_ref_fine_union"])


def test_pool_matches_encounter_union(gold, runs):
    for qi, res in enumerate(runs):
        for g, r in enumerate(res):
            assert np.array_equal(r["pool"], gold.z[f"q{qi}_{g}_ref_pool"])
            assert np.array_equal(np.sort(r["pool"]), gold.z[f"q{qi}_{g}_ref_expand_lists"])


def test_stage15_frontier_matches_reference_tree_merge(gold, runs):
    """The reference ranks Stage-1.5 per pool shard and merges the six
    shards' rows in a 6->3->2->1 tree into a 2048-score frontier
    (``merge_tree_reference``, score only), whose first 1600 scores enter the
    union.  The oracle's top-1600 per head has exactly those scores."""
    for qi, res in enumerate(runs):
        for g, r in enumerate(res):
            want = gold.z[f"q{qi}_{g}_ref_s15_frontier"]
            for h in range(4):
                top = r["s15_top"][h]
                got = np.sort(O.ord16(r["s15_scores"][h][top]))[::-1]
                assert np.array_equal(got, want[h][:len(top)]), (qi, g, h)


def test_stage15_union_matches_source_union(gold, runs):
    for qi, res in enumerate(runs):
        for g, r in enumerate(res):
            assert np.array_equal(r["u15"], gold.z[f"q{qi}_{g}_ref_s15_union"])


def test_final_outputs_are_stable(gold, runs):
    for qi, res in enumerate(runs):
        assert np.array_equal(np.stack([r["final_ids"] for r in res]), gold.z[f"q{qi}_final_ids"])


def test_group_scale_codec_matches_reference(gold):
    z = gold.z
    cell = dict(centroids=torch.from_numpy(z["codec_in_centroids"].copy()).view(torch.float16),
                offsets=torch.from_numpy(z["codec_in_offsets"].copy()),
                values=torch.from_numpy(z["codec_in_values"].copy()))
    enc = _codecs.encode_group_scale_cell(cell)
    for name in ("upper", "lower", "scale", "group_fine_scale", "fine_scale", "coarse_residual_norm", "coarse2",
                 "offsets", "values", "levels", "centroids", "decoded", "coarse_odd", "coarse_centroids"):
        t = enc[name]
        got = (t.view(torch.int16) if t.dtype in (torch.float16, torch.bfloat16) else t).numpy()
        assert np.array_equal(got, z[f"codec_out_{name}"]), name


def test_posting_mates_match_reference(gold):
    for g in range(4):
        got = posting_mates(gold.z[f"{g}_offsets"], gold.z[f"{g}_values"])
        assert np.array_equal(got, gold.z[f"{g}_mates"])
