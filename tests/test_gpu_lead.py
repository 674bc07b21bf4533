"""The fused launch's lead cluster (a small synthetic cell decoded ahead of
the real cells, so that the kernel's instructions are in L2 when they reach
them): the real cells' results do not depend on it, and the lead cell itself
runs the whole funnel without a timeout or a capacity error."""

import numpy as np
import pytest
import torch

from seoulkv_b200 import SeoulKV4, SeoulKV4Config, SeoulKV4Batch
from tests.helpers import Case, bits

pytestmark = pytest.mark.gpu
C_TAGS, C_SEL, C_POOL, C_U15, C_CAND, C_STATUS = 0, 1, 2, 3, 4, 5


@pytest.fixture(scope="module")
def case():
    return Case(context=32768, nprobe=256, seed=71)


def _decode(case, lead, queries):
    cfg = SeoulKV4Config(debug=True, lead_cluster=lead)
    ids, outs = [], []
    with SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index, config=cfg) as attn:
        for q in queries:
            outs.append(bits(attn.run(q).to_torch()).copy())
            ids.append(attn.debug_snapshot()["selected_ids"].numpy().copy())
        lead_counts = attn._engine.read_stage(0, "lead_counts", np.int32, 8) if lead else None
    return np.stack(ids), np.stack(outs), lead_counts


def test_lead_cluster_changes_no_bit(case, cuda):
    queries = [case.query(s) for s in (1, 2, 3)]
    ids_a, out_a, counts = _decode(case, True, queries)
    ids_b, out_b, _ = _decode(case, False, queries)
    assert np.array_equal(ids_a, ids_b) and np.array_equal(out_a, out_b)
    # the lead cell took the real cells' path: a legal pool, every stage populated, no error
    assert counts[C_STATUS] == 0, counts
    assert 2048 <= counts[C_POOL] <= 13056 and counts[C_SEL] > 0 and counts[C_U15] > 0 and counts[C_CAND] > 0, counts


def test_lead_cluster_in_a_batch(case, cuda):
    q = torch.stack([case.query(5), case.query(6)]).reshape(2, 1, 16, 256)
    outs = []
    for lead in (True, False):
        b = SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v, case.index)] * 2,
                          config=SeoulKV4Config(debug=True, lead_cluster=lead))
        outs.append(bits(b.run(q).to_torch()).copy())
        b.close()
    assert np.array_equal(outs[0], outs[1])
