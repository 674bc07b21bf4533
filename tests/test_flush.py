"""What the canonical definition's operand flush changes (CPU, oracle only).

Every scoring dot is the exact sum of (operand x integer weight) rounded once
to FP32, after elements below 2^(E-22) of their row's top exponent E are
flushed to zero (the flush lets the GPU hold an operand element in four int8
digits).  These tests decode the 128K headline layer twice, once with the
flush and once with an unflushed exact sum of every element (128-bit
integers, oracle.set_unflushed), and compare the selected ids.

* BASELINE-generator queries: no element falls below the flush level, so the
  two definitions agree on every intermediate.
* Queries with six elements per head row planted at 2^-23 .. 2^-44 of the
  row maximum: the flush changes some coarse bounds by one BF16 step, and no
  selected id.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import bits


@pytest.fixture(scope="module")
def layer(headline_case):
    O.set_threads(8)
    yield headline_case
    O.set_unflushed(False)
    O.set_threads(1)


def _flushed(qb):
    x = O.bf16_to_f32(qb).astype(np.float64)
    n = 0
    for row in x:
        e = np.floor(np.log2(np.abs(row).max()))
        n += int(((row != 0) & (np.abs(row) < 2.0 ** (e - 22))).sum())
    return n


def _both(case, qb):
    cells = case.cells()
    out = []
    for mode in (False, True):
        O.set_unflushed(mode)
        out.append([O.run_cell(c, qb[4 * g:4 * g + 4]) for g, c in enumerate(cells)])
    O.set_unflushed(False)
    return out


def _planted(qb, rng):
    """Six elements of every row set to +-max * 2^-e (1 + u), e = 23 .. 44."""
    x = O.bf16_to_f32(qb).copy()
    for j in range(16):
        m = np.abs(x[j]).max()
        for d, e in zip(rng.choice(256, 6, replace=False), (23, 25, 28, 31, 36, 44)):
            x[j, d] = np.sign(rng.standard_normal()) * m * 2.0 ** -e * (1 + rng.random())
    return torch.from_numpy(x).bfloat16().view(torch.int16).numpy().view(np.uint16)


def test_generator_queries_are_not_flushed(layer):
    for i in range(30):
        qb = bits(layer.query(100 + i)).reshape(16, 256)
        assert _flushed(qb) == 0
        flushed, exact = _both(layer, qb)
        for a, b in zip(flushed, exact):
            for key in ("lo", "hi", "fine_scores", "pool", "s15_scores", "final_ids"):
                if key in a:
                    assert np.array_equal(a[key], b[key]), (i, key)


def test_planted_small_elements_change_no_id(layer):
    rng = np.random.default_rng(5)
    changed_bounds = flushed = 0
    for i in range(50):
        qb = _planted(bits(layer.query(200 + i)).reshape(16, 256), rng)
        flushed += _flushed(qb)
        a, b = _both(layer, qb)
        for ra, rb in zip(a, b):
            changed_bounds += int((ra["lo"] != rb["lo"]).sum() + (ra["hi"] != rb["hi"]).sum())
            assert np.array_equal(ra["final_ids"], rb["final_ids"]), f"query {i}: the flush changed selected ids"
    assert O.unflushed_dropped() == 0
    # the planted elements are flushed and do move coarse bounds
    assert flushed > 0 and changed_bounds > 0, (flushed, changed_bounds)
