"""Selection tie order of the CPU restatement, re-derived independently (CPU).

Stage-1.5 (top-1600 of the pool per query head), Stage-1.6 (top-256 of the
union) and Stage-II (top-100 of the candidates, in rank order) rank by the
ordered BF16 score, descending, and break equal scores by the lower position
(pool position for Stage-1.5, union position for Stage-1.6 and Stage-II).
The reference leaves these ties to its TT top-k library, whose order is not
in its repository, so the rule is the restatement's canonical choice.  These
tests re-derive every selection with a numpy sort on the 128K headline layer
and count how often a selection boundary falls inside a run of equal scores:
only there could another tie rule select another set of tokens.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import bits

QUERIES = 12


@pytest.fixture(scope="module")
def case(headline_case):
    O.set_threads(8)
    yield headline_case
    O.set_tie_high(False)
    O.set_threads(1)


@pytest.fixture(scope="module")
def runs(case):
    cells = case.cells()
    out = []
    for i in range(QUERIES):
        qb = bits(case.query(300 + i)).reshape(16, 256)
        out.append([O.run_cell(c, qb[4 * g:4 * g + 4]) for g, c in enumerate(cells)])
    return out


def _ranked(scores, positions):
    """Indices of `scores` in rank order: ordered score descending, position ascending."""
    return np.lexsort((np.asarray(positions, np.int64), -O.ord16(scores).astype(np.int64)))


def _boundary_tie(scores, order, k):
    """True when the k-th and (k+1)-th ranked scores are equal."""
    if k >= len(order):
        return False
    s = O.ord16(scores)
    return bool(s[order[k - 1]] == s[order[k]])


def test_selections_follow_score_then_position(runs):
    ties = {"stage15": 0, "stage16": 0, "stage2": 0, "stage2_inner": 0}
    heads = 0
    for cells in runs:
        for r in cells:
            npool, nu, ncand = len(r["pool"]), len(r["u15"]), len(r["cand"])
            for h in range(4):
                heads += 1
                # Stage-1.5: pool positions 0..npool-1
                k = min(O.UNION15, npool)
                order = _ranked(r["s15_scores"][h], np.arange(npool))
                assert np.array_equal(order[:k], r["s15_top"][h][:k]), "stage-1.5 ranking"
                ties["stage15"] += _boundary_tie(r["s15_scores"][h], order, k)
                # Stage-1.6: union positions 0..nu-1
                k = min(O.M16, nu)
                order = _ranked(r["s16_scores"][h], np.arange(nu))
                assert np.array_equal(order[:k], r["s16_top"][h][:k]), "stage-1.6 ranking"
                ties["stage16"] += _boundary_tie(r["s16_scores"][h], order, k)
                # Stage-II: candidates, positions = their union positions
                k = min(O.TOPK, ncand)
                order = _ranked(r["s2_scores"][h], r["cand"])
                assert np.array_equal(r["cand"][order[:k]], r["final_pos"][h][:k]), "stage-II ranking"
                ties["stage2"] += _boundary_tie(r["s2_scores"][h], order, k)
                top = O.ord16(r["s2_scores"][h][order[:k]])
                ties["stage2_inner"] += int(np.any(top[1:] == top[:-1]))
    # (the counts are the exposure to the unpinned tie order; printed for the record)
    print(f"\n{heads} query heads; selection boundary inside equal scores: {ties}")
    assert heads == QUERIES * 16


def test_the_tie_order_decides_ids_and_moves_the_output(case):
    """Decode with ties toward the higher position instead (a measurement of
    the unpinned choice, printed for the record): the top-100 set changes in
    most query heads, and the output moves with it."""
    changed_heads = changed_ids = 0
    worst_max = worst_mean = 0.0
    for i in range(8):
        q = case.query(300 + i)
        O.set_tie_high(False)
        low, out_low = case.oracle(q)
        O.set_tie_high(True)
        high, out_high = case.oracle(q)
        O.set_tie_high(False)
        for a, b in zip(low, high):
            for h in range(4):
                d = len(set(a["final_ids"][h].tolist()) - set(b["final_ids"][h].tolist()))
                changed_heads += d > 0
                changed_ids += d
        err = np.abs(O.bf16_to_f32(out_low).astype(np.float64) - O.bf16_to_f32(out_high).astype(np.float64))
        worst_max, worst_mean = max(worst_max, float(err.max())), max(worst_mean, float(err.mean()))
    print(f"\nopposite tie order over 128 query heads: {changed_heads} heads with a different top-100 set, "
          f"{changed_ids} ids swapped; output max-abs {worst_max:.3g}, worst per-query mean-abs {worst_mean:.3g}")
    assert changed_heads > 0 and worst_max > 0.0
    assert np.isfinite(worst_max)
