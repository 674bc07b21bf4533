"""What an FP32 accumulation of the scoring dots would change (CPU, oracle only).

Every scoring dot of the canonical definition is an exact sum rounded once to
FP32.  The reference forms its dots on the TT FPU, whose accumulation order
and precision are not in its repository.  These tests decode the 128K
headline layer twice, once exactly and once with every dot summed in FP32 in
dimension order (``oracle.set_fp32_accumulation``, one rounding per add, a
plausible float pipeline), and record how many coarse bounds, stage scores
and selected ids move, and how far the output moves: the exposure of the
id parity to the unpinned accumulation.
"""

import numpy as np
import pytest

from oracle import oracle as O

QUERIES = 8


@pytest.fixture(scope="module")
def case(headline_case):
    O.set_threads(8)
    yield headline_case
    O.set_fp32_accumulation(False)
    O.set_threads(1)


def test_fp32_accumulation_exposure(case):
    moved = {"lo_hi": 0, "pool_changed": 0, "heads_ids_changed": 0, "ids_swapped": 0}
    bounds = 0
    worst_max = worst_mean = 0.0
    for i in range(QUERIES):
        q = case.query(500 + i)
        O.set_fp32_accumulation(False)
        exact, out_exact = case.oracle(q)
        O.set_fp32_accumulation(True)
        approx, out_approx = case.oracle(q)
        O.set_fp32_accumulation(False)
        for a, b in zip(exact, approx):
            bounds += a["lo"].size + a["hi"].size
            moved["lo_hi"] += int((a["lo"] != b["lo"]).sum() + (a["hi"] != b["hi"]).sum())
            for key in ("fine_scores", "s15_scores", "s16_scores", "s2_scores"):
                if a[key].shape == b[key].shape:
                    moved[key] = moved.get(key, 0) + int((a[key] != b[key]).sum())
            moved["pool_changed"] += int(not np.array_equal(a["pool"], b["pool"]))
            for h in range(4):
                d = len(set(a["final_ids"][h].tolist()) - set(b["final_ids"][h].tolist()))
                moved["heads_ids_changed"] += d > 0
                moved["ids_swapped"] += d
        err = np.abs(O.bf16_to_f32(out_exact).astype(np.float64) - O.bf16_to_f32(out_approx).astype(np.float64))
        worst_max, worst_mean = max(worst_max, float(err.max())), max(worst_mean, float(err.mean()))
    print(f"\nFP32 accumulation vs exact over {QUERIES} queries ({QUERIES * 16} query heads, {bounds} coarse "
          f"bounds): {moved}; output max-abs {worst_max:.3g}, worst query mean-abs {worst_mean:.3g}")
    # the exact sum and the FP32 sum do differ, so the accumulation is a real
    # degree of freedom of the definition
    assert moved["lo_hi"] > 0
