"""How far the reference device's attention numerics can sit from the restatement (CPU).

The reference's attention (TTNN sparse SDPA) widens the FP8 [V | K] records
into bfloat8_b tiles before the matmuls (a block float: 16 consecutive
elements of a tile row share one exponent and keep 7 magnitude bits each,
`_kernels/stage16/seoulkv4_stage16_fused.py:1717-1723`) and holds q.k in a
BF16 buffer (`CB.ATTENTION_QK`); the restatement keeps every FP8 value and
computes in float64.  How those conversions round lives in the TT libraries,
not in the reference's repository, so it is not pinned.  This test decodes
the 128K headline layer's winners through both block-float roundings
(nearest-even and truncation of the block mantissas) with BF16 q.k, and
records the spread of the output beside the parity tolerance.
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import bits

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def block_float(x: np.ndarray, rne: bool) -> np.ndarray:
    """bfloat8_b values of x [..., n*16]: per 16-element block, one shared
    exponent E (the block maximum's) and magnitudes m * 2^(E-6), m in 0..127."""
    shape = x.shape
    b = x.reshape(-1, 16)
    a = np.abs(b)
    mx = a.max(axis=1, keepdims=True)
    e = np.floor(np.log2(np.where(mx > 0, mx, 1.0)))
    quantum = np.exp2(e - 6)
    m = a / quantum
    m = np.round(m) if rne else np.floor(m)
    m = np.minimum(m, 127.0)
    return (np.sign(b) * m * quantum).reshape(shape)


def _bf16(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.asarray(x, np.float32)).bfloat16().float().numpy().astype(np.float64)


def _attend(q_bits, kk, vv):
    """softmax(bf16(q.k) / 16) v in float64, BF16 out (bit patterns)."""
    q = O.bf16_to_f32(q_bits).astype(np.float64)
    s = _bf16(kk @ q) / 16.0
    p = np.exp(s - s.max())
    return O.bf16_bits(((p[:, None] * vv).sum(axis=0) / p.sum()).astype(np.float32))


@pytest.fixture(scope="module")
def case(headline_case):
    O.set_threads(8)
    yield headline_case
    O.set_threads(1)


def test_block_float_values():
    """Known blocks: the maximum keeps 7 bits; smaller elements lose the bits
    below 2^(E-6) (rounded or cut); a block of zeros stays zero."""
    x = np.zeros(32)
    x[:4] = [1.5, -0.75, 2.0 ** -6 * 1.5, 2.0 ** -7 * 1.25]   # E = 0: quantum 2^-6
    got_rne, got_cut = block_float(x, True), block_float(x, False)
    assert got_rne[0] == 1.5 and got_rne[1] == -0.75
    assert got_rne[2] == 2.0 ** -6 * 2 and got_cut[2] == 2.0 ** -6      # 1.5 quanta
    assert got_rne[3] == 2.0 ** -6 * 1 and got_cut[3] == 0.0           # 0.625 quanta
    assert not got_rne[16:].any()
    x[0] = 1.999
    assert block_float(x, True)[0] == 127 * 2.0 ** -6                    # clamped at 7 bits


def test_block_float_attention_spread(case):
    """The output spread between TT-like numerics and the restatement,
    printed for the record: about the size of the tolerance itself."""
    worst = {}
    for i in range(6):
        q = case.query(400 + i)
        qb = bits(q).reshape(16, 256)
        res, ref = case.oracle(q)
        want = O.bf16_to_f32(ref).astype(np.float64)
        for rne in (True, False):
            got = np.zeros((16, 256))
            for j in range(16):
                g, h = divmod(j, 4)
                keys = O.attention_keys(case.context, case.sink, case.local, res[g]["final_ids"][h])
                idx = torch.from_numpy(np.asarray(keys, dtype=np.int64))
                k8 = O.fp8_e4m3(case.k[g].index_select(0, idx).float().numpy())
                v8 = O.fp8_e4m3(case.v[g].index_select(0, idx).float().numpy())
                got[j] = O.bf16_to_f32(_attend(qb[j], block_float(k8, rne), block_float(v8, rne)))
            err = np.abs(got - want)
            w = worst.setdefault(rne, [0.0, 0.0])
            w[0], w[1] = max(w[0], float(err.max())), max(w[1], float(err.mean()))
    print(f"\nblock-float K/V and BF16 q.k vs the restatement, 6 queries x 16 heads: "
          f"nearest-even max-abs {worst[True][0]:.3g}, worst query mean-abs {worst[True][1]:.3g}; "
          f"truncation max-abs {worst[False][0]:.3g}, worst query mean-abs {worst[False][1]:.3g} "
          f"(tolerance {MAX_ABS} / {MEAN_ABS})")
    for rne in (True, False):
        assert 0.0 < worst[rne][0] < 10 * MAX_ABS and worst[rne][1] < 10 * MEAN_ABS
