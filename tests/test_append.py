"""Cache append on the CPU: the oracle's definition, host validation, ABI."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import SeoulKV4, SeoulKV4Batch, SeoulKV4Config, _native
from seoulkv_b200 import _clustering
from seoulkv_b200.index import posting_mates
from tests.helpers import Case, bits


def _pack2(codes):
    c = codes.reshape(codes.shape[0], -1, 4).astype(np.uint8)
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def _random_codebook(nc, seed):
    rng = np.random.default_rng(seed)
    code = rng.integers(0, 16, size=(nc, 256))
    fs = rng.uniform(0.01, 0.05, size=nc // 32).astype(np.float16).astype(np.float32)
    return _pack2(code >> 2), _pack2(code & 3), fs, code


def _grid_ints(vals):
    """The decode's operand grid in exact Python integers (flush below 2^(E-22), unit 2^(E-29))."""
    import math

    nz = [abs(v) for v in vals if v != 0]
    if not nz:
        return [0] * len(vals)
    E = max(math.frexp(v)[1] - 1 for v in nz)
    out = []
    for v in vals:
        if v == 0 or math.frexp(abs(v))[1] - 1 < E - 22:
            out.append(0)
        else:
            q = math.ldexp(v, 29 - E)
            assert q == int(q)
            out.append(int(q))
    return out


def test_assign_spill2_is_the_exact_score_top2():
    nc = 96
    upper, lower, fs, code = _random_codebook(nc, 1)
    # two equal rows in one scale group: every key ties on them
    code[40] = code[41]
    upper, lower = _pack2(code >> 2), _pack2(code & 3)
    rng = np.random.default_rng(2)
    keys = torch.from_numpy(rng.normal(size=(6, 256)).astype(np.float32)).bfloat16()
    keys[3] = 0  # all scores 0: the two lowest ids
    keys[4, 7] = 2.0 ** -40  # below 2^(E-22): flushed
    kb = bits(keys)
    got = O.assign_spill2(kb, upper, lower, fs)
    for j in range(len(keys)):
        xs = _grid_ints([float(x) for x in O.bf16_to_f32(kb[j])])
        scores = [float(sum(xs[d] * (2 * int(code[c, d]) - 15) for d in range(256))) * float(fs[c // 32])
                  for c in range(nc)]
        want = sorted(range(nc), key=lambda c: (-scores[c], c))[:2]
        assert list(got[j]) == want, j
    assert list(got[3]) == [0, 1]
    # a key that picks the tied pair gets the lower id first
    tk = torch.from_numpy((2 * code[40] - 15).astype(np.float32))[None].bfloat16()
    assert list(O.assign_spill2(bits(tk), upper, lower, fs)[0]) == [40, 41]


def test_append_postings_equals_a_csr_over_all_tokens():
    rng = np.random.default_rng(3)
    nc, r, extra = 64, 500, 37
    lab = np.stack([rng.choice(nc, 2, replace=False) for _ in range(r + extra)])
    tok0 = 100  # retrieval tokens start after the sink
    off0, val0 = _clustering.to_csr(torch.from_numpy(lab[:r]), nc)
    off0, val0 = off0.numpy(), val0.numpy() + tok0
    mates0 = posting_mates(off0, val0)
    # in two steps, like two appends
    a = O.append_postings(off0, val0, mates0, np.arange(tok0 + r, tok0 + r + 20), lab[r:r + 20])
    b = O.append_postings(*a, np.arange(tok0 + r + 20, tok0 + r + extra), lab[r + 20:])
    full_off, full_val = _clustering.to_csr(torch.from_numpy(lab), nc)
    assert np.array_equal(b[0], full_off.numpy())
    assert np.array_equal(b[1], full_val.numpy() + tok0)
    assert np.array_equal(b[2], posting_mates(b[0], b[1]))


def test_encode_planes_under_fixed_scales():
    case_k = torch.randn(2, 40, 256).bfloat16()
    scales, p2, r2, r4 = O.key_codec(bits(case_k))
    for g in range(2):
        e = O.encode_planes(bits(case_k[g]), scales[g])
        assert np.array_equal(e[0], p2[g]) and np.array_equal(e[1], r2[g]) and np.array_equal(e[2], r4[g])
    # keys beyond the build's range clamp to the end codes
    big = torch.full((1, 256), 1e4).bfloat16()
    small = torch.full((1, 256), -1e4).bfloat16()
    assert (O.encode_planes(bits(big), scales[0])[0] == 0xFF).all()
    assert (O.encode_planes(bits(small), scales[0])[2] == 0).all()


@pytest.fixture(scope="module")
def case():
    return Case(context=8192, nprobe=128, seed=41)


def test_append_config_and_validation(case):
    with pytest.raises(ValueError):
        SeoulKV4Config(max_context=100)
    with pytest.raises(ValueError):
        SeoulKV4Config(max_context=8192.0)
    with pytest.raises(ValueError):
        SeoulKV4Config(max_context=(1 << 20) + 1)
    with pytest.raises(ValueError, match="below the index"):
        SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index, config=SeoulKV4Config(max_context=7000))
    k1, v1 = case.k[:, :3].clone(), case.v[:, :3].clone()
    static = SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index)
    with pytest.raises(ValueError, match="max_context"):
        static.append(k1, v1)
    grow = SeoulKV4(device="cuda:0", k=case.k, v=case.v, index=case.index,
                    config=SeoulKV4Config(max_context=8200))
    assert grow.context == 8192 and grow.metadata()["max_context"] == 8200
    for bad_k, bad_v in ((k1.float(), v1), (k1[:3], v1[:3]), (k1[:, :0], v1[:, :0]), (k1, v1[:, :2]),
                         (k1[..., :128], v1[..., :128])):
        with pytest.raises(ValueError):
            grow.append(bad_k, bad_v)
    nan = k1.clone()
    nan[1, 2, 3] = float("nan")
    with pytest.raises(ValueError, match="finite"):
        grow.append(nan, v1)
    with pytest.raises(ValueError, match="passes max_context"):
        grow.append(case.k[:, :9], case.v[:, :9])
    assert not grow.initialized and grow.context == 8192
    grow.close()
    with pytest.raises(RuntimeError):
        grow.append(k1, v1)
    batch = SeoulKV4Batch(device="cuda:0", caches=[(case.k, case.v, case.index)] * 2,
                          config=SeoulKV4Config(max_context=8200))
    with pytest.raises(ValueError):
        batch.append(k1, v1)  # needs [2, 4, m, 256]
    with pytest.raises(ValueError, match="passes max_context"):
        batch.append(case.k[:, :9].expand(2, -1, -1, -1), case.v[:, :9].expand(2, -1, -1, -1))


def test_engine_rejects_bad_max_context():
    lib = _native.load()
    h = ctypes.c_void_p()
    for mc in (8191, (1 << 20) + 4):
        d = _native.SkvDesc(n_slots=1, context=8192, sink=128, local=256, nc=1952, stage15_capacity=13056,
                            device=0, max_context=mc)
        assert lib.skv_create(ctypes.byref(d), ctypes.byref(h)) == -1
        assert b"max_context" in lib.skv_last_error()
