"""skv_attention_noalloc: the attention entry point that allocates nothing.

Some callers cannot allocate device memory once they are running: a server
that has committed its whole HBM budget at start-up treats a later cudaMalloc
as a failure (and cudaMalloc would also synchronise the device under its
other streams).  They pass every buffer themselves; the only scratch is the
library's fixed file-scope device array.

These tests call the entry point through the C ABI and check its output
against the existing entry point (SeoulKV4.run -> skv_run) and against the
CPU oracle's attention, on two calls in a row, with two slots (a different
cache per slot), with ids outside [0, context) skipped, and with a head that
has no key at all.  This file is collected last so that a run stopping at the
first failure has already run every other test.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import SeoulKV4, SeoulKV4Config, _native
from tests.helpers import Case, bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3  # the north_star tolerance of the BF16 output


def _bind(lib):
    f = lib.skv_attention_noalloc
    f.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
                  ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def _records(case, cuda):
    """FP8-e4m3 [K | V] records [T][512] of the four KV heads (device)."""
    return [torch.cat([case.k[g].to(cuda).to(torch.float8_e4m3fn).view(torch.uint8),
                       case.v[g].to(cuda).to(torch.float8_e4m3fn).view(torch.uint8)], dim=-1).contiguous()
            for g in range(4)]


def _err(got_bits, want_bits):
    return np.abs(O.bf16_to_f32(got_bits).astype(np.float64) - O.bf16_to_f32(want_bits).astype(np.float64))


def _oracle_out(case, q_bits, ids, sink, local):
    """The oracle's attention of every query head over its dense zones and its
    ids that lie inside the context (BF16 bits [16, 256])."""
    k8, v8 = case.kv8()
    out = np.zeros((16, 256), np.uint16)
    for j in range(16):
        g, h = divmod(j, 4)
        keep = ids[g, h][(ids[g, h] >= 0) & (ids[g, h] < case.context)]
        keys = O.attention_keys(case.context, sink, local, keep)
        if len(keys):
            out[j] = O.attention(q_bits[j], k8[g], v8[g], keys)
    return out


@pytest.fixture(scope="module")
def cases():
    return [Case(context=8192, nprobe=128, seed=61), Case(context=8192, nprobe=128, seed=62)]


def test_noalloc_two_slots_match_skv_run_and_oracle(cuda, cases):
    lib = _native.load()
    attn_noalloc = _bind(lib)
    T = cases[0].context
    recs = [r for c in cases for r in _records(c, cuda)]  # slot-major, 8 record buffers
    kv_ptrs = (ctypes.c_void_p * 8)(*[t.data_ptr() for t in recs])
    out = torch.empty(2, 16, 256, dtype=torch.bfloat16, device=cuda)
    engines = [SeoulKV4(device=cuda, k=c.k, v=c.v, index=c.index, config=SeoulKV4Config(debug=True)) for c in cases]
    try:
        for call, qseeds in enumerate(((71, 81), (72, 82))):  # two calls in a row share the scratch
            qs = [c.query(s) for c, s in zip(cases, qseeds)]
            want, ids = [], []
            for e, q in zip(engines, qs):
                want.append(bits(e.run(q).to_torch()).reshape(16, 256))
                ids.append(e.debug_snapshot()["selected_ids"].numpy().astype(np.int32))
            qd = torch.stack([q.reshape(16, 256) for q in qs]).to(cuda).contiguous()
            idd = torch.from_numpy(np.stack(ids)).to(cuda).contiguous()
            out.fill_(float("nan"))
            rc = attn_noalloc(2, qd.data_ptr(), kv_ptrs, idd.data_ptr(), T, cases[0].sink, cases[0].local,
                              out.data_ptr(), None)
            assert rc == 0, lib.skv_last_error()
            torch.cuda.synchronize(cuda)
            got = bits(out.cpu())
            for s, c in enumerate(cases):
                e = _err(got[s], want[s])
                assert e.max() <= MAX_ABS and e.mean() <= MEAN_ABS, ("vs skv_run", call, s, e.max(), e.mean())
                ref = _oracle_out(c, bits(qs[s]).reshape(16, 256), ids[s], c.sink, c.local)
                e = _err(got[s], ref)
                assert e.max() <= MAX_ABS and e.mean() <= MEAN_ABS, ("vs oracle", call, s, e.max(), e.mean())
    finally:
        for e in engines:
            e.close()


def test_noalloc_skips_ids_outside_the_context(cuda, cases):
    """Ids of -1 or >= context are left out of the softmax; with no dense zones
    a head whose ids are all outside gets zeros."""
    lib = _native.load()
    attn_noalloc = _bind(lib)
    rng = np.random.default_rng(5)
    T = cases[0].context
    recs = [r for c in cases for r in _records(c, cuda)]
    kv_ptrs = (ctypes.c_void_p * 8)(*[t.data_ptr() for t in recs])
    ids = rng.integers(0, T, size=(2, 4, 4, 100)).astype(np.int32)
    ids[0, 1, 2, ::3] = -1
    ids[0, 3, 0, 10:40] = T
    ids[1, 2, 1, :] = T + 77
    ids[1, 0, 3, 50:] = -5
    qs = [c.query(91 + i) for i, c in enumerate(cases)]
    qd = torch.stack([q.reshape(16, 256) for q in qs]).to(cuda).contiguous()
    idd = torch.from_numpy(ids).to(cuda).contiguous()
    out = torch.empty(2, 16, 256, dtype=torch.bfloat16, device=cuda)
    for sink, local in ((128, 256), (0, 0)):
        for _ in range(2):  # two calls in a row
            out.fill_(float("nan"))
            rc = attn_noalloc(2, qd.data_ptr(), kv_ptrs, idd.data_ptr(), T, sink, local, out.data_ptr(), None)
            assert rc == 0, lib.skv_last_error()
            torch.cuda.synchronize(cuda)
            got = bits(out.cpu())
            for s, c in enumerate(cases):
                ref = _oracle_out(c, bits(qs[s]).reshape(16, 256), ids[s], sink, local)
                e = _err(got[s], ref)
                assert e.max() <= MAX_ABS and e.mean() <= MEAN_ABS, (sink, local, s, e.max(), e.mean())
            if sink == 0 and local == 0:
                # KV head 2, query head 1 of slot 1 has no key inside the context
                assert not np.any(got[1][2 * 4 + 1]), "a head without keys must be zero"


def test_noalloc_rejects_oversized_requests(cuda):
    lib = _native.load()
    attn_noalloc = _bind(lib)
    dummy = torch.zeros(16, dtype=torch.int32, device=cuda)
    ptrs = (ctypes.c_void_p * 12)(*([dummy.data_ptr()] * 12))
    rc = attn_noalloc(3, dummy.data_ptr(), ptrs, dummy.data_ptr(), 8192, 128, 256, dummy.data_ptr(), None)
    assert rc == -1
    assert b"SKV_NOALLOC_MAX_SLOTS" in lib.skv_last_error()
