"""skv_attention_noalloc: the attention entry point that allocates nothing.

Callers that cannot allocate device memory after start-up (a server that has
committed its whole HBM budget, where cudaMalloc would fail or stall the
device) pass every buffer themselves; the only scratch is the library's
fixed file-scope device array.  Here its output is checked against the
existing entry point (SeoulKV4.run -> skv_run) on two calls in a row.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from seoulkv_b200 import SeoulKV4, SeoulKV4Config, _native
from tests.helpers import Case, bits

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _bind(lib):
    f = lib.skv_attention_noalloc
    f.argtypes = [ctypes.c_int32, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p,
                  ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


def test_noalloc_attention_matches_skv_run(cuda):
    lib = _native.load()
    attn_noalloc = _bind(lib)
    case = Case(context=8192, nprobe=128, seed=61)
    T = case.context
    kv8 = [torch.cat([case.k[g].to(cuda).to(torch.float8_e4m3fn).view(torch.uint8),
                      case.v[g].to(cuda).to(torch.float8_e4m3fn).view(torch.uint8)], dim=-1).contiguous()
           for g in range(4)]
    kv_ptrs = (ctypes.c_void_p * 4)(*[t.data_ptr() for t in kv8])
    out = torch.empty(16, 256, dtype=torch.bfloat16, device=cuda)
    with SeoulKV4(device=cuda, k=case.k, v=case.v, index=case.index, config=SeoulKV4Config(debug=True)) as attn:
        for qseed in (71, 72):  # two calls in a row share the scratch
            q = case.query(qseed)
            want = attn.run(q).to_torch().reshape(16, 256)
            ids = attn.debug_snapshot()["selected_ids"].to(torch.int32).to(cuda).contiguous()
            qd = q.reshape(16, 256).to(cuda).contiguous()
            rc = attn_noalloc(1, qd.data_ptr(), kv_ptrs, ids.data_ptr(), T, case.sink, case.local,
                              out.data_ptr(), None)
            assert rc == 0, lib.skv_last_error()
            torch.cuda.synchronize(cuda)
            got = out.cpu()
            err = np.abs(O.bf16_to_f32(bits(got)).astype(np.float64) - O.bf16_to_f32(bits(want)).astype(np.float64))
            assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (qseed, err.max(), err.mean())


def test_noalloc_rejects_oversized_requests(cuda):
    lib = _native.load()
    attn_noalloc = _bind(lib)
    dummy = torch.zeros(16, dtype=torch.int32, device=cuda)
    ptrs = (ctypes.c_void_p * 12)(*([dummy.data_ptr()] * 12))
    rc = attn_noalloc(3, dummy.data_ptr(), ptrs, dummy.data_ptr(), 8192, 128, 256, dummy.data_ptr(), None)
    assert rc == -1
    assert b"SKV_NOALLOC_MAX_SLOTS" in lib.skv_last_error()
