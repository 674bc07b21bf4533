"""SeoulKV4Batch on a B200: n independent caches in one launch per step give
the same ids and outputs, bit for bit, as n single-cache SeoulKV4 instances,
and the ids the CPU restatement gives."""

import numpy as np
import pytest
import torch

from seoulkv_b200 import SeoulKV4, SeoulKV4Batch, SeoulKV4Config
from tests.helpers import Case

pytestmark = pytest.mark.gpu


def test_batch_matches_single_instances(cuda):
    cases = [Case(context=8192, nprobe=128, seed=s) for s in (41, 42, 43)]
    cfg = SeoulKV4Config(debug=True)
    with SeoulKV4Batch(device="cuda:0", caches=[(c.k, c.v, c.index) for c in cases], config=cfg) as batch:
        for step in range(2):
            qs = [c.query(700 + 10 * step + i) for i, c in enumerate(cases)]
            q = torch.cat(qs, 0)
            out_b = batch.run(q).to_torch()
            ids_b = batch.debug_snapshot()["selected_ids"]
            assert tuple(ids_b.shape) == (3, 4, 4, 100)
            # device-resident queries: same results
            out_d = batch.run(q.cuda()).to_torch()
            assert torch.equal(out_b.view(torch.int16), out_d.view(torch.int16))
            dev = batch.run(q).device_tensor
            assert torch.equal(dev.cpu().view(torch.int16), out_b.view(torch.int16))
            for i, (c, qi) in enumerate(zip(cases, qs)):
                with SeoulKV4(device="cuda:0", k=c.k, v=c.v, index=c.index, config=cfg) as single:
                    out_s = single.run(qi).to_torch()
                    ids_s = single.debug_snapshot()["selected_ids"]
                assert torch.equal(ids_b[i], ids_s), f"cache {i}: ids"
                assert torch.equal(out_b[i:i + 1].view(torch.int16), out_s.view(torch.int16)), f"cache {i}: output"
                res, _ = c.oracle(qi)
                assert np.array_equal(ids_b[i].numpy(), np.stack([r["final_ids"] for r in res])), f"cache {i}: oracle"


def test_run_captured_in_a_callers_graph(cuda):
    """attn.run(q) inside torch.cuda.graph: the step's kernels join the
    caller's graph; replays with new query contents give the same results as
    plain runs."""
    c = Case(context=8192, nprobe=128, seed=51)
    qs = [c.query(900 + i).cuda() for i in range(3)]
    cfg = SeoulKV4Config(debug=True)
    with SeoulKV4(device="cuda:0", k=c.k, v=c.v, index=c.index, config=cfg) as attn:
        plain = []
        for q in qs:
            plain.append((attn.run(q).to_torch(), attn.debug_snapshot()["selected_ids"]))
        q_static = qs[0].clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                res = attn.run(q_static)
        torch.cuda.current_stream().wait_stream(s)
        for q, (out_p, ids_p) in zip(qs, plain):
            q_static.copy_(q)
            g.replay()
            torch.cuda.synchronize()
            out_g = res.device_tensors
            got = torch.cat([t.reshape(4, 256) for t in out_g]).cpu()
            assert torch.equal(got.view(torch.int16), out_p.reshape(16, 256).view(torch.int16))
            assert torch.equal(torch.from_numpy(attn._engine.debug_ids()[0]).long(), ids_p)
        del g
