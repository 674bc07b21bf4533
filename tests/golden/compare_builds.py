"""Top-100 recall of the reference's index build against this package's build.

Both indices are built on the same synthetic K (BASELINE generator), both are
decoded by the CPU restatement of the funnel (``oracle/``) on the same
queries, and each query head's selected ids are compared with the exact
dense top-100 of q.k over the retrieval zone.  The reference's build is
imported from the directory in ``SEOULKV_REFERENCE`` (the one holding
``seoulkv4/``); its index travels to this package's loader through the
shared NPZ v4 format.  Test infrastructure: it decides whether
``SeoulKV4Index.build`` is a drop-in in results, not only in API.

    SEOULKV_REFERENCE=/path/to/reference/src python tests/golden/compare_builds.py [T] [nprobe] [queries]
"""

from __future__ import annotations

import os
import sys
import tempfile
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
REF = os.environ.get("SEOULKV_REFERENCE")
if not REF:
    sys.exit("set SEOULKV_REFERENCE to the reference's source directory (the one holding seoulkv4/)")
sys.path.insert(0, REF)

import seoulkv4  # noqa: E402

from oracle import oracle as O  # noqa: E402
from seoulkv_b200 import SeoulKV4Index, synthetic  # noqa: E402
from seoulkv_b200.index import device_view  # noqa: E402
from tests.helpers import bits  # noqa: E402


def cells_of(k, index):
    scales, p2, r2, r4 = O.key_codec(bits(k))
    out = []
    for g, c in enumerate(index.cells()):
        dv = device_view(c)
        out.append(O.CellInputs(nc=dv["nc"], nprobe=dv["nprobe"], lam=dv["lam"], upper=dv["upper"],
                                lower=dv["lower"], coarse_scale4=dv["coarse_scale4"], fine_scale=dv["fine_scale"],
                                resid_bf16=dv["resid_bf16"], offsets=dv["offsets"], values=dv["values"],
                                context=k.shape[1], prefix2=p2[g], residual2=r2[g], residual4=r4[g],
                                key_scale=scales[g]))
    return out


def main():
    T = int(sys.argv[1]) if len(sys.argv) > 1 else 32768
    nprobe = int(sys.argv[2]) if len(sys.argv) > 2 else 384
    nq = int(sys.argv[3]) if len(sys.argv) > 3 else 40
    seed = 1000
    k, v, mixes = synthetic.make_kv(T, seed=seed)
    t0 = time.time()
    ours = SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=nprobe)
    t_ours = time.time() - t0
    t0 = time.time()
    ref = seoulkv4.SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=nprobe)
    t_ref = time.time() - t0
    with tempfile.TemporaryDirectory() as d:
        ref.dump(os.path.join(d, "ref.npz"))
        ref_loaded = SeoulKV4Index.load(os.path.join(d, "ref.npz"))
    print(f"T={T} nprobe={nprobe}: build on the CPU {t_ours:.1f} s (this package), {t_ref:.1f} s (reference)")
    O.set_threads(2)
    qs = [synthetic.make_query(T, mixes, seed=seed * 7919 + i) for i in range(nq)]
    kz = k[:, 128:T - 256].float()
    for name, idx in (("this package", ours), ("reference", ref_loaded)):
        cells = cells_of(k, idx)
        hits = total = failed = 0
        with ThreadPoolExecutor(4) as pool:
            for q in qs:
                qb = bits(q).reshape(16, 256)
                try:
                    res = list(pool.map(lambda g: O.run_cell(cells[g], qb[4 * g:4 * g + 4]), range(4)))
                except O.OracleError:
                    failed += 1
                    continue
                sc = torch.einsum("ghd,grd->ghr", q.float().view(4, 4, 256), kz)
                top = (sc.topk(100, dim=-1).indices + 128).numpy()
                for g in range(4):
                    for h in range(4):
                        hits += len(np.intersect1d(res[g]["final_ids"][h], top[g, h]))
                        total += 100
        print(f"{name}: top-100 recall {hits / max(total, 1):.4f} over {total // 1600} queries ({failed} failed)")


if __name__ == "__main__":
    main()
