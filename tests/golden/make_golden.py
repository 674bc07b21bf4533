"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a checkout that has the reference package available (its ``src``
directory on ``sys.path``, e.g. ``SEOULKV_REFERENCE=/path/to/reference/src``)::

    python tests/golden/make_golden.py                      # golden_t8192.npz
    python tests/golden/make_golden.py --context 6400 --kv-seed 29 --nprobe 96 \
        --sink 64 --local 512 --q-seeds 401,402,403          # golden_t6400.npz

(the second one is the reference's smallest context, with other zones and
another probe budget).

The reference's decode path needs a Tenstorrent board, so the fixtures pin
everything that *can* run here:

* the index is built by the reference's own ``SeoulKV4Index.build`` on a
  seeded synthetic cache (K/V are regenerated from the seed in tests and
  checked against the stored SHA-256 fingerprints);
* the key codec planes come from the reference's ``_stage15_key_codec`` /
  ``encode_planes`` (stored as SHA-256 digests plus the scale table);
* query operands come from the reference's ``query_prepare.reference``;
* for each query, the oracle's Fine survivors/scores are fed to the
  reference's ``tree_top_p`` and ``distributed_union_reference``, its
  selected clusters to ``encounter_union`` / ``expand_lists``, its Stage-1.5
  scores (split over the reference's six pool shards) to the score-only
  ``merge_tree_reference`` of the 6->3->2->1 frontier merge, and its
  Stage-1.5 frontiers to ``source_union_reference``; their outputs are stored;
* the group-scale centroid codec and the posting-mate map of the reference
  are stored for a small input and for the fixture index.

The oracle's own final outputs (selected ids, BF16 attention output) are
stored too, as the end-to-end expectation for the CUDA engine.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
REF = os.environ.get("SEOULKV_REFERENCE")
if not REF:
    sys.exit("set SEOULKV_REFERENCE to the reference's source directory (the one holding seoulkv4/)")
sys.path.insert(0, REF)

from oracle import oracle as O  # noqa: E402
from seoulkv_b200 import synthetic  # noqa: E402
from seoulkv_b200.index import device_view  # noqa: E402

HERE = Path(__file__).resolve().parent


def parse():
    import argparse

    p = argparse.ArgumentParser()
    p.add_argument("--context", type=int, default=8192)
    p.add_argument("--kv-seed", type=int, default=17)
    p.add_argument("--nprobe", type=int, default=128)
    p.add_argument("--sink", type=int, default=128)
    p.add_argument("--local", type=int, default=256)
    p.add_argument("--q-seeds", default="301,302,303")
    return p.parse_args()


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main():
    args = parse()
    CONTEXT, KV_SEED, NPROBE, SINK, LOCAL = args.context, args.kv_seed, args.nprobe, args.sink, args.local
    Q_SEEDS = tuple(int(x) for x in args.q_seeds.split(","))
    OUT = HERE / f"golden_t{CONTEXT}.npz"
    from seoulkv4 import SeoulKV4Index as RefIndex
    from seoulkv4._codecs.index import encode_group_scale_cell, expand_lists
    from seoulkv4._codecs.keys import _stage15_key_codec, encode_planes
    from seoulkv4._kernels.common.seoulkv4_cluster_blocks import encounter_union, posting_mates
    from seoulkv4._kernels.query_prepare.host import reference as qp_reference
    from seoulkv4._kernels.stage15.seoulkv4_stage15_tree_merge import merge_tree_reference
    from seoulkv4._kernels.stage15.seoulkv4_stage15_union import source_union_reference
    from seoulkv4._kernels.stage1_fine.seoulkv4_fine_native_select import distributed_union_reference
    from seoulkv4._kernels.stage1_fine.seoulkv4_fine_parallel import schedule, tree_top_p

    k, v, mixes = synthetic.make_kv(CONTEXT, seed=KV_SEED)
    ref_index = RefIndex.build(k, v, sink=SINK, local=LOCAL, nprobe=NPROBE)
    cells = ref_index._cells
    data, meta = {}, {"context": CONTEXT, "kv_seed": KV_SEED, "nprobe": NPROBE, "q_seeds": list(Q_SEEDS),
                      "sink": SINK, "local": LOCAL, "key_hashes": [c["key_hash"] for c in cells], "cells": []}
    for g, c in enumerate(cells):
        for name in ("upper", "lower", "scale", "group_fine_scale", "coarse_residual_norm", "offsets", "values"):
            t = c[name]
            data[f"{g}_{name}"] = (t.view(torch.int16) if t.dtype == torch.float16 else t).numpy()
        meta["cells"].append({k2: c[k2] for k2 in ("context", "r0", "r1", "p", "lam", "spill")})
        data[f"{g}_mates"] = posting_mates(c).numpy().astype(np.int64).astype(np.int32)

    # key codec (reference) -- digests of the planes, the scale table in full
    codec = _stage15_key_codec(k)
    planes = encode_planes(codec, 1, 4)
    data["key_scales"] = codec["scales"].numpy()
    meta["plane_sha256"] = {n: sha(planes[n].numpy()) for n in ("prefix2_token", "residual2", "residual4")}

    # group-scale codec on a small deterministic input
    gen = torch.Generator().manual_seed(5)
    cent = (torch.randn(64, 256, generator=gen) * 0.07).half()
    lists = torch.randint(0, 1000, (64 * 6,), generator=gen).int()
    offsets = torch.arange(0, 64 * 6 + 1, 6, dtype=torch.int32)
    enc, _ = encode_group_scale_cell(dict(centroids=cent, offsets=offsets, values=lists))
    data["codec_in_centroids"] = cent.view(torch.int16).numpy()
    data["codec_in_offsets"] = offsets.numpy()
    data["codec_in_values"] = lists.numpy()
    for name in ("upper", "lower", "scale", "group_fine_scale", "fine_scale", "coarse_residual_norm",
                 "coarse2", "offsets", "values", "levels"):
        t = enc[name]
        data[f"codec_out_{name}"] = (t.view(torch.int16) if t.dtype in (torch.float16, torch.bfloat16) else t).numpy()
    for name in ("centroids", "decoded", "coarse_odd", "coarse_centroids"):
        t = enc[name]
        data[f"codec_out_{name}"] = t.view(torch.int16).numpy()

    # oracle inputs built from the reference index + reference planes
    p2 = planes["prefix2_token"].numpy().reshape(4, CONTEXT, 64)
    r2 = planes["residual2"].numpy().reshape(4, CONTEXT, 64)
    r4 = planes["residual4"].numpy().reshape(4, CONTEXT, 128)
    ocells = []
    for g, c in enumerate(cells):
        dv = device_view(c)
        ocells.append(O.CellInputs(
            nc=dv["nc"], nprobe=dv["nprobe"], lam=dv["lam"], upper=dv["upper"], lower=dv["lower"],
            coarse_scale4=dv["coarse_scale4"], fine_scale=dv["fine_scale"], resid_bf16=dv["resid_bf16"],
            offsets=dv["offsets"], values=dv["values"], context=CONTEXT, prefix2=p2[g], residual2=r2[g],
            residual4=r4[g], key_scale=codec["scales"][g].numpy()))
    k8 = O.fp8_e4m3(k.float().numpy())
    v8 = O.fp8_e4m3(v.float().numpy())

    for qi, qs in enumerate(Q_SEEDS):
        q = synthetic.make_query(CONTEXT, mixes, seed=qs)
        qb = bits(q).reshape(16, 256)
        ref_q = qp_reference(q, codec["scales"], [float(c["lam"]) for c in cells])
        # invert the reference's layouts back to plain [4][4][256] operands
        from seoulkv4._kernels.stage15.stage15_sfpu_native import coordinate_order
        order = coordinate_order()
        st15 = ref_q["stage15"][0, :, :4].float()  # [4 groups][4 heads][256] = q15[..., order] * 16
        q15 = torch.empty(4, 4, 256)
        q15[..., order] = st15 / 16
        order4 = torch.arange(256).reshape(32, 8).T.flatten()
        qsm = torch.empty(4, 4, 256)
        qsm[..., order4] = ref_q["matrix"][0, :, 32:36].float()
        data[f"q{qi}_ref_q15"] = bits(q15.bfloat16())
        data[f"q{qi}_ref_qs"] = bits(qsm.bfloat16())
        data[f"q{qi}_ref_norm"] = ref_q["norm"].double().numpy()
        data[f"q{qi}_ref_qsum"] = ref_q["query_sum"].numpy()

        res = [O.run_cell(ocells[g], qb[4 * g:4 * g + 4]) for g in range(4)]
        out = np.zeros((16, 256), np.uint16)
        for j in range(16):
            g, h = divmod(j, 4)
            out[j] = O.attention(qb[j], k8[g], v8[g], O.attention_keys(CONTEXT, SINK, LOCAL, res[g]["final_ids"][h]))
        data[f"q{qi}_final_ids"] = np.stack([r["final_ids"] for r in res])
        data[f"q{qi}_out"] = out

        for g, (c, r) in enumerate(zip(cells, res)):
            tags = torch.from_numpy(r["tags"].astype(np.int64))
            coarse_ids = tags & 0x0FFFFFFF
            head_mask = (tags >> 28) & 15
            n = len(tags)
            # Fine: reference tree top-P over the fused [bf16 | u16 position] keys
            fused = ((r["fine_scores"].astype(np.uint32) << 16) | (np.arange(n, dtype=np.uint32) & 0xFFFF))
            scores = torch.from_numpy(fused.view(np.float32).copy())
            allowed = torch.stack([((head_mask >> h) & 1).bool() for h in range(4)])
            cohorts = schedule([n], cohort_counts=(7,))
            tp = tree_top_p(scores, allowed, int(c["p"]), cohorts)
            data[f"q{qi}_{g}_ref_tree_top_p"] = np.sort(tp.numpy(), axis=1)
            sel, _, status = distributed_union_reference(coarse_ids, head_mask, tp)
            data[f"q{qi}_{g}_ref_fine_union"] = sel.numpy().astype(np.int32)
            pool = encounter_union(c, sel)
            data[f"q{qi}_{g}_ref_pool"] = pool.numpy().astype(np.int32)
            data[f"q{qi}_{g}_ref_expand_lists"] = expand_lists(c, sel).numpy().astype(np.int32)
            # Stage-1.5 frontier: each of the six pool shards (24 workers of
            # 32-position chunks, four per shard) ranks its own scores, and
            # the reference's tree merges the six rows into the top 2048
            npool = len(r["pool"])
            chunks = (npool + 31) // 32
            frontier = []
            for h in range(4):
                sc = O.ord16(r["s15_scores"][h]).astype(np.int64)
                rows = []
                for sh in range(6):
                    lo = (chunks * (4 * sh) // 24) * 32
                    hi = min((chunks * (4 * sh + 4) // 24) * 32, npool)
                    rows.append(sorted(sc[lo:hi].tolist(), reverse=True)[:2048])
                frontier.append(merge_tree_reference(rows, k=2048))
            data[f"q{qi}_{g}_ref_s15_frontier"] = np.asarray(frontier, dtype=np.uint16)
            by_source, parts = source_union_reference(
                [row[:1600] for row in r["s15_top"].tolist()], 13056, 6, 1600)
            data[f"q{qi}_{g}_ref_s15_union"] = np.asarray([x for p in parts for x in p], dtype=np.int32)
            meta.setdefault("fine_status", []).append(int(status))

    data["metadata"] = np.array(json.dumps(meta))
    np.savez_compressed(OUT, **data)
    print(OUT, OUT.stat().st_size)


if __name__ == "__main__":
    main()
