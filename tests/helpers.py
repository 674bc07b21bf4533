"""Shared test helpers: seeded cases and oracle runs (test infrastructure)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O
from seoulkv_b200 import synthetic
from seoulkv_b200.index import SeoulKV4Index, device_view


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def attend_rows(q_bits, k, v, keys):
    """The oracle's attention of one query head over rows ``keys`` of BF16
    K/V [T, 256], decoding only those rows to FP8 (a whole long cache in
    float64 would take gigabytes)."""
    idx = torch.from_numpy(np.asarray(keys, dtype=np.int64))
    kk = O.fp8_e4m3(k.index_select(0, idx).float().numpy())
    vv = O.fp8_e4m3(v.index_select(0, idx).float().numpy())
    return O.attention(q_bits, kk, vv, np.arange(len(keys)))


class Case:
    """A seeded synthetic cache + index + queries, with oracle results per query."""

    def __init__(self, context=8192, nprobe=128, seed=11, components=256, index=None, sink=128, local=256):
        self.context, self.sink, self.local = context, sink, local
        self.k, self.v, self.mixes = synthetic.make_kv(context, seed=seed, components=components)
        self.index = index or SeoulKV4Index.build(self.k, self.v, sink=sink, local=local, nprobe=nprobe)
        self.planes = O.key_codec(bits(self.k))
        self._k8 = self._v8 = None

    def cells(self, nprobe=None):
        scales, p2, r2, r4 = self.planes
        out = []
        for g, c in enumerate(self.index.cells()):
            dv = device_view(c, None if nprobe is None else nprobe[g])
            out.append(O.CellInputs(
                nc=dv["nc"], nprobe=dv["nprobe"], lam=dv["lam"], upper=dv["upper"], lower=dv["lower"],
                coarse_scale4=dv["coarse_scale4"], fine_scale=dv["fine_scale"], resid_bf16=dv["resid_bf16"],
                offsets=dv["offsets"], values=dv["values"], context=self.context,
                prefix2=p2[g], residual2=r2[g], residual4=r4[g], key_scale=scales[g]))
        return out

    def query(self, seed):
        return synthetic.make_query(self.context, self.mixes, seed=seed)

    def kv8(self):
        if self._k8 is None:
            self._k8 = O.fp8_e4m3(self.k.float().numpy())
            self._v8 = O.fp8_e4m3(self.v.float().numpy())
        return self._k8, self._v8

    def oracle(self, q, capacity=13056, nprobe=None):
        qb = bits(q).reshape(16, 256)
        res = [O.run_cell(c, qb[4 * g:4 * g + 4], capacity=capacity) for g, c in enumerate(self.cells(nprobe))]
        out = np.zeros((16, 256), np.uint16)
        for j in range(16):
            g, h = divmod(j, 4)
            keys = O.attention_keys(self.context, self.sink, self.local, res[g]["final_ids"][h])
            out[j] = attend_rows(qb[j], self.k[g], self.v[g], keys)
        return res, out


class ShardCase(Case):
    """One shard of a sequence-sharded synthetic cache (``ShardPlan``)."""

    def __init__(self, plan, nprobe=128, seed=31, components=64):
        self.plan = plan
        self.context, self.sink, self.local = plan.context, plan.shard_sink, plan.shard_local
        self.k, self.v, self.mixes = synthetic.make_kv_range(plan.total, plan.begin, plan.end, seed=seed,
                                                             components=components)
        self.index = SeoulKV4Index.build(self.k, self.v, sink=self.sink, local=self.local, nprobe=nprobe)
        self.planes = O.key_codec(bits(self.k))
        self._k8 = self._v8 = None

    def reference_view(self):
        k8, v8 = self.kv8()
        return dict(cells=self.cells(), begin=self.plan.begin, context=self.context, sink=self.sink,
                    local=self.local, k8=k8, v8=v8)


# ------------------------------------------------------------ golden data

GOLDEN_DIR = __import__("pathlib").Path(__file__).resolve().parent / "golden"
GOLDEN = GOLDEN_DIR / "golden_t8192.npz"
# every fixture tests/golden/make_golden.py wrote: the default one and the
# reference's smallest context with other zones and another probe budget
GOLDEN_FILES = ("golden_t8192.npz", "golden_t6400.npz")


class Golden:
    """The reference-built fixture (tests/golden/make_golden.py) + regenerated K/V."""

    def __init__(self, name: str = "golden_t8192.npz"):
        import json

        z = np.load(GOLDEN_DIR / name, allow_pickle=False)
        self.z = {k: z[k] for k in z.files}
        self.meta = json.loads(str(self.z["metadata"]))
        self.context = self.meta["context"]
        self.sink, self.local = self.meta["sink"], self.meta["local"]
        self.k, self.v, self.mixes = synthetic.make_kv(self.context, seed=self.meta["kv_seed"])
        self.queries = [synthetic.make_query(self.context, self.mixes, seed=s) for s in self.meta["q_seeds"]]

    def views(self):
        """Engine/oracle cell views of the reference-built index."""
        from seoulkv_b200.index import posting_mates

        out = []
        for g, info in enumerate(self.meta["cells"]):
            z = self.z
            upper, lower = z[f"{g}_upper"], z[f"{g}_lower"]
            nc = upper.shape[0]
            scale = z[f"{g}_scale"].astype(np.float32).reshape(-1, 32)
            gfs = z[f"{g}_group_fine_scale"].view(np.float16).astype(np.float32)
            resid = torch.from_numpy(z[f"{g}_coarse_residual_norm"].view(np.float16).copy()).bfloat16()
            offsets = z[f"{g}_offsets"].astype(np.int32)
            values = z[f"{g}_values"].astype(np.int32)
            out.append(dict(
                nc=nc, nprobe=int(info["p"]), lam=float(info["lam"]), upper=upper, lower=lower,
                coarse_scale4=(scale[:, 0] / np.float32(4)).astype(np.float32), fine_scale=gfs,
                resid_bf16=resid.view(torch.int16).numpy().view(np.uint16), offsets=offsets, values=values,
                mates=posting_mates(offsets, values)))
        return out

    def oracle_cells(self):
        scales, p2, r2, r4 = O.key_codec(bits(self.k))
        return [O.CellInputs(nc=v["nc"], nprobe=v["nprobe"], lam=v["lam"], upper=v["upper"], lower=v["lower"],
                             coarse_scale4=v["coarse_scale4"], fine_scale=v["fine_scale"],
                             resid_bf16=v["resid_bf16"], offsets=v["offsets"], values=v["values"],
                             context=self.context, prefix2=p2[g], residual2=r2[g], residual4=r4[g],
                             key_scale=scales[g]) for g, v in enumerate(self.views())]


# ------------------------------------------------------------ cache append


class AppendCase:
    """A cache built on its first ``context`` tokens and grown by appends up to
    ``total`` tokens, with the oracle's view of every intermediate context."""

    def __init__(self, context=8192, total=8192 + 700, nprobe=128, seed=23, components=256, sink=128, local=256,
                 kv=None):
        self.context, self.total, self.sink, self.local = context, total, sink, local
        if kv is None:
            kv = synthetic.make_kv(total, seed=seed, components=components)
        self.k_full, self.v_full, self.mixes = kv
        assert self.k_full.shape[1] == total
        self.k = self.k_full[:, :context].contiguous()
        self.v = self.v_full[:, :context].contiguous()
        self.index = SeoulKV4Index.build(self.k, self.v, sink=sink, local=local, nprobe=nprobe)
        self.kb = bits(self.k_full)
        self.scales = O.key_codec(bits(self.k))[0]
        self.planes = [O.encode_planes(self.kb[g], self.scales[g]) for g in range(4)]
        self.views = [device_view(c) for c in self.index.cells()]
        first = context - local
        self.labels = [O.assign_spill2(self.kb[g, first:total], v["upper"], v["lower"], v["fine_scale"])
                       for g, v in enumerate(self.views)]
        self._k8 = self._v8 = None

    def appended(self, a, b):
        """K and V of tokens [a, b) as BF16 [4, b-a, 256]."""
        return self.k_full[:, a:b].contiguous(), self.v_full[:, a:b].contiguous()

    def csr(self, g, t):
        """Oracle (offsets, values, mates) of KV head g at context t."""
        v = self.views[g]
        first = self.context - self.local
        entering = np.arange(first, t - self.local)
        return O.append_postings(v["offsets"], v["values"], v["mates"], entering, self.labels[g][:len(entering)])

    def cells(self, t, nprobe=None):
        out = []
        for g, v in enumerate(self.views):
            off, vals, _ = self.csr(g, t)
            p2, r2, r4 = self.planes[g]
            out.append(O.CellInputs(
                nc=v["nc"], nprobe=v["nprobe"] if nprobe is None else nprobe[g], lam=v["lam"], upper=v["upper"],
                lower=v["lower"], coarse_scale4=v["coarse_scale4"], fine_scale=v["fine_scale"],
                resid_bf16=v["resid_bf16"], offsets=off, values=vals, context=t, prefix2=p2[:t],
                residual2=r2[:t], residual4=r4[:t], key_scale=self.scales[g]))
        return out

    def query(self, t, seed):
        return synthetic.make_query(t, self.mixes, seed=seed)

    def kv8(self):
        if self._k8 is None:
            self._k8 = O.fp8_e4m3(self.k_full.float().numpy())
            self._v8 = O.fp8_e4m3(self.v_full.float().numpy())
        return self._k8, self._v8

    def reference_view(self, t, begin):
        """This cache at context t as shard [begin, begin + t) of a sharded layer (oracle view)."""
        k8, v8 = self.kv8()
        return dict(cells=self.cells(t), begin=begin, context=t, sink=self.sink, local=self.local,
                    k8=k8[:, :t], v8=v8[:, :t])

    def oracle(self, q, t, capacity=13056):
        qb = bits(q).reshape(16, 256)
        res = [O.run_cell(c, qb[4 * g:4 * g + 4], capacity=capacity) for g, c in enumerate(self.cells(t))]
        k8, v8 = self.kv8()
        out = np.zeros((16, 256), np.uint16)
        for j in range(16):
            g, h = divmod(j, 4)
            keys = O.attention_keys(t, self.sink, self.local, res[g]["final_ids"][h])
            out[j] = O.attention(qb[j], k8[g], v8[g], keys)
        return res, out
