"""Query-independent index of four KV heads (build, load, dump).

Mirrors the reference's ``SeoulKV4Index`` (``src/seoulkv4/index.py:38-179``):
same arguments, defaults, validation and errors.  The clustering is this
package's own (``_clustering.py``); the stored cell format is the
reference's NPZ v4 so files move between the two implementations.
"""

from __future__ import annotations

import math
from numbers import Real
from pathlib import Path

import numpy as np
import torch

from seoulkv_b200 import _clustering, _codecs
from seoulkv_b200.config import (
    DEFAULT_NPROBE, MAX_CENTROIDS, MAX_CONTEXT, MIN_CONTEXT, N_KV_HEADS, STAGE15_M, TOPK,
    validate_nprobe,
)


class AttentionZones:
    """Disjoint sink / retrieval / local ranges (reference attention_zones.py:7-75)."""

    def __init__(self, context: int, sink: int, local: int):
        if context <= 0 or min(sink, local) < 0:
            raise ValueError("require positive context and nonnegative sink/local")
        if sink + local > context:
            raise ValueError("sink and local must be disjoint and inside context")
        self.context, self.sink, self.local = int(context), int(sink), int(local)

    def __eq__(self, other):
        return isinstance(other, AttentionZones) and (
            (self.context, self.sink, self.local) == (other.context, other.sink, other.local))

    @property
    def local_begin(self) -> int:
        return self.context - self.local

    def count(self, retrieval: int = TOPK) -> int:
        if not 0 <= retrieval <= self.local_begin - self.sink:
            raise ValueError("retrieval count exceeds the indexed range")
        return self.sink + self.local + retrieval

    def metadata(self, retrieval: int = TOPK) -> dict:
        total = self.count(retrieval)
        return dict(context=self.context, sink=self.sink, local=self.local,
                    retrieval_begin=self.sink, retrieval_end=self.local_begin,
                    retrieval_tokens=retrieval, attention_tokens=total,
                    chunk_keys=128, chunks=(total + 127) // 128)


def posting_mates(offsets: np.ndarray, values: np.ndarray) -> np.ndarray:
    """For every CSR posting, the other list holding the same token (or -1).

    Rejects tokens listed more than twice or twice in one list, like the
    reference's ownership check (``_kernels/common/seoulkv4_cluster_blocks.py:10-32``).
    """
    off = np.asarray(offsets, dtype=np.int64)
    ids = np.asarray(values, dtype=np.int64)
    owner = np.repeat(np.arange(len(off) - 1, dtype=np.int64), np.diff(off))
    order = np.argsort(ids, kind="stable")
    sid = ids[order]
    if len(ids) > 2 and ((sid[:-2] == sid[1:-1]) & (sid[1:-1] == sid[2:])).any():
        raise ValueError("a token is listed more than twice")
    pair = np.flatnonzero(sid[:-1] == sid[1:])
    a, b = order[pair], order[pair + 1]
    if (owner[a] == owner[b]).any():
        raise ValueError("a token is listed twice in one cluster")
    mates = np.full(len(ids), -1, dtype=np.int32)
    mates[a] = owner[b]
    mates[b] = owner[a]
    return mates


class SeoulKV4Index:
    """CPU-resident IVF summary of four ordered KV heads."""

    def __init__(self, cells, metadata):
        if len(cells) != N_KV_HEADS:
            raise ValueError("SeoulKV4 requires four ordered index cells")
        context = int(cells[0]["context"])
        zones = []
        for cell in cells:
            if int(cell["context"]) != context:
                raise ValueError("index cells disagree on the context length")
            zones.append(AttentionZones(context, int(cell["r0"]), context - int(cell["r1"])))
        if any(z != zones[0] for z in zones):
            raise ValueError("all index cells must use the same sink/local zones")
        self._zones = zones[0]
        self._zones.count()
        self._cells = tuple(
            {k: v for k, v in _codecs.require_group_scale_cell(c).items() if k not in _codecs.QUERY_FIELDS}
            for c in cells
        )
        self._nprobe_source = metadata.get("nprobe_source")

    # ------------------------------------------------------------ file I/O

    @classmethod
    def load(cls, path: str | Path, *, nprobe=None) -> "SeoulKV4Index":
        """Read an index file; ``nprobe`` optionally overrides the saved probe budget."""
        cells, meta = _codecs.load_index(path)
        if nprobe is not None:
            if len(cells) != N_KV_HEADS:
                raise ValueError("SeoulKV4 requires four ordered index cells")
            probes = validate_nprobe(nprobe, min(len(c["centroids"]) for c in cells))
            cells = [dict(c, p=p) for c, p in zip(cells, probes, strict=True)]
            meta = dict(meta, nprobe_source="load override")
        return cls(cells, meta)

    def dump(self, path: str | Path) -> None:
        """Save as an NPZ (version 4) that ``load`` (here or in the reference) reopens."""
        _codecs.dump_index(path, list(self._cells), {"nprobe_source": self._nprobe_source})

    # --------------------------------------------------------------- build

    @classmethod
    def build(cls, k: torch.Tensor, v: torch.Tensor | None = None, *, sink: int = 128,
              local: int = 256, nprobe=DEFAULT_NPROBE, lam: float = 0.0625, seed: int = 0,
              build_device: str | torch.device = "cpu") -> "SeoulKV4Index":
        """Index CPU BF16 post-RoPE K [4, T, 256].  V is only checked for layout."""
        if not (isinstance(k, torch.Tensor) and k.device.type == "cpu" and k.dtype == torch.bfloat16
                and k.ndim == 3 and k.shape[0] == N_KV_HEADS and k.shape[2] == 256):
            raise ValueError("expected CPU BF16 post-RoPE K [4,T,256]")
        if v is not None and not (isinstance(v, torch.Tensor) and v.device == k.device
                                  and v.dtype == k.dtype and v.shape == k.shape):
            raise ValueError("V must match K's shape, dtype, and CPU device")
        context = k.shape[1]
        if not MIN_CONTEXT <= context <= MAX_CONTEXT or context % 4:
            raise ValueError("unsupported context for the fixed SeoulKV4 profile")
        if type(sink) is not int or type(local) is not int:
            raise ValueError("sink and local must be integer token counts")
        zones = AttentionZones(context, sink, local)
        retrieval = zones.local_begin - sink
        if retrieval < STAGE15_M:
            raise ValueError(f"retrieval zone needs at least {STAGE15_M} keys for the fixed Stage-1.5 profile")
        nc = _clustering.centroid_count(retrieval)
        if nc > MAX_CENTROIDS:
            raise ValueError("centroid count exceeds the Fine selector's 16-bit positions")
        probes = validate_nprobe(nprobe, nc)
        if isinstance(lam, bool) or not isinstance(lam, Real) or not (math.isfinite(lam) and lam >= 0):
            raise ValueError("lam must be finite and nonnegative")
        if type(seed) is not int or not 0 <= seed <= 2**63 - 1:
            raise ValueError("seed must be a nonnegative signed 64-bit integer")
        device = torch.device(build_device)
        if device.type not in ("cpu", "cuda"):
            raise ValueError("build_device must be a PyTorch CPU or CUDA device")
        if device.type == "cuda" and not torch.cuda.is_available():
            raise ValueError("build_device requests CUDA, but PyTorch CUDA is unavailable")
        cells = [build_cell(k[h], p=p, lam=float(lam), seed=seed, r0=sink, r1=zones.local_begin,
                            device=device) for h, p in enumerate(probes)]
        return cls(cells, {"nprobe_source": "explicit (build)"})

    # ----------------------------------------------------------- accessors

    def _check_keys(self, k: torch.Tensor) -> None:
        for i, cell in enumerate(self._cells):
            if _codecs.fingerprint(k[i]) != cell["key_hash"]:
                raise ValueError(f"Stage-I index K fingerprint mismatch at cell {i}")

    @property
    def zones(self) -> AttentionZones:
        return self._zones

    @property
    def nprobe(self) -> tuple[int, ...]:
        return tuple(int(c["p"]) for c in self._cells)

    def cells(self) -> tuple[dict, ...]:
        return self._cells

    def metadata(self) -> dict:
        return {
            **self._zones.metadata(),
            "summary_codec": _codecs.CODEC,
            "nprobe": [int(c["p"]) for c in self._cells],
            "lambda": [float(c["lam"]) for c in self._cells],
            "key_hashes": [c["key_hash"] for c in self._cells],
            "nprobe_source": self._nprobe_source,
        }


@torch.no_grad()
def build_cell(k: torch.Tensor, *, p: int, lam: float, seed: int, r0: int, r1: int,
               device=None) -> dict:
    """Cluster one KV head's retrieval range [r0, r1) into a group-scale cell."""
    nc = _clustering.centroid_count(r1 - r0)
    if not 0 <= r0 < r1 <= len(k) or r1 - r0 < nc or not 0 < p <= nc:
        raise ValueError("not enough retrieval keys for spill2 / requested nprobe")
    x = k[r0:r1].to(device=device or k.device, dtype=torch.float32)
    if not torch.isfinite(x).all():
        raise ValueError("retrieval keys must be finite")
    x = _clustering._normalise(x)
    centroids, labels, stats = _clustering.build_ivf(x, nc, seed)
    offsets, values = _clustering.to_csr(labels, nc)
    # the codec runs where the clustering ran (the GPU for a CUDA build)
    cell = _codecs.encode_group_scale_cell(dict(
        centroids=_clustering.midrise4(centroids).half(),
        offsets=offsets,
        values=values + r0,
        context=len(k), r0=r0, r1=r1, spill=2, p=int(p), lam=float(lam), seed=int(seed),
        key_hash=_codecs.fingerprint(k.cpu().bfloat16()),
        builder=stats,
    ))
    _codecs.validate_static_cell(cell)
    return cell


def device_view(cell: dict, nprobe: int | None = None) -> dict:
    """The arrays the CUDA engine (and the oracle) consume for one cell."""
    nc = int(cell["centroids"].shape[0])
    scale = cell["scale"].float().reshape(-1, 32)
    if not torch.equal(scale, scale[:, :1].expand_as(scale)):
        raise ValueError("coarse scoring needs one shared scale per 32 centroids")
    offsets = cell["offsets"].to(torch.int64).numpy()
    values = cell["values"].to(torch.int64).numpy()
    return dict(
        nc=nc,
        nprobe=int(cell["p"] if nprobe is None else nprobe),
        lam=float(cell["lam"]),
        upper=cell["upper"].numpy().astype(np.uint8),
        lower=cell["lower"].numpy().astype(np.uint8),
        coarse_scale4=(scale[:, 0] / 4).numpy().astype(np.float32),
        fine_scale=cell["group_fine_scale"].float().numpy().astype(np.float32),
        resid_bf16=cell["coarse_residual_norm"].bfloat16().view(torch.int16).numpy().view(np.uint16),
        offsets=offsets.astype(np.int32),
        values=values.astype(np.int32),
        mates=posting_mates(offsets, values),
    )
