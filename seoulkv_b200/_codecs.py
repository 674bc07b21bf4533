"""Static index codec and the NPZ index file format.

The on-disk format is the reference's (version 4, with version-3 grouped
fixtures still readable), so an index dumped by either implementation loads
in the other.  Field names, dtypes and the per-cell ``"{i}_{name}"`` key
scheme are therefore identical to ``src/seoulkv4/_codecs/index.py:219-230``
(dump) and ``:130-169`` (load); the code below is this package's own.

Centroid codec ("group-scale-32-v1", reference ``_codecs/index.py:233-313``):
centroids are reordered by their row range, each group of 32 rows shares one
scale ``s = max|c| * 16/15``, and every coordinate becomes a 4-bit code
``clamp(floor((c + s) / (s/8)), 0, 15)`` stored as two 2-bit planes
(``upper = code >> 2``, ``lower = code & 3``, four codes per byte,
little-endian).  Posting lists move with their centroid.
"""

from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path
from tempfile import NamedTemporaryFile

import numpy as np
import torch

INDEX_VERSION = 4
LEGACY_VERSION = 3
GROUP = 32
CODEC = "group-scale-32-v1"
CENTROID_CODEC = "fp16-scale-odd-v1"
QUERY_FIELDS = frozenset({"q", "query_hash", "coarse_ids", "head_mask"})


def fingerprint(t: torch.Tensor) -> str:
    """SHA-256 of a tensor's raw little-endian bytes (K-cache identity)."""
    return hashlib.sha256(t.contiguous().view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def pack2(codes: torch.Tensor) -> torch.Tensor:
    """Four 2-bit codes per byte, first code in the low bits."""
    c = codes.to(torch.int64).reshape(*codes.shape[:-1], -1, 4)
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).to(torch.uint8)


def unpack2(packed: torch.Tensor) -> torch.Tensor:
    p = packed.to(torch.int64)
    return torch.stack([(p >> s) & 3 for s in (0, 2, 4, 6)], dim=-1).flatten(-2)


def coarse_metadata(source: torch.Tensor, upper: torch.Tensor, scale: torch.Tensor) -> dict:
    """Two-bit centroid operands and the residual norm used by the coarse interval.

    The norm is a float32 reduction whose rounding depends on the summation
    order, so it is always taken on the host (the reference's own order):
    a device encode sends the [nc, 256] residuals over and reduces them here."""
    odd = 2 * unpack2(upper).float() - 3
    full = scale.float()[:, None] * odd / 4
    return {
        "coarse2": full.half(),
        "coarse_odd": odd.bfloat16(),
        "coarse_residual_norm": (source.float() - full).cpu().norm(dim=-1).half(),
    }


def encode_group_scale_cell(cell: dict) -> dict:
    """Quantise a cell's FP16 centroids and remap its CSR lists (query-free).

    Runs on the device that holds the centroids (a CUDA build encodes on the
    GPU: every step is elementwise, a stable sort, an integer scan, or an
    exact max, so the codes, planes, scales and lists are the bytes the host
    computes; the residual norm's float32 sum is taken on the host, see
    coarse_metadata); the returned cell holds CPU tensors."""
    original = cell.get("coarse_centroids", cell["centroids"])
    dev = original.device
    x = original.float()
    nc, d = x.shape
    if d != 256 or nc % GROUP:
        raise ValueError(f"group-scale cell needs [multiple of {GROUP}, 256], got {tuple(x.shape)}")
    ranges = cell.get("scale")
    if ranges is None:
        ranges = (x.abs().amax(-1) * (16 / 15)).clamp_min(1e-9)
    order = torch.argsort(ranges.float(), stable=True)
    x = x[order]
    group_scale = (x.reshape(-1, GROUP, d).abs().amax(dim=(1, 2)) * (16 / 15)).clamp_min(1e-9)
    scale = group_scale.repeat_interleave(GROUP)
    code = ((x + scale[:, None]) / (scale[:, None] / 8)).floor().clamp(0, 15).to(torch.uint8)
    odd = (2 * code.float() - 15).bfloat16()
    decoded = (scale[:, None] * odd.float() / 16).half()
    levels = (
        (group_scale[:, None, None] * (2 * torch.arange(16, device=dev).float()[None, None] - 15) / 16)
        .expand(-1, GROUP, -1)
        .reshape(nc, 16)
        .half()
    )
    upper, lower = pack2(code >> 2), pack2(code & 3)

    offsets = cell["offsets"].to(dev).long()
    lengths = offsets[1:] - offsets[:-1]
    owner = torch.repeat_interleave(torch.arange(nc, device=dev), lengths)
    rank = torch.empty_like(order)
    rank[order] = torch.arange(nc, device=dev)
    posting_order = torch.argsort(rank[owner], stable=True)
    new_offsets = torch.cat((torch.zeros(1, dtype=torch.long, device=dev), lengths[order].cumsum(0)))
    group_fine_scale = (group_scale / 16).half()
    fields = dict(
        coarse_centroids=x.to(original.dtype),
        centroids=decoded.bfloat16(),
        upper=upper,
        lower=lower,
        scale=scale,
        decoded=decoded.bfloat16(),
        fine_scale=group_fine_scale.repeat_interleave(GROUP),
        group_fine_scale=group_fine_scale,
        levels=levels,
        centroid_codec=CENTROID_CODEC,
        offsets=new_offsets.to(cell["offsets"].dtype),
        values=cell["values"].to(dev)[posting_order],
        max_codec_error=float((x - decoded.float()).abs().max()),
        group_scale_size=GROUP,
        summary_codec=CODEC,
        **coarse_metadata(x, upper, scale),
    )
    out = dict(cell)
    out.update({k: v.cpu() if isinstance(v, torch.Tensor) else v for k, v in fields.items()})
    return out


def validate_static_cell(c: dict) -> None:
    """Structural checks of one cell: shapes, finiteness, spill-2 CSR invariants."""
    nc, d = c["centroids"].shape
    if d != 256 or not 0 < int(c["p"]) <= min(nc, 1536):
        raise ValueError("index cell: bad centroid shape or nprobe")
    if not torch.isfinite(c["centroids"].float()).all():
        raise ValueError("index cell: non-finite centroids")
    if tuple(c["upper"].shape) != (nc, 64) or tuple(c["lower"].shape) != (nc, 64):
        raise ValueError("index cell: bad code planes")
    if tuple(c["coarse2"].shape) != (nc, d) or tuple(c["coarse_odd"].shape) != (nc, d):
        raise ValueError("index cell: bad coarse operands")
    rn = c["coarse_residual_norm"]
    if tuple(rn.shape) != (nc,) or not torch.isfinite(rn.float()).all():
        raise ValueError("index cell: bad coarse residual norms")
    off, vals = c["offsets"].long(), c["values"].long()
    if len(off) != nc + 1 or off[0] != 0 or off[-1] != len(vals) or (off[1:] < off[:-1]).any():
        raise ValueError("index cell: invalid CSR offsets")
    context = int(c["context"])
    if ((vals < 0) | (vals >= context)).any():
        raise ValueError("index cell: CSR token id out of range")
    counts = torch.bincount(vals, minlength=context)
    r0, r1, spill = int(c["r0"]), int(c["r1"]), int(c["spill"])
    if not (counts[r0:r1] == spill).all() or counts[:r0].sum() or counts[r1:].sum():
        raise ValueError("index cell: every retrieval token must be in exactly `spill` lists")
    rows = torch.repeat_interleave(torch.arange(nc), off.diff())
    entries = (rows * context + vals).sort().values
    if (entries[1:] == entries[:-1]).any():
        raise ValueError("index cell: duplicate token inside one list")


def require_group_scale_cell(cell: dict) -> dict:
    """Check the persisted group-scale summary without transforming it."""
    if cell.get("summary_codec") != CODEC or cell.get("group_scale_size") != GROUP:
        raise ValueError("index cell is not a group-scale-32 summary; rebuild it")
    nc = len(cell["centroids"])
    if nc % GROUP:
        raise ValueError("index cell has a partial centroid group")
    gs = cell.get("group_fine_scale")
    if not isinstance(gs, torch.Tensor) or tuple(gs.shape) != (nc // GROUP,):
        raise ValueError("index cell has an invalid group scale table")
    fs = cell.get("fine_scale")
    if not isinstance(fs, torch.Tensor) or tuple(fs.shape) != (nc,):
        raise ValueError("index cell is missing its per-centroid scale view")
    if not torch.equal(fs.reshape(-1, GROUP), gs[:, None].expand(-1, GROUP)):
        raise ValueError("index cell scale views disagree")
    return cell


def ensure_coarse_metadata(cell: dict) -> dict:
    """Derive coarse operands for old fixtures that predate them (in memory only)."""
    if all(k in cell for k in ("coarse2", "coarse_odd", "coarse_residual_norm")):
        return cell
    source = cell.get("coarse_centroids", cell["centroids"])
    if "scale" not in cell:
        cell = dict(cell, scale=(source.float().abs().amax(-1) * (16 / 15)).clamp_min(1e-9))
    return dict(cell, **coarse_metadata(source, cell["upper"], cell["scale"]))


def load_index(path) -> tuple[list[dict], dict]:
    """Read a version-4 index or a version-3 grouped fixture (query fields dropped)."""
    with np.load(path, allow_pickle=False) as z:
        meta = json.loads(str(z["metadata"]))
        version = meta.get("version")
        if version not in (1, 2, LEGACY_VERSION, INDEX_VERSION):
            raise ValueError("unsupported index file version")
        static = version == INDEX_VERSION
        bf16 = set(meta.get("bf16_arrays", ())) if static else set()
        if not bf16.issubset(z.files):
            raise ValueError("index file is missing a declared BF16 array")
        cells = []
        for i, info in enumerate(meta["cells"]):
            c = dict(info)
            prefix = f"{i}_"
            for name in z.files:
                if not name.startswith(prefix):
                    continue
                t = torch.from_numpy(z[name])
                if name in bf16:
                    if t.dtype != torch.int16:
                        raise ValueError(f"invalid BF16 storage for {name}")
                    t = t.view(torch.bfloat16)
                c[name[len(prefix):]] = t
            if static:
                if QUERY_FIELDS.intersection(c):
                    raise ValueError("static index contains query fields")
            else:
                c = ensure_coarse_metadata(c)
                c = {k: v for k, v in c.items() if k not in QUERY_FIELDS}
            validate_static_cell(c)
            if version >= LEGACY_VERSION:
                require_group_scale_cell(c)
            cells.append(c)
    return cells, meta


def dump_index(path, cells: list[dict], meta: dict) -> None:
    """Write a query-free version-4 NPZ; the target is replaced only on success."""
    path = Path(path)
    data, rows, bf16 = {}, [], []
    for i, cell in enumerate(cells):
        scalars = {}
        for name, value in cell.items():
            if name in QUERY_FIELDS:
                continue
            if isinstance(value, torch.Tensor):
                key = f"{i}_{name}"
                if value.dtype == torch.bfloat16:
                    value = value.view(torch.int16)
                    bf16.append(key)
                data[key] = value.cpu().numpy()
            else:
                scalars[name] = value
        rows.append(scalars)
    data["metadata"] = np.array(json.dumps(dict(meta, version=INDEX_VERSION, cells=rows, bf16_arrays=bf16)))
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = NamedTemporaryFile(dir=path.parent, prefix=f".{path.name}.", delete=False)
    try:
        with tmp:
            np.savez(tmp, **data)
        os.replace(tmp.name, path)
    finally:
        Path(tmp.name).unlink(missing_ok=True)
