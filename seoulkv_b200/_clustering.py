"""Spill-2 IVF construction for one KV head (host or CUDA PyTorch).

Two-level spherical k-means: a coarse codebook splits the unit-normalised
retrieval keys into buckets, each bucket receives a share of the ``nc``
leaves proportional to its population (at least two, so that every key can
be listed twice), and a local Lloyd solve places the leaves.  Every key is
then posted to its two best leaves inside its bucket, which gives the
spill-2 CSR the decode path expects (each retrieval token in exactly two
distinct lists), as the reference index builder does
(``src/seoulkv4/_clustering.py:73-236``, ``src/seoulkv4/_index_build.py:22-59``).

Randomness comes only from CPU ``torch.Generator`` objects seeded by ``seed``,
so CPU builds are reproducible; CUDA builds can differ in argmax ties.
"""

from __future__ import annotations

import math

import torch

GROUP = 32
_SCORE_ELEMENTS = 1 << 24  # bound on one chunk of the key x centroid score matrix


def centroid_count(retrieval_tokens: int) -> int:
    """About four keys per centroid before spill, padded to whole 32-centroid groups."""
    return math.ceil(retrieval_tokens / (4 * GROUP)) * GROUP


def _normalise(x: torch.Tensor) -> torch.Tensor:
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-9)


def _assign(x: torch.Tensor, c: torch.Tensor) -> torch.Tensor:
    rows = max(1, _SCORE_ELEMENTS // max(1, c.shape[0]))
    out = torch.empty(x.shape[0], dtype=torch.long, device=x.device)
    for s in range(0, x.shape[0], rows):
        out[s:s + rows] = (x[s:s + rows] @ c.t()).argmax(1)
    return out


def _lloyd(x: torch.Tensor, c: torch.Tensor, iters: int) -> torch.Tensor:
    k = c.shape[0]
    for _ in range(iters):
        lab = _assign(x, c)
        sums = torch.zeros_like(c).index_add_(0, lab, x)
        cnt = torch.bincount(lab, minlength=k)
        c = _normalise(torch.where((cnt > 0)[:, None], sums, c))
    return c


def _seeded_pick(n: int, k: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n, generator=g)
    if k > n:
        perm = perm.repeat((k + n - 1) // n)
    return perm[:k].to(device)


def _leaf_shares(counts: torch.Tensor, nc: int) -> torch.Tensor:
    """Split nc leaves over buckets: proportional, largest remainder, >= 2 per live bucket."""
    counts = counts.cpu().long()
    live = counts > 0
    total = int(counts.sum())
    raw = counts.double() * (nc / max(total, 1))
    share = torch.floor(raw).long()
    share = torch.where(live, share.clamp_min(2), torch.zeros_like(share))
    diff = nc - int(share.sum())
    if diff > 0:
        frac = (raw - share.double()).masked_fill(~live, -math.inf)
        order = torch.argsort(frac, descending=True, stable=True)
        i = 0
        while diff > 0:
            b = int(order[i % len(order)])
            if live[b]:
                share[b] += 1
                diff -= 1
            i += 1
    elif diff < 0:
        # take leaves back from the buckets with most spare leaves above two
        while diff < 0:
            spare = (share - 2).masked_fill(~live, -1)
            b = int(torch.argmax(spare))
            if int(spare[b]) <= 0:
                raise ValueError("not enough leaves for two distinct lists per bucket")
            take = min(-diff, int(spare[b]))
            share[b] -= take
            diff += take
    return share


@torch.no_grad()
def build_ivf(keys: torch.Tensor, nc: int, seed: int, *, coarse: int = 128,
              coarse_iters: int = 5, leaf_iters: int = 8):
    """Cluster unit keys [R, 256] into nc leaves with two postings per key.

    Returns (centroids [nc,256] f32 unit rows, labels [R,2] long, stats dict).
    """
    n, d = keys.shape
    device = keys.device
    if n < nc:
        raise ValueError("fewer retrieval keys than centroids")
    k0 = max(2, min(coarse, nc // 2, n))
    c0 = keys[_seeded_pick(n, k0, seed, device)].clone()
    c0 = _lloyd(keys, c0, coarse_iters)
    bucket = _assign(keys, c0)
    counts = torch.bincount(bucket, minlength=k0)
    shares = _leaf_shares(counts, nc)
    starts = torch.cumsum(shares, 0) - shares
    order = torch.argsort(bucket, stable=True)
    bstart = (torch.cumsum(counts, 0) - counts).cpu()
    counts_c = counts.cpu()

    centroids = torch.empty(nc, d, dtype=keys.dtype, device=device)
    labels = torch.empty(n, 2, dtype=torch.long, device=device)
    for b in range(k0):
        m, L = int(counts_c[b]), int(shares[b])
        if m == 0:
            continue
        ids = order[int(bstart[b]):int(bstart[b]) + m]
        xb = keys[ids]
        cb = xb[_seeded_pick(m, L, seed * 7919 + 1 + b, device)].clone()
        if m > L:
            cb = _lloyd(xb, cb, leaf_iters)
        s0 = int(starts[b])
        centroids[s0:s0 + L] = cb
        top = (xb @ cb.t()).topk(2, dim=1).indices
        labels[ids] = top + s0
    stats = {"algorithm": "two-level-spherical", "coarse_clusters": int(k0),
             "coarse_iters": int(coarse_iters), "leaf_iters": int(leaf_iters)}
    return centroids, labels, stats


def midrise4(x: torch.Tensor) -> torch.Tensor:
    """Per-row max-abs mid-rise 4-bit reconstruction (16 levels)."""
    a = x.abs().amax(dim=-1, keepdim=True).clamp_min(1e-9)
    step = 2 * a / 16
    return -a + (torch.clamp(torch.floor((x + a) / step), 0, 15) + 0.5) * step


def to_csr(labels: torch.Tensor, nc: int):
    """CSR of spill lists: offsets [nc+1] int32, values [2R] local token ids
    (token order), on the labels' device (integer sort and scan: the same
    lists on the host and the GPU)."""
    flat = labels.reshape(-1)
    tokens = torch.arange(labels.shape[0], device=flat.device).repeat_interleave(labels.shape[1])
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=nc)
    offsets = torch.cat([torch.zeros(1, dtype=torch.long, device=flat.device), counts.cumsum(0)])
    return offsets.int(), tokens[order].int()
