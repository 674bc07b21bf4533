"""Seeded synthetic K/V/Q with the benchmark's shapes and value distributions.

Per KV head, K is a mixture of Gaussian components (centres ~ N(0, 1)^256,
within-component std 0.35, Dirichlet(1) mixture weights) with RoPE
(theta = 10000, rotate-half, positions 0..T-1) applied; V ~ N(0, 1).  A query
head picks a random component centre of its KV head, adds N(0, 0.2) noise and
is RoPE'd at position T.  Everything is BF16 on the CPU and reproducible from
``seed`` alone (CPU ``torch.Generator``), so fixtures can be regenerated
instead of stored.
"""

from __future__ import annotations

import torch

N_KV, N_Q, DIM = 4, 16, 256


def _rope(x: torch.Tensor, pos: torch.Tensor, theta: float = 10000.0) -> torch.Tensor:
    half = x.shape[-1] // 2
    inv = 1.0 / (theta ** (torch.arange(half, dtype=torch.float64) * 2 / x.shape[-1]))
    ang = pos.to(torch.float64)[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], dim=-1).to(torch.float32)
    sin = torch.cat([ang.sin(), ang.sin()], dim=-1).to(torch.float32)
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


class Mixture:
    """Component centres and weights of one KV head."""

    def __init__(self, components: int, gen: torch.Generator):
        self.centres = torch.randn(components, DIM, generator=gen)
        e = -torch.log(torch.rand(components, generator=gen).clamp_min(1e-12))
        self.weights = e / e.sum()


def make_kv(context: int, *, seed: int, components: int = 256, chunk: int = 65536):
    """Return (k, v, mixtures): CPU BF16 [4, T, 256] each, plus the per-head mixtures."""
    gen = torch.Generator().manual_seed(int(seed))
    k = torch.empty(N_KV, context, DIM, dtype=torch.bfloat16)
    v = torch.empty(N_KV, context, DIM, dtype=torch.bfloat16)
    mixes = []
    for h in range(N_KV):
        mix = Mixture(components, gen)
        mixes.append(mix)
        comp = torch.multinomial(mix.weights, context, replacement=True, generator=gen)
        for s in range(0, context, chunk):
            e = min(context, s + chunk)
            x = mix.centres[comp[s:e]] + 0.35 * torch.randn(e - s, DIM, generator=gen)
            k[h, s:e] = _rope(x, torch.arange(s, e)).bfloat16()
            v[h, s:e] = torch.randn(e - s, DIM, generator=gen).bfloat16()
    return k, v, mixes


def make_kv_range(total: int, begin: int, end: int, *, seed: int, components: int = 256, block: int = 65536):
    """K/V of tokens [begin, end) of a ``total``-token sequence, generated block by block.

    Each ``block``-token block of each KV head draws its components, noise and
    V from its own generator (seeded by seed, head and block), so any token
    range of the same sequence can be produced on its own: a shard of a long
    context generates only its slice and every shard agrees on the mixtures.
    Returns (k, v, mixtures) like make_kv (a different sequence than make_kv
    for the same seed).
    """
    if not 0 <= begin < end <= total:
        raise ValueError("require 0 <= begin < end <= total")
    gen = torch.Generator().manual_seed(int(seed))
    mixes = [Mixture(components, gen) for _ in range(N_KV)]
    n = end - begin
    k = torch.empty(N_KV, n, DIM, dtype=torch.bfloat16)
    v = torch.empty(N_KV, n, DIM, dtype=torch.bfloat16)
    for h, mix in enumerate(mixes):
        for b0 in range(begin - begin % block, end, block):
            bg = torch.Generator().manual_seed(int(seed) * 1_000_003 + h * 100_003 + b0 // block)
            b1 = min(total, b0 + block)
            comp = torch.multinomial(mix.weights, b1 - b0, replacement=True, generator=bg)
            x = mix.centres[comp] + 0.35 * torch.randn(b1 - b0, DIM, generator=bg)
            vb = torch.randn(b1 - b0, DIM, generator=bg)
            s, e = max(begin, b0), min(end, b1)
            k[h, s - begin:e - begin] = _rope(x[s - b0:e - b0], torch.arange(s, e)).bfloat16()
            v[h, s - begin:e - begin] = vb[s - b0:e - b0].bfloat16()
    return k, v, mixes


def make_query(context: int, mixes, *, seed: int) -> torch.Tensor:
    """CPU BF16 Q [1, 1, 16, 256]: a component centre of head j // 4 plus N(0, 0.2), RoPE'd at T."""
    gen = torch.Generator().manual_seed(int(seed))
    rows = []
    for j in range(N_Q):
        mix = mixes[j // (N_Q // N_KV)]
        c = int(torch.randint(len(mix.centres), (1,), generator=gen))
        rows.append(mix.centres[c] + 0.2 * torch.randn(DIM, generator=gen))
    q = _rope(torch.stack(rows), torch.full((N_Q,), context))
    return q.bfloat16().reshape(1, 1, N_Q, DIM)
