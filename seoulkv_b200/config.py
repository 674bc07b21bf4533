"""Runtime settings (mirrors ``src/seoulkv4/config.py:1-40`` of the reference)."""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

DEFAULT_NPROBE = 256

# Fixed funnel budgets of the validated profile (reference config.py:25-40).
N_KV_HEADS = 4
N_HEADS = 16
HEAD_DIM = 256
TOPK = 100
STAGE15_M = 2048          # per-head frontier; the first 1600 enter the union
STAGE15_UNION_M = 1600
STAGE16_M = 256
MIN_CONTEXT = 6400
MAX_CONTEXT = 524288      # reference limit (index.py:114); the engine itself takes up to 2^20
MAX_CENTROIDS = 65536     # Fine's 16-bit survivor positions (index.py:126)
ENGINE_MAX_CONTEXT = 1 << 20  # largest context the engine holds (appends included)


def validate_nprobe(nprobe, nc: int) -> tuple[int, ...]:
    """One value for all heads or four per-head values; multiples of 16 in [16, min(512, nc)]."""
    if type(nprobe) is int:
        probes = (nprobe,) * N_KV_HEADS
    elif isinstance(nprobe, Sequence) and not isinstance(nprobe, (str, bytes)):
        probes = tuple(nprobe)
    else:
        raise ValueError("nprobe must be an integer or four per-head integers")
    hi = min(512, nc)
    if len(probes) != N_KV_HEADS or any(type(p) is not int or not 16 <= p <= hi or p % 16 for p in probes):
        raise ValueError(f"each nprobe must be a multiple of 16 in [16, {hi}]")
    return probes


@dataclass(frozen=True)
class SeoulKV4Config:
    """Stage-1.5 key capacity per KV head, diagnostics, optional nprobe override.

    ``stage15_capacity`` must be a multiple of 768 in [12288, 24576]; a live
    pool above it is reported as an error, never truncated.  ``nprobe``
    (None = keep the index's value) overrides the index's probe budget for this
    instance without rebuilding the index.  ``max_context`` (None = the
    index's context: a static cache, as in the reference) is the context the
    cache may grow to by ``append``; device buffers are sized for it.
    ``l2_resident`` keeps the index's centroid planes in the persisting part
    of L2 across steps (the reference keeps its coarse centroid plane in
    on-chip SRAM); it applies where the device's persisting set-aside can hold
    them, and is a no-op otherwise.  ``lead_cluster`` adds to every fused
    launch one cluster that decodes a small synthetic cell ahead of the real
    ones, so that the kernel's instructions are in L2 when the real cells
    reach them; results do not depend on it (off only to measure it).
    ``trace_stages`` makes the single-kernel path also write every stage's
    intermediates (coarse bounds, survivor tags, selected clusters, pool,
    unions) for stage-by-stage inspection; decoding does not need them.
    """

    stage15_capacity: int = 13056
    debug: bool = False
    nprobe: int | tuple[int, ...] | None = None
    max_context: int | None = None
    l2_resident: bool = True
    lead_cluster: bool = True
    trace_stages: bool = False

    def __post_init__(self):
        n = self.stage15_capacity
        if type(n) is not int or not 12288 <= n <= 24576 or n % (6 * 4 * 32):
            raise ValueError("stage15_capacity must be a multiple of 768 in [12288, 24576]")
        if type(self.debug) is not bool:
            raise TypeError("debug must be a bool")
        if type(self.l2_resident) is not bool:
            raise TypeError("l2_resident must be a bool")
        if type(self.lead_cluster) is not bool:
            raise TypeError("lead_cluster must be a bool")
        if type(self.trace_stages) is not bool:
            raise TypeError("trace_stages must be a bool")
        if self.nprobe is not None:
            validate_nprobe(self.nprobe if type(self.nprobe) is int else tuple(self.nprobe), 512)
            if not isinstance(self.nprobe, int):
                object.__setattr__(self, "nprobe", tuple(self.nprobe))
        if self.max_context is not None and (type(self.max_context) is not int
                                             or not MIN_CONTEXT <= self.max_context <= ENGINE_MAX_CONTEXT):
            raise ValueError(f"max_context must be None or an integer in [{MIN_CONTEXT}, {ENGINE_MAX_CONTEXT}]")
