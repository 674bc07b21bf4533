"""Independent static caches decoded together: one query token per cache,
one launch per step.

The reference's operator (``src/seoulkv4/api.py``) serves one request; a
server with many requests, or a model with a stack of layers whose caches are
independent, would hold one ``SeoulKV4`` per cache and run them one after the
other.  ``SeoulKV4Batch`` keeps the same contract per cache (the same index,
K/V and query shapes, the same results bit for bit) but decodes every cache in
one step graph: the engine's slots are the caches, each slot's four KV heads
are four cells, and one launch of the fused kernel covers every cell (one
thread-block cluster each), which fills the GPU where a single cache uses 4 of
its clusters.

All caches must share the context length, the attention zones and the
centroid count (caches built from the same shapes do); nprobe may differ.
"""

from __future__ import annotations

from typing import Sequence

import torch

from seoulkv_b200 import _native
from seoulkv_b200.api import _bits, _check_append, _cuda_index, _current_stream, _enqueue_append, _max_context
from seoulkv_b200.config import MAX_CONTEXT, MIN_CONTEXT, N_HEADS, N_KV_HEADS, SeoulKV4Config, validate_nprobe
from seoulkv_b200.index import SeoulKV4Index, device_view
from seoulkv_b200.result import _DeviceBuffer


class BatchResult:
    """Outputs of one batched run, valid until the next run or close."""

    def __init__(self, owner: "SeoulKV4Batch", generation: int):
        self._owner = owner
        self._generation = generation

    def _live(self) -> "SeoulKV4Batch":
        o = self._owner
        if o._closed or o._generation != self._generation:
            raise RuntimeError("SeoulKV4Batch result is no longer live; read back before the next run or close")
        return o

    def to_torch(self) -> torch.Tensor:
        """Synchronise and copy the outputs into a CPU BF16 tensor [n, 1, 16, 256]."""
        o = self._live()
        y = torch.empty((o.n, 1, N_HEADS, 256), dtype=torch.bfloat16)
        try:
            o._engine.finish_to(y.data_ptr())  # wait, status check and output copy in one native call
        except _native.NativeError as exc:
            raise RuntimeError(str(exc)) from exc
        return y

    @property
    def device_tensor(self) -> torch.Tensor:
        """Borrowed CUDA BF16 view [n, 1, 16, 256] of the engine's output buffer."""
        o = self._live()
        buf = _DeviceBuffer(o._engine.output_device_ptr(), (o.n * N_HEADS, 256), o._stream())
        base = torch.as_tensor(buf, device=f"cuda:{o._device_index}")
        return base.view(torch.bfloat16).reshape(o.n, 1, N_HEADS, 256)


class SeoulKV4Batch:
    """Static-cache sparse decode of n independent caches, one query each per run."""

    def __init__(self, *, device, caches: Sequence[tuple[torch.Tensor, torch.Tensor, SeoulKV4Index]],
                 config: SeoulKV4Config | None = None):
        self._config = SeoulKV4Config() if config is None else config
        if not isinstance(self._config, SeoulKV4Config):
            raise TypeError("expected SeoulKV4Config")
        if len(caches) == 0:
            raise ValueError("SeoulKV4Batch needs at least one cache")
        self._device_index = _cuda_index(device)
        zones = None
        nc = None
        self._nprobe = []
        for i, cache in enumerate(caches):
            if len(cache) != 3:
                raise ValueError("each cache is (k, v, index)")
            k, v, index = cache
            if not isinstance(index, SeoulKV4Index):
                raise TypeError("expected SeoulKV4Index")
            z = index.zones
            if not MIN_CONTEXT <= z.context <= MAX_CONTEXT or z.context % 4:
                raise ValueError("unsupported context for the fixed SeoulKV4 candidate/tag profile")
            for name, value in (("K", k), ("V", v)):
                if (not isinstance(value, torch.Tensor) or value.dtype != torch.bfloat16
                        or value.device.type not in ("cpu", "cuda")
                        or tuple(value.shape) != (N_KV_HEADS, z.context, 256)):
                    raise ValueError(f"cache {i}: expected BF16 {name} [4,{z.context},256]")
            cells = index.cells()
            c_nc = int(cells[0]["centroids"].shape[0])
            if any(int(c["centroids"].shape[0]) != c_nc for c in cells):
                raise ValueError(f"cache {i}: all four index cells must have the same centroid count")
            key = (z.context, z.sink, z.local)
            if zones is None:
                zones, nc = key, c_nc
            elif key != zones or c_nc != nc:
                raise ValueError("all caches must share the context, the attention zones and the centroid count")
            index._check_keys(k.cpu() if k.device.type != "cpu" else k)
            self._nprobe.append(validate_nprobe(self._config.nprobe, c_nc) if self._config.nprobe is not None
                                else index.nprobe)
        self._caches = list(caches)
        self._zones, self._nc = zones, nc
        self._context = zones[0]
        self._max_context = _max_context(self._config, zones[0])
        self.n = len(caches)
        self._engine: _native.Engine | None = None
        self._generation = 0
        self._closed = False

    # ------------------------------------------------------------ internals

    def _require_open(self):
        if self._closed:
            raise RuntimeError("SeoulKV4Batch is closed")

    def _stream(self) -> int:
        return _current_stream(self._device_index)

    def _initialize(self) -> _native.Engine:
        context, sink, local = self._zones
        eng = _native.Engine(n_slots=self.n, context=context, sink=sink, local=local, nc=self._nc,
                             capacity=self._config.stage15_capacity, device=self._device_index,
                             max_context=self._max_context if self._max_context > context else 0,
                             lead=self._config.lead_cluster, trace=self._config.trace_stages)
        try:
            for s, (k, v, index) in enumerate(self._caches):
                eng.upload_index(s, [device_view(c, p) for c, p in zip(index.cells(), self._nprobe[s])])
                on_dev = k.device.type == "cuda"
                if on_dev:
                    kb, vb = _bits(k.to(f"cuda:{self._device_index}")), _bits(v.to(f"cuda:{self._device_index}"))
                else:
                    kb, vb = _bits(k), _bits(v)
                eng.upload_kv(s, kb.data_ptr(), vb.data_ptr(), on_dev)
            eng.set_l2_residency(self._config.l2_resident)
        except Exception:
            eng.close()
            raise
        return eng

    # -------------------------------------------------------------- public

    @property
    def initialized(self) -> bool:
        return self._engine is not None

    def run(self, q: torch.Tensor) -> BatchResult:
        """Initialise on the first call (uploads every cache), then bind the n
        queries (BF16 [n, 1, 16, 256], host or CUDA) and enqueue one step."""
        self._require_open()
        if (not isinstance(q, torch.Tensor) or q.dtype != torch.bfloat16 or q.device.type not in ("cpu", "cuda")
                or tuple(q.shape) != (self.n, 1, N_HEADS, 256)):
            raise ValueError(f"expected BF16 Q [{self.n},1,16,256]")
        first = self._engine is None
        if first:
            self._engine = self._initialize()
            self._caches = [(None, None, c[2]) for c in self._caches]  # K/V now live on the device
        if q.device.type == "cuda":
            qd = _bits(q.to(f"cuda:{self._device_index}"))
            self._engine.step(qd.data_ptr(), True, self._stream())
        else:
            self._engine.step(_bits(q).data_ptr(), False, self._stream())
        self._generation += 1
        if first:
            st = self._engine.status()
            if st.flags:
                raise ValueError(
                    f"live Stage-I key counts [{st.pool_min}, {st.pool_max}] outside the capacity range "
                    f"(status {st.flags:#x}); change capacity, never truncate")
        return BatchResult(self, self._generation)

    @property
    def context(self) -> int:
        """Tokens in every cache: the shared context plus every appended token."""
        return self._context

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Grow every cache by m tokens: BF16 K and V [n, 4, m, 256], host or CUDA.

        The same contract as ``SeoulKV4.append`` per cache; all caches keep one
        shared context.
        """
        self._require_open()
        m = _check_append(k, v, (self.n, N_KV_HEADS), self._context, self._max_context)
        if self._engine is None:
            self._engine = self._initialize()
            self._caches = [(None, None, c[2]) for c in self._caches]
        _enqueue_append(self._engine, k, v, self._device_index, self._stream())
        self._context += m

    def synchronize(self) -> None:
        """Wait for the last run; raises RuntimeError if a live count left its range."""
        self._require_open()
        if self._engine is not None:
            try:
                self._engine.sync()
            except _native.NativeError as exc:
                raise RuntimeError(str(exc)) from exc

    def debug_snapshot(self) -> dict:
        """Selected token ids of the latest run: LongTensor [n, 4, 4, 100] (cache, KV group, head, rank)."""
        self._require_open()
        if self._engine is None:
            raise RuntimeError("run(q) must initialize SeoulKV4Batch first")
        if not self._config.debug:
            raise RuntimeError("debug_snapshot requires SeoulKV4Config(debug=True)")
        self.synchronize()
        return {"selected_ids": torch.from_numpy(self._engine.debug_ids()).long()}

    def metadata(self) -> dict:
        self._require_open()
        context, sink, local = self._zones
        meta = {"initialized": self.initialized, "caches": self.n, "context": self._context,
                "max_context": self._max_context, "sink": sink,
                "local": local, "centroids_per_head": self._nc, "nprobe": [list(p) for p in self._nprobe]}
        if self._engine is not None:
            meta.update(kernels_per_step=self._engine.kernels_per_step(),
                        device_path="fused cluster kernel" if self._engine.fused else "staged kernels",
                        graph_replay=True)
        return meta

    def close(self) -> None:
        """Release the device buffers after pending work (idempotent)."""
        if self._closed:
            return
        try:
            if self._engine is not None:
                try:
                    self._engine.sync()
                except _native.NativeError:
                    pass
        finally:
            self._closed = True
            if self._engine is not None:
                self._engine.close()
            self._engine = None
            self._caches = []

    def __enter__(self):
        self._require_open()
        return self

    def __exit__(self, exc_type, exc, tb):
        self.close()
