"""Public SeoulKV4 lifecycle on a B200 (mirrors ``src/seoulkv4/api.py:14-145``).

``SeoulKV4(device=..., k=..., v=..., index=..., config=...)`` validates and
keeps the inputs; the first ``run(q)`` uploads the index, key planes and FP8
records, captures the decode step as a CUDA graph and runs it; later calls
only copy Q and replay the graph on the current PyTorch stream.
"""

from __future__ import annotations

import torch

from seoulkv_b200 import _native
from seoulkv_b200.config import (
    MAX_CONTEXT, MIN_CONTEXT, N_HEADS, N_KV_HEADS, STAGE15_M, SeoulKV4Config, validate_nprobe,
)
from seoulkv_b200.index import SeoulKV4Index, device_view
from seoulkv_b200.result import DecodeResult

_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _current_stream(device_index: int) -> int:
    """The cudaStream_t of PyTorch's current stream on the device (the raw
    handle without a Stream object once PyTorch's CUDA state is initialised:
    this is on every decode step's host path)."""
    if _raw_stream is None or not torch.cuda.is_initialized():
        return torch.cuda.current_stream(device_index).cuda_stream
    return _raw_stream(device_index)


def _cuda_index(device) -> int:
    if device is None:
        raise ValueError("supply a caller-owned CUDA device")
    dev = torch.device(device if not isinstance(device, int) else f"cuda:{device}")
    if dev.type != "cuda":
        raise ValueError("SeoulKV4 runs on a CUDA device")
    return dev.index if dev.index is not None else torch.cuda.current_device()


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16)


def _max_context(config: SeoulKV4Config, context: int) -> int:
    if config.max_context is None:
        return context
    if config.max_context < context:
        raise ValueError(f"max_context {config.max_context} is below the index's context {context}")
    return config.max_context


def _check_append(k, v, lead: tuple, context: int | None, max_context: int) -> int:
    """Validate appended K/V (BF16 [*lead, m, 256], one device type); returns m.

    ``context`` None: the append is being captured into a CUDA graph, where
    nothing may wait on the device; the engine's device-side capacity check
    (a skipped append and an error at the next synchronize) replaces the
    host's.
    """
    shape = None
    for name, t in (("K", k), ("V", v)):
        if (not isinstance(t, torch.Tensor) or t.dtype != torch.bfloat16 or t.device.type not in ("cpu", "cuda")
                or t.ndim != len(lead) + 2 or tuple(t.shape[:len(lead)]) != lead or t.shape[-1] != 256
                or t.shape[-2] < 1):
            dims = ",".join(str(x) for x in lead)
            raise ValueError(f"expected BF16 appended {name} [{dims},m,256] with m >= 1")
        shape = shape or tuple(t.shape)
        if tuple(t.shape) != shape:
            raise ValueError("appended K and V must have the same shape")
    if k.device != v.device:
        raise ValueError("appended K and V must be on one device")
    m = int(k.shape[-2])
    if context is None:
        return m
    # host keys are checked here; CUDA keys on the device (no wait), where a
    # non-finite element counts as 0 and the next synchronize raises
    if k.device.type == "cpu" and not bool(torch.isfinite(k).all()):
        raise ValueError("appended keys must be finite")
    if context + m > max_context:
        hint = " (SeoulKV4Config(max_context=...) lets the cache grow)" if max_context == context else ""
        raise ValueError(f"append of {m} tokens to context {context} passes max_context {max_context}{hint}")
    return m


def _enqueue_append(eng, k, v, device_index: int, stream: int) -> None:
    """Append [..., m, 256] K/V in chunks the engine takes in one call."""
    m = k.shape[-2]
    on_dev = k.device.type == "cuda"
    for j0 in range(0, m, _native.APPEND_MAX):
        n = min(_native.APPEND_MAX, m - j0)
        kc, vc = k[..., j0:j0 + n, :], v[..., j0:j0 + n, :]
        if on_dev:
            kc, vc = kc.to(f"cuda:{device_index}"), vc.to(f"cuda:{device_index}")
        kb, vb = _bits(kc), _bits(vc)
        eng.append(kb.data_ptr(), vb.data_ptr(), n, on_dev, stream)


class SeoulKV4:
    """Static-cache sparse decode: one request, one query token per run."""

    def __init__(self, *, device, k: torch.Tensor, v: torch.Tensor, index: SeoulKV4Index,
                 config: SeoulKV4Config | None = None):
        self._config = SeoulKV4Config() if config is None else config
        if not isinstance(self._config, SeoulKV4Config) or not isinstance(index, SeoulKV4Index):
            raise TypeError("expected SeoulKV4Config and SeoulKV4Index")
        self._device_index = _cuda_index(device)
        context = index.zones.context
        if not MIN_CONTEXT <= context <= MAX_CONTEXT or context % 4:
            raise ValueError("unsupported context for the fixed SeoulKV4 candidate/tag profile")
        for name, value in (("K", k), ("V", v)):
            if (not isinstance(value, torch.Tensor) or value.dtype != torch.bfloat16
                    or value.device.type not in ("cpu", "cuda")
                    or tuple(value.shape) != (N_KV_HEADS, context, 256)):
                raise ValueError(f"expected BF16 {name} [4,{context},256]")
        index._check_keys(k.cpu() if k.device.type != "cpu" else k)
        nc = min(int(c["centroids"].shape[0]) for c in index.cells())
        self._nprobe = (validate_nprobe(self._config.nprobe, nc) if self._config.nprobe is not None
                        else index.nprobe)
        self._index = index
        self._host_kv = (k, v)
        self._context = context
        self._max_context = _max_context(self._config, context)
        self._captured_appends = False
        self._engine: _native.Engine | None = None
        self._generation = 0
        self._closed = False

    # -------------------------------------------------------------- state

    def _require_open(self):
        if self._closed:
            raise RuntimeError("SeoulKV4 is closed")

    def _require_initialized(self):
        self._require_open()
        if self._engine is None:
            raise RuntimeError("run(q) must initialize SeoulKV4 first")
        return self._engine

    @property
    def initialized(self) -> bool:
        return self._engine is not None

    @staticmethod
    def _validate_query(q):
        if (not isinstance(q, torch.Tensor) or q.dtype != torch.bfloat16
                or q.device.type not in ("cpu", "cuda") or tuple(q.shape) != (1, 1, N_HEADS, 256)):
            raise ValueError("expected BF16 Q [1,1,16,256]")

    def _stream(self) -> int:
        return _current_stream(self._device_index)

    def _initialize(self):
        zones = self._index.zones
        cells = self._index.cells()
        nc = int(cells[0]["centroids"].shape[0])
        if any(int(c["centroids"].shape[0]) != nc for c in cells):
            raise ValueError("all four index cells must have the same centroid count")
        eng = _native.Engine(n_slots=1, context=zones.context, sink=zones.sink, local=zones.local,
                             nc=nc, capacity=self._config.stage15_capacity, device=self._device_index,
                             max_context=self._max_context if self._max_context > zones.context else 0,
                             lead=self._config.lead_cluster, trace=self._config.trace_stages)
        try:
            eng.upload_index(0, [device_view(c, p) for c, p in zip(cells, self._nprobe)])
            k, v = self._host_kv
            if k.device.type == "cuda":
                kb, vb = _bits(k.to(f"cuda:{self._device_index}")), _bits(v.to(f"cuda:{self._device_index}"))
                eng.upload_kv(0, kb.data_ptr(), vb.data_ptr(), True)
            else:
                kb, vb = _bits(k), _bits(v)
                eng.upload_kv(0, kb.data_ptr(), vb.data_ptr(), False)
            eng.set_l2_residency(self._config.l2_resident)
        except Exception:
            eng.close()
            raise
        return eng

    # -------------------------------------------------------------- public

    def run(self, q: torch.Tensor) -> DecodeResult:
        """Initialise on the first call, then bind Q and enqueue the decode step."""
        self._require_open()
        self._validate_query(q)
        first = self._engine is None
        if first:
            self._engine = self._initialize()
            self._host_kv = None
        eng = self._engine
        # (a contiguous BF16 Q is passed as it is: the engine takes its bytes)
        if q.device.type == "cuda":
            if q.device.index != self._device_index:
                q = q.to(f"cuda:{self._device_index}")
            qd = q if q.is_contiguous() else q.contiguous()
            eng.step(qd.data_ptr(), True, self._stream())
        else:
            qh = q if q.is_contiguous() else q.contiguous()
            eng.step(qh.data_ptr(), False, self._stream())
        self._generation += 1
        if first:
            # the reference's first run checks the live pool against capacity
            st = self._engine.status()
            if st.flags:
                raise ValueError(
                    f"live Stage-I key counts [{st.pool_min}, {st.pool_max}] outside "
                    f"[{STAGE15_M},{self._config.stage15_capacity}] (status {st.flags:#x}); "
                    "change capacity, never truncate")
        return DecodeResult(self, self._generation)

    @property
    def context(self) -> int:
        """Tokens in the cache: the index's context plus every appended token
        (read from the device, after pending work, once appends were captured
        into a graph: its replays append too)."""
        if self._captured_appends and self._engine is not None:
            return self._engine.current_context()
        return self._context

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Grow the cache by m tokens: BF16 K and V [4, m, 256], host or CUDA.

        Stream-ordered on the current PyTorch stream, like ``run``; the first
        call initialises the instance as ``run`` does.  The new tokens enter
        the local window and the window's m oldest tokens join the retrieval
        zone, each posted to its two nearest stored centroids (the index's
        centroids and key-code scales stay those of the build).  Needs
        ``SeoulKV4Config(max_context=...)`` with room for the m tokens.  May
        be captured into a CUDA graph (CUDA K/V, instance already
        initialised); every replay then appends m more tokens.
        """
        self._require_open()
        capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
        if capturing and self._engine is None:
            raise RuntimeError("initialise SeoulKV4 (run or append once) before capturing an append")
        if not capturing and self._captured_appends and self._engine is not None:
            self._context = self._engine.current_context()
        m = _check_append(k, v, (N_KV_HEADS,), None if capturing else self._context, self._max_context)
        if self._engine is None:
            self._engine = self._initialize()
            self._host_kv = None
        _enqueue_append(self._engine, k, v, self._device_index, self._stream())
        if capturing:
            self._captured_appends = True
        else:
            self._context += m

    def _bind_query(self, q: torch.Tensor) -> None:
        self._validate_query(q)
        eng = self._require_initialized()
        if q.device.type == "cuda":
            qd = _bits(q.to(f"cuda:{self._device_index}"))
            eng.bind_query(qd.data_ptr(), True, self._stream())
        else:
            qh = _bits(q)
            eng.bind_query(qh.data_ptr(), False, self._stream())

    def synchronize(self) -> None:
        """Wait for the last run; raises RuntimeError if a live count left its range."""
        self._require_open()
        if self._engine is not None:
            try:
                self._engine.sync()
            except _native.NativeError as exc:
                raise RuntimeError(str(exc)) from exc

    def metadata(self) -> dict:
        """Host-only configuration; never reads device tensors."""
        self._require_open()
        zones = self._index.zones
        meta = {
            "initialized": self.initialized,
            "cache_layout": "flat",
            "index": self._index.metadata(),
            "nprobe": list(self._nprobe),
            "context": self._context,
            "max_context": self._max_context,
        }
        if self.initialized:
            meta.update(
                implementation="coarse 2-bit intervals -> fine 4-bit top-nprobe -> spill-2 pool -> "
                               "2-bit top-1600 union -> 4-bit top-256 union -> 8-bit exact top-100 -> "
                               "FP8 sink+local+top-100 attention",
                device=torch.cuda.get_device_name(self._device_index),
                attention_zones=zones.metadata(),
                attention_kv_dtype="FP8_E4M3",
                kernels_per_step=self._engine.kernels_per_step(),
                device_path="fused cluster kernel" if self._engine.fused else "staged kernels",
                stage15_capacity=self._config.stage15_capacity,
                graph_replay=True,
                l2_resident_bytes=getattr(self._engine, "l2_resident_bytes", 0),
            )
        return meta

    def debug_snapshot(self) -> dict:
        """Selected token ids of the latest run: LongTensor [4, 4, 100] (KV group, head, rank)."""
        eng = self._require_initialized()
        if not self._config.debug:
            raise RuntimeError("debug_snapshot requires SeoulKV4Config(debug=True)")
        self.synchronize()
        return {"selected_ids": torch.from_numpy(eng.debug_ids()[0]).long()}

    def close(self) -> None:
        """Release this instance's device buffers after pending work (idempotent)."""
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
            self._host_kv = self._index = None

    def __enter__(self):
        self._require_open()
        return self

    def __exit__(self, exc_type, exc, tb):
        self.close()
