"""ctypes binding of ``include/seoulkv_b200.h`` (the engine's C ABI).

There is no CPU fallback: if the sm_100a library cannot be loaded, every
entry point raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import numpy as np

from seoulkv_b200 import _build

SKV_STATUS_POOL_OVER = 1
SKV_STATUS_POOL_UNDER = 2
SKV_STATUS_FINE_SHORT = 4
SKV_STATUS_APPEND_FULL = 16
APPEND_MAX = 512  # tokens per skv_append call
SKV_E_CAPACITY = -3

STAGE = dict(counts=0, thresh=1, tags=2, selected=3, pool=4, u15=5, cand=6, final_pos=7, lohi=8,
             prefix2=9, residual2=10, residual4=11, kv8=12, key_scale=13, final_keys=14, offsets=15,
             values=16, mates=17, labels=18, lead_counts=19)

EXPORTS = (
    "skv_last_error", "skv_version", "skv_create", "skv_destroy", "skv_upload_index",
    "skv_upload_kv", "skv_bind_query", "skv_run", "skv_sync", "skv_status", "skv_output",
    "skv_debug_ids", "skv_read_stage", "skv_traffic", "skv_profile_step", "skv_kernel_name",
    "skv_kernels_per_step", "skv_step_kernel_name", "skv_profile_phases", "skv_phase_name", "skv_profile_ctas", "skv_step", "skv_finish",
    "skv_shard_outputs", "skv_shard_merge", "skv_shard_attention", "skv_shard_combine",
    "skv_shard_setup", "skv_shard_connect", "skv_shard_ipc_handle_bytes", "skv_shard_gids",
    "skv_append", "skv_context", "skv_set_l2_residency",
)

SKV_FLAG_STAGED = 1
SKV_FLAG_NO_LEAD = 2
SKV_FLAG_TRACE = 4
# Engines created without an explicit ``staged=`` use the staged (14-kernel)
# path when this is true; tests flip it to run both paths through the API.
FORCE_STAGED = False


class SkvDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("n_slots", "context", "sink", "local", "nc", "stage15_capacity", "device", "flags",
                 "max_context")]


class SkvCellView(ctypes.Structure):
    _fields_ = [
        ("nc", ctypes.c_int32), ("nprobe", ctypes.c_int32), ("lam", ctypes.c_float),
        ("n_postings", ctypes.c_int32),
        ("upper", ctypes.c_void_p), ("lower", ctypes.c_void_p), ("coarse_scale4", ctypes.c_void_p),
        ("fine_scale", ctypes.c_void_p), ("resid_bf16", ctypes.c_void_p), ("offsets", ctypes.c_void_p),
        ("values", ctypes.c_void_p), ("mates", ctypes.c_void_p),
    ]


class SkvStatus(ctypes.Structure):
    _fields_ = [("flags", ctypes.c_uint32)] + [(n, ctypes.c_int32) for n in (
        "first_bad_cell", "survivors_max", "pool_max", "pool_min", "union15_max", "union16_max", "reserved")]


class SkvTraffic(ctypes.Structure):
    _fields_ = [(n, ctypes.c_double) for n in
                ("coarse", "fine", "stage15", "stage16", "stage2", "attention", "total")]


_lock = threading.Lock()
_lib = None


def library_path() -> Path:
    return _build.LIB


def load() -> ctypes.CDLL:
    """Load (building first if stale and nvcc exists) the CUDA library."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        try:
            if _build.stale():
                _build.build()
        except Exception as exc:  # no nvcc: only an existing library will do
            if not path.exists():
                raise RuntimeError(f"seoulkv_b200 CUDA library missing and cannot be built: {exc}") from exc
        if not path.exists():
            raise RuntimeError(f"seoulkv_b200 CUDA library missing: {path}")
        lib = ctypes.CDLL(str(path))
        for name in EXPORTS:
            getattr(lib, name)  # raises AttributeError if an export is missing
        lib.skv_last_error.restype = ctypes.c_char_p
        lib.skv_version.restype = ctypes.c_char_p
        lib.skv_create.argtypes = [ctypes.POINTER(SkvDesc), ctypes.POINTER(ctypes.c_void_p)]
        lib.skv_destroy.argtypes = [ctypes.c_void_p]
        lib.skv_destroy.restype = None
        lib.skv_upload_index.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(SkvCellView)]
        lib.skv_upload_kv.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_int32]
        lib.skv_bind_query.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        lib.skv_run.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.skv_sync.argtypes = [ctypes.c_void_p]
        lib.skv_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(SkvStatus)]
        lib.skv_output.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32]
        lib.skv_debug_ids.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.skv_read_stage.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                       ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
        lib.skv_traffic.argtypes = [ctypes.c_void_p, ctypes.POINTER(SkvTraffic)]
        lib.skv_profile_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                         ctypes.POINTER(ctypes.c_int32)]
        lib.skv_kernel_name.restype = ctypes.c_char_p
        lib.skv_kernel_name.argtypes = [ctypes.c_int32]
        lib.skv_kernels_per_step.restype = ctypes.c_int32
        lib.skv_step_kernel_name.restype = ctypes.c_char_p
        lib.skv_step_kernel_name.argtypes = [ctypes.c_void_p, ctypes.c_int32]
        lib.skv_profile_phases.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                           ctypes.c_int32, ctypes.POINTER(ctypes.c_int32)]
        lib.skv_phase_name.restype = ctypes.c_char_p
        lib.skv_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p]
        lib.skv_finish.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        lib.skv_profile_ctas.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_int32, ctypes.POINTER(ctypes.c_int32),
                                         ctypes.POINTER(ctypes.c_float), ctypes.c_void_p, ctypes.c_int32]
        lib.skv_phase_name.argtypes = [ctypes.c_int32]
        lib.skv_shard_outputs.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_void_p),
                                          ctypes.POINTER(ctypes.c_void_p)]
        lib.skv_shard_merge.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                        ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p]
        lib.skv_shard_attention.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p,
                                            ctypes.c_void_p]
        lib.skv_shard_combine.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                          ctypes.c_void_p]
        lib.skv_shard_setup.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
        lib.skv_shard_connect.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        lib.skv_shard_ipc_handle_bytes.restype = ctypes.c_int32
        lib.skv_shard_gids.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]
        lib.skv_append.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32,
                                   ctypes.c_int32, ctypes.c_void_p]
        lib.skv_context.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32)]
        lib.skv_set_l2_residency.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.POINTER(ctypes.c_size_t)]
        _lib = lib
        return lib


class NativeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().skv_last_error().decode(errors="replace")
        raise NativeError(rc, f"{what}: {msg}")


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


class Engine:
    """One engine instance: ``n_slots`` caches x 4 KV heads on one CUDA device."""

    def __init__(self, *, n_slots: int, context: int, sink: int, local: int, nc: int,
                 capacity: int, device: int, staged: bool | None = None, max_context: int = 0,
                 lead: bool = True, trace: bool = False):
        self.lib = load()
        self.n_slots, self.context, self.nc, self.capacity = n_slots, context, nc, capacity
        self.sink, self.local, self.device = sink, local, device
        self.max_context = max_context or context
        staged = FORCE_STAGED if staged is None else staged
        desc = SkvDesc(n_slots=n_slots, context=context, sink=sink, local=local, nc=nc,
                       stage15_capacity=capacity, device=device,
                       flags=(SKV_FLAG_STAGED if staged else 0) | (0 if lead else SKV_FLAG_NO_LEAD)
                       | (SKV_FLAG_TRACE if trace else 0),
                       max_context=max_context)
        h = ctypes.c_void_p()
        check(self.lib.skv_create(ctypes.byref(desc), ctypes.byref(h)), "skv_create")
        self.handle = h
        self._keep = []

    def close(self) -> None:
        if self.handle:
            self.lib.skv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def upload_index(self, slot: int, views: list[dict]) -> None:
        arrs = []
        cells = (SkvCellView * 4)()
        for g, v in enumerate(views):
            a = {k: np.ascontiguousarray(v[k]) for k in
                 ("upper", "lower", "coarse_scale4", "fine_scale", "resid_bf16", "offsets", "values", "mates")}
            arrs.append(a)
            cells[g] = SkvCellView(
                nc=int(v["nc"]), nprobe=int(v["nprobe"]), lam=float(v["lam"]),
                n_postings=int(len(a["values"])),
                **{k: _ptr(x) for k, x in a.items()},
            )
        check(self.lib.skv_upload_index(self.handle, slot, cells), "skv_upload_index")

    def upload_kv(self, slot: int, k_ptr: int, v_ptr: int, on_device: bool) -> None:
        check(self.lib.skv_upload_kv(self.handle, slot, ctypes.c_void_p(k_ptr), ctypes.c_void_p(v_ptr),
                                     int(on_device)), "skv_upload_kv")

    def bind_query(self, q_ptr: int, on_device: bool, stream: int = 0) -> None:
        check(self.lib.skv_bind_query(self.handle, ctypes.c_void_p(q_ptr), int(on_device),
                                      ctypes.c_void_p(stream or None)), "skv_bind_query")

    def run(self, stream: int = 0) -> None:
        check(self.lib.skv_run(self.handle, ctypes.c_void_p(stream or None)), "skv_run")

    def step(self, q_ptr: int, on_device: bool, stream: int = 0) -> None:
        """bind_query + run in one call."""
        # (the argtypes convert the integers: no ctypes objects on the per-step path)
        check(self.lib.skv_step(self.handle, q_ptr, on_device, stream or None), "skv_step")

    def finish(self, out: np.ndarray | None) -> None:
        """Wait for the last step; copy its output into `out` (uint16 [n_slots, 16, 256]) if given.
        Raises NativeError (SKV_E_CAPACITY) when a live count left its range."""
        check(self.lib.skv_finish(self.handle, None if out is None else _ptr(out), None), "skv_finish")

    def finish_to(self, out_ptr: int) -> None:
        """``finish`` into host memory at ``out_ptr`` (BF16 [n_slots, 16, 256], C order)."""
        check(self.lib.skv_finish(self.handle, out_ptr, None), "skv_finish")

    def sync(self) -> None:
        check(self.lib.skv_sync(self.handle), "skv_sync")

    def append(self, k_ptr: int, v_ptr: int, n_tokens: int, on_device: bool, stream: int = 0) -> None:
        """Append n_tokens (<= APPEND_MAX) tokens to every slot: BF16 [n_slots][4][n_tokens][256]."""
        check(self.lib.skv_append(self.handle, ctypes.c_void_p(k_ptr), ctypes.c_void_p(v_ptr), n_tokens,
                                  int(on_device), ctypes.c_void_p(stream or None)), "skv_append")

    def current_context(self) -> int:
        """The slots' context after every enqueued append (waits)."""
        t = ctypes.c_int32()
        check(self.lib.skv_context(self.handle, ctypes.byref(t)), "skv_context")
        return t.value

    def read_csr(self, slot: int) -> list[tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """Live (offsets, values, mates) of the slot's four cells."""
        offs = self.read_stage(slot, "offsets", np.int32, (4, self.nc + 1))
        total = int(offs[:, -1].sum())
        vals = self.read_stage(slot, "values", np.int32, (max(total, 1),))
        mates = self.read_stage(slot, "mates", np.int32, (max(total, 1),))
        out, o = [], 0
        for g in range(4):
            n = int(offs[g, -1])
            out.append((offs[g], vals[o:o + n], mates[o:o + n]))
            o += n
        return out

    def status(self) -> SkvStatus:
        s = SkvStatus()
        check(self.lib.skv_status(self.handle, ctypes.byref(s)), "skv_status")
        return s

    def output_host(self) -> np.ndarray:
        out = np.empty((self.n_slots, 16, 256), dtype=np.uint16)
        check(self.lib.skv_output(self.handle, _ptr(out), 1), "skv_output")
        return out

    def output_device_ptr(self) -> int:
        p = ctypes.c_void_p()
        check(self.lib.skv_output(self.handle, ctypes.byref(p), 0), "skv_output")
        return int(p.value)

    def debug_ids(self) -> np.ndarray:
        out = np.empty((self.n_slots, 4, 4, 100), dtype=np.int32)
        check(self.lib.skv_debug_ids(self.handle, _ptr(out)), "skv_debug_ids")
        return out

    def read_stage(self, slot: int, which: str, dtype, shape) -> np.ndarray:
        out = np.zeros(shape, dtype=dtype)
        written = ctypes.c_size_t()
        check(self.lib.skv_read_stage(self.handle, slot, STAGE[which], _ptr(out), out.nbytes,
                                      ctypes.byref(written)), "skv_read_stage")
        return out

    def profile_step(self, stream: int = 0) -> list[tuple[str, float]]:
        """One non-graph step with per-kernel device times (ms)."""
        ms = np.zeros(64, dtype=np.float32)
        n = ctypes.c_int32()
        check(self.lib.skv_profile_step(self.handle, ctypes.c_void_p(stream or None), _ptr(ms), 64,
                                        ctypes.byref(n)), "skv_profile_step")
        return [(self.lib.skv_step_kernel_name(self.handle, i).decode(), float(ms[i])) for i in range(n.value)]

    def set_l2_residency(self, enable: bool) -> int:
        """Hold the centroid planes in the persisting part of L2 (or stop);
        returns the bytes now resident (0: off, or they do not fit)."""
        n = ctypes.c_size_t()
        check(self.lib.skv_set_l2_residency(self.handle, int(bool(enable)), ctypes.byref(n)), "skv_set_l2_residency")
        self.l2_resident_bytes = int(n.value)
        return self.l2_resident_bytes

    def kernels_per_step(self) -> int:
        """Kernels one step of this engine launches (1 on the fused path)."""
        n = 0
        while self.lib.skv_step_kernel_name(self.handle, n):
            n += 1
        return n

    @property
    def fused(self) -> bool:
        return self.lib.skv_step_kernel_name(self.handle, 0) == b"k_funnel"

    def profile_phases(self, stream: int = 0) -> list[tuple[str, float]]:
        """One fused step: (segment name, SM cycles) in order (CTA 0 of cell 0)."""
        tags = np.zeros(128, dtype=np.int32)
        cyc = np.zeros(128, dtype=np.float64)
        n = ctypes.c_int32()
        check(self.lib.skv_profile_phases(self.handle, ctypes.c_void_p(stream or None), _ptr(tags), _ptr(cyc),
                                          128, ctypes.byref(n)), "skv_profile_phases")
        return [(self.lib.skv_phase_name(int(tags[i])).decode(), float(cyc[i])) for i in range(n.value)]

    def profile_ctas(self, stream: int = 0):
        """One fused launch: per-CTA (entry, exit) global-timer ns relative to
        the earliest entry, shaped [cells, 16]; the launch's event time (µs);
        and the phase marks of cell 0's 16 CTAs as {rank: [(name, ns), ...]}
        on the same time base."""
        cap, mm = 16 * 1024, 128
        s = np.zeros(cap, dtype=np.int64)
        e = np.zeros(cap, dtype=np.int64)
        marks = np.zeros(16 * mm * 2, dtype=np.int64)
        n = ctypes.c_int32()
        ms = ctypes.c_float()
        check(self.lib.skv_profile_ctas(self.handle, ctypes.c_void_p(stream or None), _ptr(s), _ptr(e), cap,
                                        ctypes.byref(n), ctypes.byref(ms), _ptr(marks), mm), "skv_profile_ctas")
        s, e = s[:n.value], e[:n.value]
        t0 = s.min()
        marks = marks.reshape(16, mm, 2)
        per = {r: [(self.lib.skv_phase_name(int(tag)).decode(), int(ns - t0)) for tag, ns in marks[r] if tag >= 0]
               for r in range(16)}
        return (s - t0).reshape(-1, 16), (e - t0).reshape(-1, 16), ms.value * 1e3, per

    def shard_outputs(self, slot: int = 0) -> tuple[int, int]:
        """Device addresses of this engine's Stage-II keys and shard-local ids [4][4][100]."""
        k, i = ctypes.c_void_p(), ctypes.c_void_p()
        check(self.lib.skv_shard_outputs(self.handle, slot, ctypes.byref(k), ctypes.byref(i)), "skv_shard_outputs")
        return int(k.value), int(i.value)

    def shard_attention(self, gids: int, token_begin: int, partials: int, stream: int = 0) -> None:
        check(self.lib.skv_shard_attention(self.handle, ctypes.c_void_p(gids), token_begin,
                                           ctypes.c_void_p(partials), ctypes.c_void_p(stream or None)),
              "skv_shard_attention")

    def shard_setup(self, rank: int, n_shards: int, begin: list[int], total: int, sink: int, local: int) -> bytes:
        """Allocate this shard's peer-exchange region; returns its IPC handles (region + FP8 records)."""
        nb = int(self.lib.skv_shard_ipc_handle_bytes())
        h = ctypes.create_string_buffer(nb)
        b = np.asarray(begin, dtype=np.int32)
        check(self.lib.skv_shard_setup(self.handle, rank, n_shards, _ptr(b), total, sink, local, h),
              "skv_shard_setup")
        return h.raw

    def shard_gids_ptr(self) -> int:
        """Device address of the connected group's global winners [4][4][100]."""
        p = ctypes.c_void_p()
        check(self.lib.skv_shard_gids(self.handle, ctypes.byref(p)), "skv_shard_gids")
        return int(p.value)

    def shard_connect(self, handles: bytes) -> None:
        """Map every peer's region (handles of all shards, in shard order)."""
        buf = ctypes.create_string_buffer(handles, len(handles))
        check(self.lib.skv_shard_connect(self.handle, buf), "skv_shard_connect")

    def traffic(self) -> dict:
        t = SkvTraffic()
        check(self.lib.skv_traffic(self.handle, ctypes.byref(t)), "skv_traffic")
        return {n: getattr(t, n) for n, _ in SkvTraffic._fields_}


def shard_merge(keys: int, ids: int, begin: int, n_shards: int, n_cells: int, out_gids: int, stream: int = 0) -> None:
    """Exact global top-100 from every shard's lists (device addresses)."""
    check(load().skv_shard_merge(ctypes.c_void_p(keys), ctypes.c_void_p(ids), ctypes.c_void_p(begin), n_shards,
                                 n_cells, ctypes.c_void_p(out_gids), ctypes.c_void_p(stream or None)),
          "skv_shard_merge")


def shard_combine(partials: int, n_shards: int, n_cells: int, out: int, stream: int = 0) -> None:
    """Log-sum-exp combine of every shard's partials into BF16 output (device addresses)."""
    check(load().skv_shard_combine(ctypes.c_void_p(partials), n_shards, n_cells, ctypes.c_void_p(out),
                                   ctypes.c_void_p(stream or None)), "skv_shard_combine")
