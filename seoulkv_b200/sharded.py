"""Sequence-sharded SeoulKV4 decode: one process and GPU per contiguous token range.

The reference decodes a layer on one device; this module spreads a long
context over the GPUs of one node.  GPU ``r`` of ``n`` holds tokens
``[r*T//n, (r+1)*T//n)`` with its own index, key planes and FP8 records; the
sink zone lives on the first shard and the local window on the last (the
other shards index their whole range, sink = local = 0).  One decode step:

1. every shard runs the funnel on its range (``SeoulKV4.run``) and keeps, per
   query head, its local top-100 with their Stage-II keys;
2. the lists are all-gathered and every GPU merges them into the same exact
   global top-100 (Stage-II score descending, then local rank, then global
   token id: a total order);
3. every shard attends over the winners it owns plus its dense zones and
   produces an un-normalised (m, l, o) partial per query head;
4. the partials are all-gathered and combined by log-sum-exp into the same
   BF16 output on every GPU.

Steps 2-4 are CUDA kernels behind the C ABI.  Two transports move the lists
and partials between GPUs:

* ``"p2p"`` (default with more than one shard): every GPU maps its peers'
  exchange regions and FP8 records once (CUDA IPC handles swapped over the
  process group).  On the fused path the whole step is one launch of the
  funnel kernel: each head's top-100 goes to every peer as tagged 8-byte
  entries (the step counter's low byte, polled with a bound, no flag), every
  GPU merges the lists itself and attends over the global winners and the
  dense zones, reading the records that other shards own over NVLink, so
  steps 3-4 need no exchange of partials.  On the staged path (shards above
  the fused kernel's limits) separate merge, attention and combine kernels
  write into the peers' memory and wait (bounded) on per-step flags, all in
  one CUDA graph with no host round trip;
* ``"nccl"``: two ``torch.distributed`` all-gathers between separate
  merge / attention / combine launches.
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import torch

from . import _native
from .api import SeoulKV4, _check_append, _enqueue_append
from .config import SeoulKV4Config

PART = 260  # floats per (cell, head) partial: m, l, 0, 0, o[256]


@dataclass(frozen=True)
class ShardPlan:
    """Token range and attention zones of shard ``shard`` of ``n_shards``."""

    total: int
    n_shards: int
    shard: int
    sink: int = 128
    local: int = 256

    def __post_init__(self):
        if self.n_shards < 1 or not 0 <= self.shard < self.n_shards:
            raise ValueError("require 0 <= shard < n_shards")
        if self.total < self.n_shards or min(self.sink, self.local) < 0:
            raise ValueError("require total >= n_shards and non-negative zones")
        if self.shard_sink + self.shard_local > self.context:
            raise ValueError("zones do not fit in the shard")

    @property
    def begin(self) -> int:
        return self.shard * self.total // self.n_shards

    @property
    def end(self) -> int:
        return (self.shard + 1) * self.total // self.n_shards

    @property
    def context(self) -> int:
        return self.end - self.begin

    @property
    def shard_sink(self) -> int:
        return self.sink if self.shard == 0 else 0

    @property
    def shard_local(self) -> int:
        return self.local if self.shard == self.n_shards - 1 else 0


class _Dev:
    """A raw device pointer as a torch tensor (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, shape, typestr: str, stream: int):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None, "stream": stream or 1}


class Exchange:
    """All-gather over a process group (or the identity for one shard).

    ``gather(dst, src)`` fills ``dst`` [n_shards, *src.shape] with every
    rank's ``src`` in rank order.
    """

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.size = self.dist.get_world_size(group) if self.dist else 1
        self.rank = self.dist.get_rank(group) if self.dist else 0

    def gather(self, dst: torch.Tensor, src: torch.Tensor) -> None:
        if self.size == 1:
            dst[0].copy_(src)
        elif self.dist.get_backend(self.group) == "nccl":
            self.dist.all_gather_into_tensor(dst.view(-1), src.contiguous().view(-1), group=self.group)
        else:
            parts = [torch.empty_like(src) for _ in range(self.size)]
            self.dist.all_gather(parts, src.contiguous(), group=self.group)
            for r, p in enumerate(parts):
                dst[r].copy_(p)


class ShardedSeoulKV4:
    """This process's shard of a sequence-sharded SeoulKV4 layer.

    ``k``/``v``: this shard's slice, BF16 [4, plan.context, 256]; ``index``: a
    SeoulKV4Index built on that slice with ``sink=plan.shard_sink`` and
    ``local=plan.shard_local``.  ``run(q)`` returns the layer's BF16 output
    [1, 1, 16, 256] on this GPU (the same on every shard); ``group`` is the
    torch.distributed group of the shards (rank r holds shard r).
    """

    def __init__(self, *, device, k, v, index, plan: ShardPlan, config: SeoulKV4Config | None = None,
                 group=None, transport: str | None = None, grow: int = 0):
        zones = index.zones
        if (zones.context, zones.sink, zones.local) != (plan.context, plan.shard_sink, plan.shard_local):
            raise ValueError("index zones do not match the shard plan")
        if type(grow) is not int or grow < 0:
            raise ValueError("grow must be a non-negative token count")
        if grow:  # every shard's engine gets the same room (the last one uses it)
            config = dataclasses.replace(config or SeoulKV4Config(), max_context=plan.context + grow)
        self.plan = plan
        self.grow, self.appended = grow, 0
        self.exchange = Exchange(group)
        if self.exchange.size != plan.n_shards or self.exchange.rank != plan.shard:
            raise ValueError("the process group must hold one rank per shard, rank r = shard r")
        self.attn = SeoulKV4(device=device, k=k, v=v, index=index, config=config)
        dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        n = plan.n_shards
        self.keys_all = torch.empty(n, 4, 4, 100, dtype=torch.int32, device=dev)
        self.ids_all = torch.empty_like(self.keys_all)
        self.begin = torch.tensor([r * plan.total // n for r in range(n)], dtype=torch.int32, device=dev)
        self.gids = torch.empty(4, 4, 100, dtype=torch.int32, device=dev)
        self.part = torch.empty(4, 4, PART, dtype=torch.float32, device=dev)
        self.part_all = torch.empty(n, 4, 4, PART, dtype=torch.float32, device=dev)
        self.out = torch.empty(16, 256, dtype=torch.int16, device=dev)
        self.transport = transport or ("p2p" if n > 1 else "nccl")
        if self.transport not in ("p2p", "nccl"):
            raise ValueError("transport must be 'p2p' or 'nccl'")
        if self.transport == "p2p":
            # the engine now, so that its step graph is captured with the exchange kernels
            self.attn._engine = self.attn._initialize()
            self.attn._host_kv = None
            mine = self.attn._engine.shard_setup(plan.shard, n, [r * plan.total // n for r in range(n)],
                                                 plan.total, plan.sink, plan.local)
            handles = [mine]
            if n > 1:
                handles = [None] * n
                self.exchange.dist.all_gather_object(handles, mine, group=group)
            self.attn._engine.shard_connect(b"".join(handles))

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def run(self, q: torch.Tensor) -> torch.Tensor:
        """One decode step of the whole layer; returns CUDA BF16 [1, 1, 16, 256]."""
        st = self._stream()
        if self.transport == "p2p":
            # funnel + merge + attention + combine, one graph; the engine's output is the layer's
            self.attn.run(q)
            eng = self.attn._engine
            out = torch.as_tensor(_Dev(eng.output_device_ptr(), (16, 256), "<i2", st), device=self.device)
            return out.view(torch.bfloat16).reshape(1, 1, 16, 256)
        self.attn.run(q)  # this shard's funnel (its own attention output is not used)
        eng = self.attn._engine
        kp, ip = eng.shard_outputs(0)
        keys = torch.as_tensor(_Dev(kp, (4, 4, 100), "<i4", st), device=self.device)
        ids = torch.as_tensor(_Dev(ip, (4, 4, 100), "<i4", st), device=self.device)
        n = self.plan.n_shards
        self.exchange.gather(self.keys_all, keys)
        self.exchange.gather(self.ids_all, ids)
        _native.shard_merge(self.keys_all.data_ptr(), self.ids_all.data_ptr(), self.begin.data_ptr(), n, 4,
                            self.gids.data_ptr(), st)
        eng.shard_attention(self.gids.data_ptr(), self.plan.begin, self.part.data_ptr(), st)
        self.exchange.gather(self.part_all, self.part)
        _native.shard_combine(self.part_all.data_ptr(), n, 4, self.out.data_ptr(), st)
        return self.out.view(torch.bfloat16).reshape(1, 1, 16, 256)

    @property
    def total(self) -> int:
        """Tokens in the layer: the plan's total plus every appended token."""
        return self.plan.total + self.appended

    def append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Grow the layer by m tokens: BF16 K and V [4, m, 256] (host or CUDA),
        the same on every rank, which all call this.  The tokens join the last
        shard (it holds the local window, whose oldest tokens enter its
        retrieval zone); with the peer-memory transport every shard's kernel
        learns the layer's new length on the device.  Needs ``grow`` room."""
        m = _check_append(k, v, (4,), 0, 1 << 30)
        if self.appended + m > self.grow:
            raise ValueError(f"append of {m} tokens passes the layer's room to grow ({self.grow - self.appended} "
                             "tokens left; set ShardedSeoulKV4(grow=...))")
        if self.plan.shard == self.plan.n_shards - 1:
            self.attn.append(k, v)
        elif self.transport == "p2p":
            _enqueue_append(self.attn._engine, k, v, self.device.index, self._stream())
        self.appended += m

    def selected_ids(self) -> torch.Tensor:
        """Global token ids of the last step: CUDA int32 [4, 4, 100] (KV head, query head, rank; -1 past the end)."""
        if self.transport == "p2p":
            eng = self.attn._engine
            ptr = eng.shard_gids_ptr()
            return torch.as_tensor(_Dev(ptr, (4, 4, 100), "<i4", self._stream()), device=self.device)
        return self.gids

    def close(self) -> None:
        self.attn.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
