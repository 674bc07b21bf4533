"""Benchmark: µs per layer of SeoulKV4 sparse decode at 128K context on B200.

One step = one decode of one query token through one layer (4 KV heads,
16 query heads, d=256): coarse -> fine -> Stage-1.5 -> Stage-1.6 -> Stage-II
-> FP8 attention.  Each step uses a fresh Q; L2 is flushed (a 256 MiB write)
before every timed step, so the index planes are read cold.  With
``--gpus N`` (torchrun) the layer is sequence-sharded: by default a context
of N x 131072 tokens (weak scaling; 1M at N = 8) split
into contiguous ranges, one per GPU, each with its own index over a mixture
of 2048 components per KV head; ``--total T`` fixes the layer's context
instead (strong scaling).  Every step runs the local funnels, an exact global
top-100 merge and a log-sum-exp combine of the attention partials over
NVLink.  The value is the time per decode step of the whole sharded layer,
max over ranks.

``--impl reference`` times the CPU restatement of the reference pipeline
(the reference ships no runnable CPU decode; its device path needs a
Tenstorrent board) on this host's cores, on the same layer, the same queries
and the same config as the GPU arm.  Both arms define the CPU figure the
same way: the median latency of one decode step, the step's four KV heads on
four threads and each head's scoring loops on cores / 4 more.
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "µs/layer sparse decode at 128K ctx; top-100 ID parity vs ref; achieved HBM GB/s"
UNIT = "µs/layer"
CONFIG_INDEX = 1  # 1xB200 headline profile


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--impl", default="ours", choices=("ours", "reference"))
    p.add_argument("--context", type=int, default=131072)
    p.add_argument("--nprobe", type=int, default=384)
    p.add_argument("--e2e-steps", type=int, default=200)
    p.add_argument("--cpu-steps", type=int, default=5)
    p.add_argument("--components", type=int, default=None,
                   help="mixture components per KV head (default 2048 for the sharded layer, 256 otherwise)")
    p.add_argument("--total", type=int, default=0,
                   help="sharded mode: the layer's whole context (strong scaling); default --context x GPUs")
    p.add_argument("--staged", action="store_true", help="run the 14-kernel staged path instead of the fused one")
    p.add_argument("--layers", type=int, default=0,
                   help="decode-stack mode: L independent layers of --context tokens (BASELINE configs[2])")
    p.add_argument("--requests", type=int, default=0,
                   help="batched mode: R independent requests of --context tokens, split over the GPUs "
                        "(BASELINE configs[4]); sweeps --sweep nprobe values")
    p.add_argument("--sweep", default="16,64,128,256,384,512", help="nprobe values of the batched mode")
    p.add_argument("--append", type=int, default=0,
                   help="decode-loop mode: every step appends this many tokens to the --context cache, then "
                        "decodes one query over the grown cache")
    p.add_argument("--transport", default="p2p", choices=("p2p", "nccl"),
                   help="sharded exchange: peer memory inside the step graph, or NCCL all-gathers")
    a = p.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    sharded = world > 1 and not (a.requests or a.layers or a.append)
    if a.components is None:
        a.components = 2048 if sharded else 256
    return a


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampler (SM clock + throttle reasons) around the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.proc, self.lines = gpu, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


HEADLINE_SEED = CONFIG_INDEX * 1000   # the headline layer (rank 0's layer)
SHARDED_SEED = 3 * 1000               # the sequence-sharded layer


def query_seed(layer_seed: int, i: int) -> int:
    """Seed of the i-th query of a layer (warm-up queries first, then timed)."""
    return layer_seed * 7919 + i


def make_layer(context, nprobe, seed, device):
    from seoulkv_b200 import SeoulKV4Index, synthetic

    k, v, mixes = synthetic.make_kv(context, seed=seed)
    index = SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=nprobe, build_device=device)
    return k, v, mixes, index


def headline_config(args) -> dict:
    """The config dict of the single-layer line (both arms print this one)."""
    return {"workload": "1 layer, 1 query token, T=131072, 4 KV / 16 Q heads, d=256, nprobe=384, "
                        "sink=128, local=256, top-100",
            "context": args.context, "nprobe": args.nprobe,
            "l2": "flushed (256 MiB write) before every step; the layer's centroid planes sit in the persisting "
                  "L2 set-aside (access-policy window), which the flush does not evict",
            "parallelism": "1 GPU"}


def sharded_total(args, world) -> int:
    return args.total or args.context * world


def sharded_config(args, world) -> dict:
    """The config dict of the sequence-sharded line (both arms print this one)."""
    total = sharded_total(args, world)
    per = total // world
    mode = "strong scaling: fixed layer context" if args.total else "weak scaling: fixed context per GPU"
    return {"workload": f"1 layer sequence-sharded over {world} GPUs, T={total} (~{per} per GPU), 4 KV / 16 Q "
                        f"heads, d=256, nprobe={args.nprobe} per shard, sink on the first shard, local on the "
                        "last, exact global top-100",
            "context": total, "context_per_gpu": per, "nprobe": args.nprobe, "components": args.components,
            "scaling_mode": mode, "l2": "flushed before every step",
            "parallelism": f"sequence-sharded x{world}, " + (
                "top-100 lists exchanged over peer memory (NVLink) inside the fused kernel"
                if args.transport == "p2p" else "NCCL all-gathers of top-100 lists and partials"),
            "transport": args.transport}


def oracle_cells(k, index):
    from oracle import oracle as O
    from seoulkv_b200.index import device_view

    kb = k.contiguous().view(torch.int16).numpy().view(np.uint16)
    scales, p2, r2, r4 = O.key_codec(kb)
    cells = []
    for g, c in enumerate(index.cells()):
        dv = device_view(c)
        cells.append(O.CellInputs(
            nc=dv["nc"], nprobe=dv["nprobe"], lam=dv["lam"], upper=dv["upper"], lower=dv["lower"],
            coarse_scale4=dv["coarse_scale4"], fine_scale=dv["fine_scale"], resid_bf16=dv["resid_bf16"],
            offsets=dv["offsets"], values=dv["values"], context=k.shape[1],
            prefix2=p2[g], residual2=r2[g], residual4=r4[g], key_scale=scales[g]))
    return cells


class CpuShard:
    """One layer, or one shard of a sequence-sharded layer, restated on the
    host: the oracle's cell inputs plus the BF16 K/V from which the FP8 records
    of the attended rows are decoded when a step needs them."""

    def __init__(self, k, v, index, begin=0, sink=128, local=256):
        self.cells = oracle_cells(k, index)
        self.k, self.v = k, v
        self.begin, self.context, self.sink, self.local = begin, k.shape[1], sink, local


def cpu_threads() -> int:
    """Host threads a CPU decode step uses: four KV heads x (cores / 4)."""
    return max(4, ((os.cpu_count() or 1) // 4) * 4)


def cpu_decode(shards, q, pool):
    """One decode step of a whole layer on the host: every shard's funnel (the
    four KV heads on the pool's threads, each cell's scoring loops on the
    oracle's OpenMP threads), the exact global top-100 merge when sharded, then
    the attention over the dense zones and the winners.  Returns (per-shard
    run_cell results, global ids [4, 4, 100], BF16 output bits [16, 256])."""
    from oracle import oracle as O

    qb = q.contiguous().view(torch.int16).numpy().view(np.uint16).reshape(16, 256)
    results = [list(pool.map(lambda g, sh=sh: O.run_cell(sh.cells[g], qb[4 * g:4 * g + 4]), range(4)))
               for sh in shards]
    if len(shards) == 1:
        gids = np.stack([r["final_ids"] for r in results[0]])
    else:
        keys = np.stack([[O.stage2_rank_keys(r) for r in res] for res in results])
        ids = np.stack([[r["final_ids"] for r in res] for res in results])
        gids = O.merge_shards(keys, ids, [sh.begin for sh in shards])
    total = shards[-1].begin + shards[-1].context
    dense = np.concatenate([np.arange(shards[0].sink), np.arange(total - shards[-1].local, total)]).astype(np.int64)
    starts = np.array([sh.begin for sh in shards])
    out = np.zeros((16, 256), np.uint16)
    for g in range(4):
        for h in range(4):
            toks = np.concatenate([dense, gids[g, h][gids[g, h] >= 0].astype(np.int64)])
            owner = np.searchsorted(starts, toks, side="right") - 1
            krows = np.empty((len(toks), 256), np.float32)
            vrows = np.empty_like(krows)
            for s, sh in enumerate(shards):
                m = owner == s
                if m.any():
                    loc = torch.from_numpy(toks[m] - sh.begin)
                    krows[m] = sh.k[g].index_select(0, loc).float().numpy()
                    vrows[m] = sh.v[g].index_select(0, loc).float().numpy()
            out[4 * g + h] = O.attention(qb[4 * g + h], O.fp8_e4m3(krows), O.fp8_e4m3(vrows),
                                         np.arange(len(toks)))
    return results, gids, out


def cpu_latencies(shards, qs, warm, steps):
    """Per-step latency (µs) of `steps` CPU decode steps after `warm` untimed
    ones, every step on all host cores (cpu_threads()); also the last step's
    results.  The same definition serves both arms."""
    from oracle import oracle as O

    O.set_threads(cpu_threads() // 4)
    lat, last = [], None
    with ThreadPoolExecutor(max_workers=4) as pool:
        for i in range(warm):
            cpu_decode(shards, qs[i], pool)
        for i in range(steps):
            t0 = time.perf_counter()
            last = cpu_decode(shards, qs[warm + i], pool)
            lat.append((time.perf_counter() - t0) * 1e6)
    O.set_threads(1)
    return np.array(lat), last


def cpu_baseline_line(lat, kind_sample):
    return {"value": float(np.median(lat)), "unit": UNIT, "cores": cpu_threads(), "kind": "port",
            "definition": "median latency of one decode step, all host threads",
            "mean_us": float(np.mean(lat)), "steps": int(len(lat)), "sample": kind_sample}


def run_reference(args):
    """CPU arm: the oracle port of the reference pipeline on host cores, on the
    GPU arm's layer, queries and config; exactly K timed steps after W untimed
    ones, value = median step latency."""
    world, rank, _ = dist_env()
    if rank != 0:
        return
    from seoulkv_b200 import SeoulKV4Index, synthetic
    from seoulkv_b200.sharded import ShardPlan

    dev = "cuda:0" if torch.cuda.is_available() else "cpu"
    steps, warm = max(1, args.steps), max(0, args.warmup)
    if world > 1:
        total = sharded_total(args, world)
        shards, mixes = [], None
        for r in range(world):
            plan = ShardPlan(total, world, r)
            k, v, mixes = synthetic.make_kv_range(total, plan.begin, plan.end, seed=SHARDED_SEED,
                                                  components=args.components)
            index = SeoulKV4Index.build(k, v, sink=plan.shard_sink, local=plan.shard_local, nprobe=args.nprobe,
                                        build_device=dev)
            shards.append(CpuShard(k, v, index, plan.begin, plan.shard_sink, plan.shard_local))
        qs = [synthetic.make_query(total, mixes, seed=query_seed(SHARDED_SEED, i)) for i in range(warm + steps)]
        config = sharded_config(args, world)
        sample = (f"{steps} decode steps of the whole {total}-token layer: all {world} shards' funnels in turn, "
                  "the global merge and the attention (C restatement of the reference funnel)")
    else:
        k, v, mixes, index = make_layer(args.context, args.nprobe, HEADLINE_SEED, dev)
        shards = [CpuShard(k, v, index)]
        qs = [synthetic.make_query(args.context, mixes, seed=query_seed(HEADLINE_SEED, i))
              for i in range(warm + steps)]
        config = headline_config(args)
        sample = (f"{steps} decode steps of the {args.context}-token layer (fresh Q each; "
                  "C restatement of the reference funnel)")
    lat, _ = cpu_latencies(shards, qs, warm, steps)
    us = float(np.median(lat))
    line = {
        "metric": METRIC, "value": us, "unit": UNIT, "n_gpus": world, "steps": steps, "warmup": warm,
        "ms_per_step": us / 1e3, "higher_is_better": False, "scaling": "weak" if not args.total else "strong",
        "vs_baseline": None, "dtype": "int64-exact dots, f32 post-ops, bf16 scores, f64 softmax",
        "data": "synthetic (BASELINE generator, seeded), fresh Q per step", "impl": "reference",
        "config": config, "p50_us": us, "mean_us": float(np.mean(lat)), "p99_us": float(np.percentile(lat, 99)),
        "cpu_baseline": cpu_baseline_line(lat, sample),
        "e2e": {"value": us, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_sharded(args, world, rank, local, device):
    """The sequence-sharded layer: N x args.context tokens, one range per rank."""
    import torch.distributed as dist

    from oracle import oracle as O
    from seoulkv_b200 import SeoulKV4Config, SeoulKV4Index, synthetic
    from seoulkv_b200.sharded import ShardedSeoulKV4, ShardPlan

    total = sharded_total(args, world)
    plan = ShardPlan(total, world, rank)
    seed = SHARDED_SEED
    k, v, mixes = synthetic.make_kv_range(total, plan.begin, plan.end, seed=seed, components=args.components)
    index = SeoulKV4Index.build(k, v, sink=plan.shard_sink, local=plan.shard_local, nprobe=args.nprobe,
                                build_device=str(device))
    sh = ShardedSeoulKV4(device=device, k=k, v=v, index=index, plan=plan, config=SeoulKV4Config(debug=True),
                         transport=args.transport)
    n_q = args.warmup + args.steps
    qs_host = [synthetic.make_query(total, mixes, seed=query_seed(seed, i)) for i in range(max(n_q, args.e2e_steps + 2))]
    q_dev = [q.to(device) for q in qs_host[:n_q]]
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for i in range(args.warmup):
        flush.zero_()
        sh.run(q_dev[i])
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = Clocks(local)
    dist.barrier()
    torch.cuda.synchronize(device)
    clocks.start()
    time.sleep(0.3)
    # every host enqueues ahead of its device (a device-side sleep long
    # enough for the host to queue the whole timed loop, ~150 us of host time
    # per step at most; no garbage collection meanwhile), so that the GPUs
    # run their steps back to back and meet at each step's list exchange, as
    # a decode loop does; otherwise a step would also carry the hosts' launch
    # skew and any pause of one host would stall every GPU at the exchange
    gc.disable()
    torch.cuda._sleep(int(2e7 + args.steps * 150e-6 * 2.0e9))
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        sh.run(q_dev[args.warmup + i])
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    gc.enable()
    dist.barrier()
    clk = clocks.stop()
    per = np.array([a.elapsed_time(b) for a, b in zip(starts, ends)]) * 1e3  # µs
    t = torch.tensor([float(per.sum())], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    value = float(t.item()) / args.steps

    # this shard's funnel alone (one non-graph launch, L2 flushed), every rank
    fun = []
    for _ in range(5):
        flush.zero_()
        torch.cuda.synchronize(device)
        fun.append(sum(ms for _, ms in sh.attn._engine.profile_step(stream.cuda_stream)) * 1e3)
    fun_all = torch.empty(world, dtype=torch.float64, device=device)
    dist.all_gather_into_tensor(fun_all, torch.tensor([float(np.median(fun))], dtype=torch.float64, device=device))
    shard_funnel_us = [round(float(x), 1) for x in fun_all.cpu()]
    # phase marks of one whole group step on every rank (fused path only):
    # the profiled step follows two back-to-back steps, so the ranks meet as
    # in the timed loop; "shard_list_exchange" is the wait for the other
    # shards' top-100 lists, "attn_items" the attention over the merged
    # winners (records of other shards read over NVLink)
    phases = None
    if sh.attn._engine.fused and args.transport == "p2p":
        mhz = (clk or {}).get("sm_mhz") or 1965.0
        acc = {}
        for rep in range(3):
            torch.cuda.synchronize(device)
            dist.barrier()
            torch.cuda._sleep(int(2e6))
            for j in range(2):
                flush.zero_()
                sh.run(q_dev[j])
            flush.zero_()
            for name, cyc in sh.attn._engine.profile_phases(stream.cuda_stream):
                acc[name] = acc.get(name, 0.0) + cyc / 3
        mine = {n: round(v / mhz, 2) for n, v in acc.items()}
        every = [None] * world
        dist.all_gather_object(every, mine)
        phases = {f"rank{r}": every[r] for r in range(world)}

    # parity: this shard's funnel vs the CPU restatement (ids bit-exact); the
    # merge vs the restated merge rule on the gathered lists; one output on
    # every rank
    qi = args.warmup + args.steps - 1
    out = sh.run(q_dev[qi]).clone()
    torch.cuda.synchronize(device)
    cells = oracle_cells(k, index)
    qb = q_dev[qi].cpu().contiguous().view(torch.int16).numpy().view(np.uint16).reshape(16, 256)
    with ThreadPoolExecutor(max_workers=4) as pool:
        res = list(pool.map(lambda g: O.run_cell(cells[g], qb[4 * g:4 * g + 4]), range(4)))
    local_ok = np.array_equal(sh.attn.debug_snapshot()["selected_ids"].numpy(),
                              np.stack([r["final_ids"] for r in res]))
    begin = [ShardPlan(total, world, r).begin for r in range(world)]
    from seoulkv_b200.sharded import _Dev

    kp, ip = sh.attn._engine.shard_outputs(0)
    mine = torch.stack([torch.as_tensor(_Dev(p, (4, 4, 100), "<i4", stream.cuda_stream), device=device)
                        for p in (kp, ip)]).clone()
    lists = torch.empty(world, 2, 4, 4, 100, dtype=torch.int32, device=device)
    dist.all_gather_into_tensor(lists.view(-1), mine.view(-1))
    lists = lists.cpu().numpy()
    merged = O.merge_shards(lists[:, 0].view(np.uint32), lists[:, 1], begin)
    merge_ok = np.array_equal(merged, sh.selected_ids().cpu().numpy())
    outs = torch.empty(world, *out.shape, dtype=out.dtype, device=device)
    dist.all_gather_into_tensor(outs.view(-1), out.contiguous().view(-1))
    same_out = bool(all(torch.equal(outs[0], outs[r]) for r in range(world)))
    flags = torch.tensor([int(local_ok), int(merge_ok)], device=device)
    dist.all_reduce(flags, op=dist.ReduceOp.MIN)
    parity = {"local_ids_bit_exact_all_shards": bool(flags[0]), "global_merge_exact": bool(flags[1]),
              "same_output_on_every_rank": same_out,
              "note": "per-shard funnel ids vs the CPU restatement, global merge vs the restated merge rule"}

    # end to end through the public API: pinned host Q -> run -> host output;
    # each step timed alone after an L2 flush (as the device-timed value),
    # then a back-to-back loop with L2 warm
    qp = [q.pin_memory() for q in qs_host[:args.e2e_steps + 2]]
    for i in range(2):
        sh.run(qp[i]).cpu()
    cold = []
    for i in range(args.e2e_steps):
        flush.zero_()
        torch.cuda.synchronize(device)
        dist.barrier()
        t0 = time.perf_counter()
        sh.run(qp[i + 2]).cpu()
        cold.append(time.perf_counter() - t0)
    dist.barrier()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        sh.run(qp[i + 2]).cpu()
    e2e_us = torch.tensor([float(np.mean(cold)) * 1e6, (time.perf_counter() - t0) / max(1, args.e2e_steps) * 1e6],
                          device=device, dtype=torch.float64)
    dist.all_reduce(e2e_us, op=dist.ReduceOp.MAX)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": value / 1e3, "higher_is_better": False,
            "scaling": "strong" if args.total else "weak",
            "vs_baseline": None, "dtype": "int8 (exact digit dots, int32/int64 accumulation), f32 softmax, bf16 scores, fp8 K/V",
            "data": "synthetic (BASELINE generator, seeded, block-seeded per token range), fresh Q per step",
            "config": sharded_config(args, world),
            "p50_us": float(np.percentile(per, 50)), "p99_us": float(np.percentile(per, 99)),
            "tokens_per_s": 1e6 / value, "shard_funnel_us": shard_funnel_us, "phase_us": phases, "parity": parity,
            "cpu_baseline": None,
            "e2e": {"value": float(e2e_us[0].item()), "unit": UNIT, "h2d_bytes_per_step": 16 * 256 * 2,
                    "d2h_bytes_per_step": 16 * 256 * 2, "l2_warm_value": float(e2e_us[1].item()),
                    "timing": "host wall clock of run(pinned Q) + host readback, each step after an L2 flush "
                              "and a barrier (value) or back to back with L2 warm (l2_warm_value); mean, max over ranks"},
            "clocks": clk,
            # our kernels per step on each GPU: the funnel (one fused kernel, which
            # also exchanges and merges over peer memory, or the 14 staged ones
            # plus merge, attention, combine and step-counter kernels), or, with
            # the NCCL transport, the funnel plus merge, attention and combine
            "gpu_launches": (sh.attn._engine.kernels_per_step()
                             + ((0 if sh.attn._engine.fused else 4) if args.transport == "p2p" else 3))
                            * args.steps * world,
        }
        print(json.dumps(line), flush=True)
    sh.close()
    dist.barrier()
    dist.destroy_process_group()


def _timed_steps(args, device, flush, step_fn):
    """W untimed steps, then K steps each after an L2 flush, CUDA events around
    each step on the current stream; returns the per-step times (us)."""
    stream = torch.cuda.current_stream(device)
    for i in range(args.warmup):
        if flush is not None:
            flush.zero_()
        step_fn(i)
    torch.cuda.synchronize(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    gc.disable()
    torch.cuda._sleep(int(2e7))  # the host enqueues ahead of the device
    for i in range(args.steps):
        if flush is not None:  # (None: steps back to back, L2 warm)
            flush.zero_()
        ev[i][0].record(stream)
        step_fn(args.warmup + i)
        ev[i][1].record(stream)
    torch.cuda.synchronize(device)
    gc.enable()
    return np.array([a.elapsed_time(b) * 1e3 for a, b in ev])


def run_stack(args, device):
    """a stack of independent layers on one GPU.  Per
    token: every layer decodes its own query.  Timed two ways: the drop-in
    use (one SeoulKV4 per layer, run one after the other) and one
    SeoulKV4Batch over all layers (one launch per token).  Reports the
    per-token latency summed over layers and the HBM footprint."""
    from seoulkv_b200 import SeoulKV4, SeoulKV4Batch, SeoulKV4Config, synthetic

    L = args.layers
    cfg = SeoulKV4Config(debug=True)
    # engines allocate with cudaMalloc: their footprint is the drop in free
    # device memory minus what PyTorch's allocator reserved meanwhile
    def engine_bytes():
        return torch.cuda.mem_get_info(device)[0] + torch.cuda.memory_reserved(device)

    free0 = engine_bytes()
    caches, qs, singles = [], [], []
    for layer in range(L):
        seed = 2 * 1000 + layer
        k, v, mixes = synthetic.make_kv(args.context, seed=seed, components=args.components)
        from seoulkv_b200 import SeoulKV4Index
        index = SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=args.nprobe, build_device=str(device))
        qs.append(torch.stack([synthetic.make_query(args.context, mixes, seed=seed * 7919 + i).reshape(1, 16, 256)
                               for i in range(args.warmup + args.steps)]).to(device))
        kd, vd = k.to(device), v.to(device)
        caches.append((kd, vd, index))
        a = SeoulKV4(device=device, k=kd, v=vd, index=index, config=cfg)
        a.run(qs[-1][0].unsqueeze(0))
        a.synchronize()
        singles.append(a)
    torch.cuda.synchronize(device)
    free1 = engine_bytes()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)

    def seq_step(i):
        for layer in range(L):
            singles[layer].run(qs[layer][i].unsqueeze(0))

    t_seq = _timed_steps(args, device, flush, seq_step)
    ids_seq = [a.debug_snapshot()["selected_ids"] for a in singles]
    for a in singles:
        a.close()
    free2 = engine_bytes()
    batch = SeoulKV4Batch(device=device, caches=caches, config=cfg)
    q_all = torch.cat(qs, 1)  # [steps, L, 16, 256]
    batch.run(q_all[0].unsqueeze(1))
    batch.synchronize()
    free3 = engine_bytes()
    t_bat = _timed_steps(args, device, flush, lambda i: batch.run(q_all[i].unsqueeze(1)))
    ids_bat = batch.debug_snapshot()["selected_ids"]
    same = all(torch.equal(ids_bat[layer], ids_seq[layer]) for layer in range(L))
    batch.close()
    line = {
        "metric": f"us/token, {L}-layer decode stack at {args.context // 1024}K ctx (per-token latency summed over "
                  "layers)",
        "value": float(np.mean(t_bat)), "unit": "us/token", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": False, "data": "synthetic (BASELINE generator, one seed per "
                                                                  "layer), fresh Q per layer and token",
        "config": {"workload": f"{L} independent layers, T={args.context}, 4 KV / 16 Q heads, d=256, "
                               f"nprobe={args.nprobe}", "l2": "flushed before every token"},
        "batched_one_launch_us": float(np.mean(t_bat)), "batched_p50_us": float(np.median(t_bat)),
        "sequential_layers_us": float(np.mean(t_seq)), "sequential_p50_us": float(np.median(t_seq)),
        "us_per_layer_batched": float(np.mean(t_bat)) / L, "us_per_layer_sequential": float(np.mean(t_seq)) / L,
        "hbm_footprint_gb": {"engines_one_instance_per_layer": (free0 - free1) / 1e9,
                             "engine_batched": (free2 - free3) / 1e9,
                             "bf16_kv_kept_by_the_benchmark": 2 * L * args.context * 4 * 256 * 2 / 1e9},
        "ids_same_sequential_and_batched": same,
    }
    print(json.dumps(line))


def run_append(args, device):
    """A growing cache at the headline context: every step appends M new
    tokens (K/V already on the device, as a model's projection leaves them)
    and decodes one fresh query over the grown cache.  Reports the append,
    the decode after it and the whole step, plus a parity check of the
    appended tokens' lists and the live CSR against the CPU restatement."""
    from oracle import oracle as O
    from seoulkv_b200 import SeoulKV4, SeoulKV4Config, SeoulKV4Index, synthetic
    from seoulkv_b200.index import device_view

    M, T0 = args.append, args.context
    n = args.warmup + args.steps
    total = T0 + n * M
    seed = CONFIG_INDEX * 1000 + 600
    k, v, mixes = synthetic.make_kv(total, seed=seed, components=args.components)
    k0, v0 = k[:, :T0].contiguous(), v[:, :T0].contiguous()
    index = SeoulKV4Index.build(k0, v0, sink=128, local=256, nprobe=args.nprobe, build_device=str(device))
    kn = [k[:, T0 + i * M:T0 + (i + 1) * M].contiguous().to(device) for i in range(n)]
    vn = [v[:, T0 + i * M:T0 + (i + 1) * M].contiguous().to(device) for i in range(n)]
    qs = torch.stack([synthetic.make_query(T0 + (i + 1) * M, mixes, seed=seed * 7919 + i)
                      for i in range(n)]).to(device)
    attn = SeoulKV4(device=device, k=k0, v=v0, index=index, config=SeoulKV4Config(debug=True, max_context=total))
    attn.run(synthetic.make_query(T0, mixes, seed=seed).to(device)).to_torch()
    eng = attn._engine
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    qbits = qs.view(torch.int16)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(n)]
    torch.cuda.synchronize(device)
    h0 = time.perf_counter()
    for i in range(args.warmup):
        flush.zero_()
        attn.append(kn[i], vn[i])
        eng.step(qbits[i].data_ptr(), True, stream.cuda_stream)
    host_us = (time.perf_counter() - h0) / max(args.warmup, 1) * 1e6  # enqueue cost of one step
    torch.cuda.synchronize(device)
    clocks = Clocks(device.index)
    clocks.start()
    time.sleep(0.3)
    gc.disable()
    # the host enqueues the whole timed loop while the device sleeps, so the
    # events time the device alone (the host's enqueue cost is reported apart)
    torch.cuda._sleep(int(2e7 + 1.5 * host_us * 1e-6 * args.steps * 2.0e9))
    for i in range(args.warmup, n):
        flush.zero_()
        ev[i][0].record(stream)
        attn.append(kn[i], vn[i])
        ev[i][1].record(stream)
        eng.step(qbits[i].data_ptr(), True, stream.cuda_stream)
        ev[i][2].record(stream)
    torch.cuda.synchronize(device)
    gc.enable()
    clk = clocks.stop()
    eng.sync()
    t_app = np.array([ev[i][0].elapsed_time(ev[i][1]) * 1e3 for i in range(args.warmup, n)])
    t_dec = np.array([ev[i][1].elapsed_time(ev[i][2]) * 1e3 for i in range(args.warmup, n)])
    assert attn.context == total and eng.current_context() == total

    # parity: the appended tokens' lists (a sample, against the restatement),
    # and the whole live CSR rebuilt on the CPU from the device's lists
    first = T0 - 256
    labels = eng.read_stage(0, "labels", np.int32, (4, total, 2))
    rng = np.random.default_rng(seed)
    sample = np.sort(rng.choice(np.arange(T0, total), size=min(8, total - T0), replace=False))
    kb = k.contiguous().view(torch.int16).numpy().view(np.uint16)
    views = [device_view(c) for c in index.cells()]
    lab_ok = all(np.array_equal(labels[g, sample], O.assign_spill2(kb[g, sample], views[g]["upper"],
                                                                   views[g]["lower"], views[g]["fine_scale"]))
                 for g in range(4))
    csr = eng.read_csr(0)
    csr_ok = True
    for g in range(4):
        want = O.append_postings(views[g]["offsets"], views[g]["values"], views[g]["mates"],
                                 np.arange(first, total - 256), labels[g, first:total - 256])
        csr_ok &= all(np.array_equal(a, b) for a, b in zip(csr[g], want))
    # algorithmic bytes of one append: the centroid codes read by the
    # assignment, the CSR read and rewritten, the new tokens' K/V read and
    # their planes and records written
    nc = views[0]["nc"]
    post = int(sum(int(c[0][-1]) for c in csr)) / 4
    app_bytes = 4 * (nc * 128 + 2 * (nc + 1) * 4 + 2 * 2 * post * 4 + M * (2 * 512 + 64 + 64 + 128 + 512))
    # tensor work of the assignment: per group of 4 new keys and cell, 16
    # int8 m16n8k32 MMAs (4096 multiply-adds each) per 16-centroid tile
    int8_ops = 4 * (nc // 16) * 16 * 4096 * 2 * ((M + 3) // 4)
    a_mean = float(np.mean(t_app))
    line = {
        "metric": f"us per decode-loop step at {T0 // 1024}K ctx: append {M} token(s), then one sparse decode",
        "value": float(np.mean(t_app + t_dec)), "unit": "us/step", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": False,
        "data": "synthetic (BASELINE generator), new K/V tokens of the same mixture, fresh Q at the grown context",
        "config": {"workload": f"T={T0} grown by {M} token(s) per step to {total}, 4 KV / 16 Q heads, d=256, "
                               f"nprobe={args.nprobe}", "l2": "flushed before every step"},
        "append_us": a_mean, "append_p50_us": float(np.median(t_app)), "append_p99_us": float(np.percentile(t_app, 99)),
        "decode_us": float(np.mean(t_dec)), "decode_p50_us": float(np.median(t_dec)),
        "host_enqueue_us_per_step": host_us,
        "append_algorithmic_bytes": app_bytes, "append_gbs": app_bytes / (a_mean * 1e-6) / 1e9,
        "append_int8_ops": int8_ops, "append_int8_tops": int8_ops / (a_mean * 1e-6) / 1e12,
        "parity": {"sampled_token_lists_equal_restatement": bool(lab_ok), "live_csr_equals_restatement": bool(csr_ok),
                   "sample_tokens": sample.tolist()},
        "clocks": clk,
    }
    attn.close()
    print(json.dumps(line))


def run_requests(args, world, rank, device):
    """independent requests (one query token each) split
    contiguously over the GPUs (no collective on the data path), decoded as one
    SeoulKV4Batch per GPU; nprobe swept; top-100 recall against the exact dense
    top-100 of q.k over each request's retrieval tokens."""
    from seoulkv_b200 import SeoulKV4Batch, SeoulKV4Config, SeoulKV4Index, synthetic

    R = args.requests
    lo, hi = R * rank // world, R * (rank + 1) // world
    caches, qs = [], []
    for r in range(lo, hi):
        seed = 4 * 1000 + r
        k, v, mixes = synthetic.make_kv(args.context, seed=seed, components=args.components)
        index = SeoulKV4Index.build(k, v, sink=128, local=256, nprobe=max(int(x) for x in args.sweep.split(",")),
                                    build_device=str(device))
        caches.append((k.to(device), v.to(device), index))
        qs.append(torch.stack([synthetic.make_query(args.context, mixes, seed=seed * 7919 + i).reshape(1, 16, 256)
                               for i in range(args.warmup + args.steps)]).to(device))
    q_all = torch.cat(qs, 1)  # [steps, n, 16, 256]
    n = hi - lo
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    T = args.context
    sweep = []
    for p in (int(x) for x in args.sweep.split(",")):
        batch = SeoulKV4Batch(device=device, caches=caches, config=SeoulKV4Config(nprobe=p, debug=True))
        err = "another GPU's first run failed"
        try:
            batch.run(q_all[0].unsqueeze(1))
            batch.synchronize()
            ok = torch.ones(1, device=device)
        except (ValueError, RuntimeError) as exc:
            # the reference's first run raises the same way (a Stage-1.5 pool
            # below 2048 keys or above capacity): this nprobe does not apply
            ok = torch.zeros(1, device=device)
            err = str(exc).split(";")[0]
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if ok.item() == 0:
            batch.close()
            sweep.append({"nprobe": p, "not_applicable": err})
            continue
        t = _timed_steps(args, device, flush, lambda i: batch.run(q_all[i].unsqueeze(1)))
        # recall of the last step's ids against the exact dense top-100 (retrieval zone)
        ids = batch.debug_snapshot()["selected_ids"].to(device)  # [n, 4, 4, 100]
        qlast = q_all[args.warmup + args.steps - 1].float()       # [n, 16, 256]
        hits = 0
        for j, (k, _, _) in enumerate(caches):
            kz = k[:, 128:T - 256].float()                          # [4, R, 256]
            sc = torch.einsum("ghd,grd->ghr", qlast[j].view(4, 4, 256), kz)
            top = sc.topk(100, dim=-1).indices + 128                # [4, 4, 100]
            for g in range(4):
                for h in range(4):
                    hits += int(torch.isin(ids[j, g, h], top[g, h]).sum())
        batch.close()
        step_us = torch.tensor([float(np.mean(t))], device=device)
        hit_t = torch.tensor([float(hits), float(n * 16 * 100)], device=device)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(step_us, op=dist.ReduceOp.MAX)
            dist.all_reduce(hit_t)
        sweep.append({"nprobe": p, "us_per_step": float(step_us.item()), "tokens_per_s": R / step_us.item() * 1e6,
                      "recall_at_100": float(hit_t[0] / hit_t[1])})
    if rank == 0:
        ran = [x for x in sweep if "tokens_per_s" in x]
        best = max(ran, key=lambda x: x["tokens_per_s"]) if ran else {"tokens_per_s": 0.0}
        line = {
            "metric": f"tokens/s batched decode, {R} requests x {T // 1024}K ctx; top-100 recall vs exact dense",
            "value": best["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "data": "synthetic (BASELINE generator, one seed per request), fresh Q per step",
            "config": {"workload": f"{R} independent requests, T={T}, 4 KV / 16 Q heads, d=256, one query token "
                                   f"each, requests split contiguously over {world} GPU(s)",
                       "l2": "flushed before every step"},
            "sweep": sweep,
        }
        print(json.dumps(line))


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    world, rank, local = dist_env()
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    device = torch.device(f"cuda:{local}")
    torch.cuda.set_device(device)
    from seoulkv_b200 import _native

    _native.FORCE_STAGED = args.staged
    if args.requests:
        run_requests(args, world, rank, device)
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()
        return
    if args.layers:
        run_stack(args, device)
        return
    if args.append:
        run_append(args, device)
        return
    if world > 1:
        run_sharded(args, world, rank, local, device)
        return
    from seoulkv_b200 import SeoulKV4, SeoulKV4Config, synthetic

    seed = HEADLINE_SEED
    k, v, mixes, index = make_layer(args.context, args.nprobe, seed, str(device))
    n_q = args.warmup + args.steps
    qs_host = [synthetic.make_query(args.context, mixes, seed=query_seed(seed, i))
               for i in range(max(n_q, args.e2e_steps + 2))]
    q_dev = torch.stack([q.reshape(16, 256) for q in qs_host[:n_q]]).to(device)
    attn = SeoulKV4(device=device, k=k, v=v, index=index, config=SeoulKV4Config(debug=True))
    attn.run(qs_host[0])
    attn.synchronize()
    eng = attn._engine
    stream = torch.cuda.current_stream(device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    qbits = q_dev.view(torch.int16)

    def step(i):
        eng.step(qbits[i].data_ptr(), True, stream.cuda_stream)

    for i in range(args.warmup):
        flush.zero_()
        step(i)
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    clocks = Clocks(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    clocks.start()
    time.sleep(0.3)
    # the host enqueues ahead of the device (a short device-side sleep before
    # the first timed step; no garbage collection meanwhile), so that no host
    # pause falls between a step's start event and its launch
    gc.disable()
    torch.cuda._sleep(int(2e7))
    for i in range(args.steps):
        flush.zero_()
        starts[i].record(stream)
        step(args.warmup + i)
        ends[i].record(stream)
    torch.cuda.synchronize(device)
    gc.enable()
    if world > 1:
        torch.distributed.barrier()
    clk = clocks.stop()
    per = np.array([s.elapsed_time(e) for s, e in zip(starts, ends)]) * 1e3  # µs
    total_us = float(per.sum())
    if world > 1:
        t = torch.tensor([total_us], device=device, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_us = float(t.item())
    eng.sync()  # status check of the last step
    value = total_us / (world * args.steps)

    # the same kind of steps without the L2 window (centroid planes read from
    # HBM after every flush), for comparison; the window is restored after
    window_bytes = int(getattr(eng, "l2_resident_bytes", 0))
    no_window = None
    if window_bytes:
        eng.set_l2_residency(False)
        t_nw = _timed_steps(argparse.Namespace(warmup=args.warmup, steps=min(args.steps, 200)), device, flush, step)
        eng.set_l2_residency(True)
        no_window = {"mean_us": float(np.mean(t_nw)), "p50_us": float(np.median(t_nw)),
                     "p99_us": float(np.percentile(t_nw, 99)), "steps": int(len(t_nw))}

    # steady state: the same steps back to back without the L2 flush (a decode
    # loop that revisits this layer finds its code and recent rows in L2)
    t_w = _timed_steps(argparse.Namespace(warmup=args.warmup, steps=min(args.steps, 200)), device, None, step)
    l2_warm = {"mean_us": float(np.mean(t_w)), "p50_us": float(np.median(t_w)),
               "p99_us": float(np.percentile(t_w, 99)), "steps": int(len(t_w)),
               "what": "steps back to back without the L2 flush (steady state); value flushes before every step"}

    # the same kind of steps on a second instance of the layer without the
    # lead cluster (the fused launch's extra cluster that runs a small
    # synthetic cell ahead of the real cells, bringing the kernel's
    # instructions into L2 before they need them), for comparison
    no_lead = None
    if eng.fused:
        attn2 = SeoulKV4(device=device, k=k, v=v, index=index, config=SeoulKV4Config(debug=True, lead_cluster=False))
        attn2.run(qs_host[0])
        attn2.synchronize()
        eng2 = attn2._engine
        t_nl = _timed_steps(argparse.Namespace(warmup=args.warmup, steps=min(args.steps, 200)), device, flush,
                            lambda i: eng2.step(qbits[i].data_ptr(), True, stream.cuda_stream))
        eng2.sync()
        attn2.close()
        no_lead = {"mean_us": float(np.mean(t_nl)), "p50_us": float(np.median(t_nl)),
                   "p99_us": float(np.percentile(t_nl, 99)), "steps": int(len(t_nl))}

    # per-kernel device times (non-graph launches, L2 flushed before each)
    prof = {}
    for _ in range(5):
        flush.zero_()
        step(args.warmup)  # same Q as a timed step, then re-run kernel by kernel
        torch.cuda.synchronize(device)
        flush.zero_()
        eng.bind_query(qbits[args.warmup].data_ptr(), True, stream.cuda_stream)
        for name, ms in eng.profile_step(stream.cuda_stream):
            prof.setdefault(name, []).append(ms)
    prof = {n: float(np.mean(v)) * 1e3 for n, v in prof.items()}  # µs
    traffic = eng.traffic()
    if "k_funnel" in prof:
        # fused path: one kernel carries the whole step
        dom, dom_bytes = "k_funnel", traffic["total"]
    else:
        stage_bytes = {"k_coarse": traffic["coarse"], "k_fine": traffic["fine"], "k_pool_s15": traffic["stage15"],
                       "k_s16": traffic["stage16"], "k_s2_score": traffic["stage2"], "k_attn": traffic["attention"]}
        dom = max(stage_bytes, key=lambda n: prof.get(n, 0.0))
        dom_bytes = stage_bytes[dom]
    peak, peak_kind = peaks()
    achieved = dom_bytes / (prof[dom] * 1e-6) / 1e9
    roof = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
            "traffic": None, "algorithmic_bytes": dom_bytes, "kernel_us": prof[dom],
            "timing": "CUDA events around one non-graph launch, L2 flushed (normal lines)"}
    if window_bytes and dom == "k_funnel":
        # bytes the window serves from persisting L2: the coarse scan's upper
        # plane (nc x 64 per cell) and the Fine rows of the survivors (128 of
        # the 132 bytes charged per survivor)
        nc = index.cells()[0]["centroids"].shape[0]
        resident = 4 * nc * 64 + traffic["fine"] * 128.0 / 132.0
        roof.update(l2_window_bytes=window_bytes, l2_resident_algorithmic_bytes=resident,
                    hbm_algorithmic_bytes=dom_bytes - resident,
                    hbm_achieved=(dom_bytes - resident) / (prof[dom] * 1e-6) / 1e9,
                    hbm_frac=(dom_bytes - resident) / (prof[dom] * 1e-6) / 1e9 / peak)
    ncu_note = ROOT / "profiles" / "traffic_128k.json"
    if ncu_note.exists():
        try:
            roof["traffic"] = json.loads(ncu_note.read_text()).get(dom)
        except Exception:
            pass
    # fused path: SM cycles per phase (CTA 0 of KV head 0), summed over repeats
    phases = None
    if eng.fused:
        mhz = (clk or {}).get("sm_mhz") or 1965.0
        acc = {}
        for _ in range(3):
            flush.zero_()
            torch.cuda.synchronize(device)
            for name, cyc in eng.profile_phases(stream.cuda_stream):
                acc.setdefault(name, [0.0, 0])
                acc[name][0] += cyc
            for name in acc:
                acc[name][1] += 1
        phases = {n: round(v[0] / v[1] / mhz, 2) for n, v in acc.items()}

    # parity of the last timed step against the CPU restatement; the CPU
    # baseline: the same restatement's median step latency on all host cores
    # (the reference arm's definition), on the first --cpu-steps timed queries
    from oracle import oracle as O

    shard = CpuShard(k, v, index)
    qi = args.warmup + args.steps - 1
    step(qi)
    ids = eng.debug_ids()[0]
    out = eng.output_host()[0]
    n_cpu = max(1, min(args.cpu_steps, args.steps))
    lat, _ = cpu_latencies([shard], qs_host, args.warmup, n_cpu)
    _, gids, ref_out = cpu_latencies([shard], [q_dev[qi].cpu().reshape(1, 1, 16, 256)], 0, 1)[1]
    err = np.abs(O.bf16_to_f32(out).astype(np.float64) - O.bf16_to_f32(ref_out).astype(np.float64))
    parity = {"ids_bit_exact": bool(np.array_equal(ids, gids)), "out_max_abs": float(err.max()),
              "out_mean_abs": float(err.mean()), "tolerance": [2e-2, 2e-3], "step": "last timed step"}
    cpu_line = cpu_baseline_line(lat, f"the first {n_cpu} timed queries of this {args.context}-token layer, one step at a time "
                                      "(C restatement of the reference funnel)")

    # end to end through the public API: pinned host Q -> run -> to_torch.
    # value: each step timed alone after an L2 flush and a device sync (the
    # device-timed value's L2 condition); l2_warm_value: back to back
    qp = [q.pin_memory() for q in qs_host[:args.e2e_steps + 2]]
    for i in range(2):
        attn.run(qp[i]).to_torch()
    cold = []
    for i in range(args.e2e_steps):
        flush.zero_()
        torch.cuda.synchronize(device)
        t0 = time.perf_counter()
        attn.run(qp[i + 2]).to_torch()
        cold.append((time.perf_counter() - t0) * 1e6)
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        attn.run(qp[i + 2]).to_torch()
    warm_us = (time.perf_counter() - t0) / args.e2e_steps * 1e6
    e2e = {"value": float(np.mean(cold)), "unit": UNIT, "h2d_bytes_per_step": 16 * 256 * 2,
           "d2h_bytes_per_step": 16 * 256 * 2, "p50": float(np.median(cold)), "l2_warm_value": warm_us,
           "timing": "host wall clock of run(pinned Q).to_torch(), each step alone after an L2 flush and a "
                     "device sync (value, p50), or back to back with L2 warm (l2_warm_value)"}

    if rank == 0:
        st = eng.status()
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": value / 1e3, "higher_is_better": False,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 (exact digit dots, int32/int64 accumulation), f32 softmax, bf16 scores, fp8 K/V",
            "data": "synthetic (BASELINE generator, seeded), fresh Q per step",
            "config": headline_config(args),
            "p50_us": float(np.percentile(per, 50)), "p99_us": float(np.percentile(per, 99)),
            "tokens_per_s": 1e6 / value,
            "roofline": roof, "kernel_us": prof, "phase_us": phases, "algorithmic_bytes_per_step": traffic,
            "l2_window": {"resident_bytes": window_bytes,
                          "what": "upper+lower centroid planes of the layer held in persisting L2 by an "
                                  "access-policy window (the flush evicts normal lines only)",
                          "without_window": no_window},
            "l2_warm": l2_warm,
            "lead_cluster": {"on": bool(eng.fused),
                             "what": "one extra 16-CTA cluster per fused launch decodes a small synthetic cell "
                                     "ahead of the real cells, so the kernel's instructions are in L2 when they "
                                     "reach them (the flush evicts them before every step)",
                             "without_lead": no_lead},
            "live_counts": {"survivors_max": st.survivors_max, "pool_min": st.pool_min, "pool_max": st.pool_max,
                            "union15_max": st.union15_max, "union16_max": st.union16_max},
            "parity": parity, "cpu_baseline": cpu_line, "e2e": e2e, "clocks": clk,
            "gpu_launches": eng.kernels_per_step() * args.steps,
        }
        print(json.dumps(line), flush=True)
    attn.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
