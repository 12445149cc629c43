"""Benchmark of the paged decode path (KV append + decode attention, one layer).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload NAME]

A step is one call of the north-star op on one batch: append the step's new
K/V rows through slot_mapping, then paged decode attention over every
sequence.  Default workload: BASELINE config 3 (Llama-3-8B shape, bf16,
B=256, 32/8 heads, D=128, log-uniform context 256..8192) — the configuration
the north-star target is quoted on.  Inputs are larger than L2 (~2.4 GB of KV
per call), so no flush is needed between steps.

Multi-GPU (torchrun, one process per GPU): sequences shard across ranks with
no collective on the data path (greedy longest-first balancing of attended
lengths); every rank holds 256 sequences' worth of work, so scaling is weak.
Timing is on the device with CUDA events, bracketed by barrier + synchronize,
max over ranks.

Rank 0 prints one JSON line.  ``--impl reference`` times the reference's CPU
algorithm (the C restatement in oracle/, all host threads) on a bounded row
sample of the same workload instead.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "decode-attn tokens/s and achieved HBM GB/s (% peak) at 1/2/4/8 B200"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


FALLBACK_BF16_TFLOPS = 1590.0


def _peaks() -> tuple[float, float, str]:
    """(HBM GB/s, dense bf16 TFLOP/s burst, source) from MEASURED_PEAKS.json."""
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during timing."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        self.lines: list[str] = []
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            ident = str(device_index)
        self.cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-lms", "200", "-i", ident]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for name, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _traffic_ratio_from_profiles(workload: str) -> float | None:
    """DRAM bytes / algorithmic bytes of the decode launch from an ncu capture
    (profiles/*.md, line 'dram_traffic_ratio[<workload>]: <ratio>'), or None."""
    for p in sorted((REPO / "profiles").glob("*.md")):
        for line in p.read_text().splitlines():
            key = f"dram_traffic_ratio[{workload}]:"
            if line.strip().startswith(key):
                try:
                    return float(line.split(":", 1)[1].strip().split()[0])
                except ValueError:
                    return None
    return None


def run_reference(args) -> None:
    """CPU arm: the reference's CPU decode algorithm (oracle/pa_oracle.c, OpenMP
    over rows, all host threads) + the append restatement, on a bounded sample."""
    world, rank, _ = _dist_setup()
    if rank != 0:
        return
    from llm_serving_runtime_b200.workloads import SPECS, make_workload, sample_lengths
    from oracle import oracle

    spec = SPECS[args.workload]
    if args.batch:
        spec = dataclasses.replace(spec, batch=args.batch)
    # The job our arm runs at this N: the one-GPU workload on every rank
    # (sequence sharding), or the one workload split by KV heads.
    copies = 1 if _shard_mode(args, world) == "head" else world
    GB = spec.batch * copies
    lens_one = sample_lengths(spec, spec.batch)
    g = torch.Generator().manual_seed(4242)
    n_sample = min(args.cpu_rows, spec.batch)
    rows = sorted(torch.randperm(spec.batch, generator=g)[:n_sample].tolist())
    w = make_workload(spec, device="cpu", rows=rows, global_batch=spec.batch)
    threads = os.cpu_count() or 1
    kc, vc = w.key_cache.clone(), w.value_cache.clone()

    def step():
        oracle.kv_append(w.new_key, w.new_value, kc, vc, w.slot_mapping)
        oracle.paged_decode(w.query, kc, vc, w.block_tables, w.context_lens, w.scale, num_threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    # scale the sample's time to the whole job by attended tokens
    L_all = copies * float((lens_one + spec.q_len).sum())
    L_smp = float((lens_one[rows] + spec.q_len).sum())
    t_full = dt * L_all / L_smp
    value = GB * spec.q_len / t_full
    sample = (f"{n_sample} of {GB} sequences of {args.workload} (seeded), append + decode per step; "
              f"time scaled to the full batch by attended tokens ({L_smp:.0f} of {L_all:.0f})")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_full * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16",
                                                          torch.float32: "fp32"}[spec.dtype],
        "data": "synthetic (seeded)",
        "config": {"workload": args.workload, "global_batch": GB, "q_len": spec.q_len,
                   "num_q_heads": spec.num_q_heads, "num_kv_heads": spec.num_kv_heads,
                   "head_dim": spec.head_dim, "block_size": spec.block_size},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _shard_mode(args, world: int) -> str:
    """Multi-GPU layout: KV heads for config 5 at N > 1 (auto), sequences otherwise."""
    if args.shard != "auto":
        return args.shard
    return "head" if (world > 1 and args.workload == "cfg5-llama3-70b") else "seq"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default="cfg3-llama3-8b")
    ap.add_argument("--cpu-rows", type=int, default=16, help="rows in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the workload's per-GPU batch (smaller cases for ncu captures)")
    ap.add_argument("--graph", action="store_true",
                    help="time replays of a CUDA graph holding the step (append + decode) instead of eager calls")
    ap.add_argument("--prefix-sharing", choices=["auto", "on", "off"], default="auto",
                    help="cascade over shared prompt prefixes (auto: when the workload has them)")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="KV-head sharding: all-gather inside the decode kernel over NVLink, or NCCL after it")
    ap.add_argument("--shard", choices=["auto", "seq", "head"], default="auto",
                    help="multi-GPU layout: sequences (weak scaling) or KV heads + NCCL all-gather "
                         "(strong scaling); auto = heads for cfg5-llama3-70b, sequences otherwise")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    if args.impl == "reference":
        run_reference(args)
        return

    import torch.distributed as dist

    from llm_serving_runtime_b200 import _lib, paged_attention_decode
    from llm_serving_runtime_b200.sharding import FusedHeadGather, HeadShardedDecode, kv_head_range
    from llm_serving_runtime_b200.workloads import SPECS, algorithmic_bytes, attention_flops, make_workload

    world, rank, local = _dist_setup()
    if world != args.gpus:
        args.gpus = world
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)

    spec = SPECS[args.workload]
    if args.batch:
        spec = dataclasses.replace(spec, batch=args.batch)
    shard = _shard_mode(args, world)
    if shard == "head":
        # every rank holds its KV heads of the whole batch; outputs all-gathered
        GB = spec.batch
        w = make_workload(spec, device=dev, kv_heads=kv_head_range(spec.num_kv_heads, world, rank))
        gather = FusedHeadGather() if args.gather == "fused" else HeadShardedDecode()
    else:
        # Weak scaling with the per-GPU work fixed: every rank holds the one-GPU
        # workload itself (its lengths and prefix groups) with its own block
        # placement and data.
        GB = spec.batch * world
        w = make_workload(spec, device=dev, seed_offset=rank)
        gather = None
    B, q = w.batch, w.q_len
    out = torch.empty_like(w.query)
    # Shared prompt prefixes (config 4): one group description per batch
    # composition, passed with every call (paged_attention_decode(prefix_groups=)).
    pg = None
    if args.prefix_sharing != "off" and gather is None:
        pg = w.shared_prefixes()
    if args.prefix_sharing == "on" and pg is None:
        raise SystemExit("--prefix-sharing on needs a workload with shared prefixes on the sequence-sharded path")
    graph = None
    if args.graph:
        if gather is not None:
            raise SystemExit("--graph covers the single-rank and sequence-sharded steps")
        from llm_serving_runtime_b200.cuda_graph import DecodeStepGraph

        graph = DecodeStepGraph([w.key_cache], [w.value_cache], batch=B, max_blocks=w.block_tables.shape[1],
                                num_q_heads=w.query.shape[1], q_len=q, scale=w.scale, prefix_groups=pg)
        graph.query[0].copy_(w.query)
        graph.new_key[0].copy_(w.new_key)
        graph.new_value[0].copy_(w.new_value)
        graph.block_tables.copy_(w.block_tables)
        graph.context_lens.copy_(w.context_lens)
        graph.slot_mapping.copy_(w.slot_mapping)

    def step():
        if graph is not None:
            return graph.replay()[0]
        if isinstance(gather, FusedHeadGather):  # returns this rank's gathered output
            return gather(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                          w.slot_mapping, w.new_key, w.new_value)
        if gather is not None:
            return gather(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                          w.slot_mapping, w.new_key, w.new_value, out=out)
        return paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens,
                                      w.scale, w.slot_mapping, w.new_key, w.new_value, out=out, prefix_groups=pg)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps of append + decode ----
    stream = torch.cuda.current_stream(dev)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
    local_ms = ev0.elapsed_time(ev1)
    t = torch.tensor([local_ms], device=dev, dtype=torch.float64)
    rank_ms = [local_ms / args.steps]
    if world > 1:
        every = torch.empty(world, device=dev, dtype=torch.float64)
        dist.all_gather_into_tensor(every, t)
        rank_ms = [v / args.steps for v in every.tolist()]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    tokens_all = torch.tensor([B * q], device=dev, dtype=torch.float64)
    if world > 1 and shard == "seq":
        dist.all_reduce(tokens_all)
    tokens_per_step = float(tokens_all.item())
    value = tokens_per_step / (ms_per_step / 1e3)
    gpu_launches = 2 * args.steps  # pa_kv_append + pa_decode per step (+ one NCCL all-gather in head mode)

    # ---- decode kernel alone, for the roofline (events around each launch) ----
    n_dec = max(20, min(args.steps, 100))
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_dec)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_dec)]
    barrier()
    torch.cuda.synchronize()
    for i in range(n_dec):
        starts[i].record(stream)
        paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                               out=out, prefix_groups=pg)
        ends[i].record(stream)
    torch.cuda.synchronize()
    dec_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    dec_ms_by_rank = [dec_ms]
    if world > 1:
        every = torch.empty(world, device=dev, dtype=torch.float64)
        dist.all_gather_into_tensor(every, torch.tensor([dec_ms], device=dev, dtype=torch.float64))
        dec_ms_by_rank = every.tolist()
    dec_kernel = _lib.last_kernel()
    # A block shared by several sequences (config 4's prefixes) is counted once:
    # the minimum bytes the call must move.  The per-sequence (logical) figure
    # is reported beside it.
    dec_bytes = algorithmic_bytes(w, include_append=False, unique=True)
    dec_bytes_logical = algorithmic_bytes(w, include_append=False)
    call_bytes = algorithmic_bytes(w, include_append=True, unique=True)
    dec_flops = attention_flops(w)
    peak_hbm, peak_tensor, peak_src = _peaks()
    # the bound is whichever resource needs more time at its peak
    tensor_bound = dec_flops / (peak_tensor * 1e12) > dec_bytes / (peak_hbm * 1e9)
    if tensor_bound:
        achieved, peak, bound, r_unit = dec_flops / (dec_ms / 1e3) / 1e12, peak_tensor, "tensor", "TFLOP/s"
    else:
        achieved, peak, bound, r_unit = dec_bytes / (dec_ms / 1e3) / 1e9, peak_hbm, "hbm", "GB/s"

    # ---- end to end through the public API with host buffers ----
    # Every step uploads its own inputs from pinned host memory and downloads its
    # output inside the timed region.  Uploads and downloads run on two copy
    # streams with double-buffered device inputs/outputs, so step i+1's upload
    # and step i-1's download overlap step i's decode (how a serving loop hides
    # the PCIe transfers).
    names = ("query", "new_key", "new_value", "slot_mapping", "context_lens", "block_tables")
    pg_names = ("member_offsets", "member_seqs", "prefix_lens", "seq_group") if pg is not None else ()

    def _src(k):
        return getattr(pg, k) if k in pg_names else getattr(w, k)

    host_in = [{k: _src(k).cpu().pin_memory() for k in names + pg_names} for _ in range(2)]
    dev_in = [{k: torch.empty_like(_src(k)) for k in names + pg_names} for _ in range(2)]
    full_out_shape = (B, spec.num_q_heads, q, spec.head_dim) if shard == "head" else tuple(out.shape)
    fused = isinstance(gather, FusedHeadGather)
    dev_out = [torch.empty(full_out_shape, dtype=out.dtype, device=dev) if fused else torch.empty_like(out)
               for _ in range(2)]
    host_out = [torch.empty(full_out_shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in host_in[0].values())
    d2h = host_out[0].numel() * host_out[0].element_size()
    n_e2e = max(10, min(args.steps, 100))
    up_stream, down_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of the slot uploaded
    ev_done = [torch.cuda.Event() for _ in range(2)]  # decode of the slot finished
    ev_out = [torch.cuda.Event() for _ in range(2)]   # download of the slot finished

    def upload(i):
        s_ = i % 2
        with torch.cuda.stream(up_stream):
            up_stream.wait_event(ev_done[s_])  # decode i-2 no longer reads these inputs
            for k in names + pg_names:
                dev_in[s_][k].copy_(host_in[s_][k], non_blocking=True)
            ev_in[s_].record(up_stream)

    def compute(i):
        s_ = i % 2
        stream.wait_event(ev_in[s_])
        stream.wait_event(ev_out[s_])  # download i-2 no longer reads this output
        d = dev_in[s_]
        args_ = (d["query"], w.key_cache, w.value_cache, d["block_tables"], d["context_lens"], w.scale,
                 d["slot_mapping"], d["new_key"], d["new_value"])
        pg_ = dataclasses.replace(pg, **{k: d[k] for k in pg_names}) if pg is not None else None
        res = gather(*args_, out=dev_out[s_]) if gather is not None else \
            paged_attention_decode(*args_, out=dev_out[s_], prefix_groups=pg_)
        ev_done[s_].record(stream)
        return res

    def download(i, res):
        s_ = i % 2
        with torch.cuda.stream(down_stream):
            down_stream.wait_event(ev_done[s_])
            host_out[s_].copy_(res, non_blocking=True)
            res.record_stream(down_stream)
            ev_out[s_].record(down_stream)

    def e2e_run(n, e_start=None):
        if e_start is not None:
            up_stream.wait_event(e_start)
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            download(i, compute(i))
        stream.wait_event(ev_out[(n - 1) % 2])

    e2e_run(3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(n_e2e, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_value = tokens_per_step / (float(t.item()) / n_e2e / 1e3)
    ok = torch.equal(host_out[(n_e2e - 1) % 2], (out if gather is None else step()).cpu())

    # ---- CPU baseline (rank 0, one GPU only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline(w, spec, args.cpu_rows)

    clk = clocks.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    # a cascade call moves other bytes than the plain call on the same workload
    ratio = _traffic_ratio_from_profiles(args.workload + ("+cascade" if pg is not None else ""))
    traffic = None if (ratio is None or tensor_bound) else ratio * dec_bytes
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong" if shard == "head" else "weak",
        "vs_baseline": None,
        "dtype": {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[spec.dtype],
        "data": "synthetic (seeded; random block placement)",
        "config": {
            "workload": args.workload, "global_batch": GB, "q_len": q, "num_q_heads": spec.num_q_heads,
            "num_kv_heads": spec.num_kv_heads, "head_dim": spec.head_dim, "block_size": spec.block_size,
            "context_lens": f"{spec.length_dist} [{spec.length_lo}, {spec.length_hi}]",
            "parallelism": ((f"kvhead-shard{world}+fused-gather" if args.gather == "fused"
                             else f"kvhead-shard{world}+allgather") if shard == "head" else f"seq-shard{world}")
            if world > 1 else "single",
            "l2": "inputs larger than L2 (no flush)",
            "launch": "cuda-graph replay" if args.graph else "eager",
            "prefix_sharing": (f"cascade over {pg.num_groups} shared-prefix groups" if pg is not None else "off"),
            "bytes_per_call": call_bytes,
        },
        "hbm_gbs_per_call": call_bytes / (ms_per_step / 1e3) / 1e9,
        "roofline": {
            "bound": bound, "achieved": achieved, "peak": peak, "unit": r_unit, "frac": achieved / peak,
            "traffic": traffic, "peak_source": peak_src, "kernel": dec_kernel,
            "kernel_ms": dec_ms, "algorithmic_bytes": dec_bytes, "algorithmic_bytes_logical": dec_bytes_logical,
            "flops": dec_flops,
            "hbm_gbs": dec_bytes / (dec_ms / 1e3) / 1e9, "tflops": dec_flops / (dec_ms / 1e3) / 1e12,
        },
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "overlap": "2 copy streams, double-buffered", "result_matches_device_run": ok},
        "gpu_launches": gpu_launches,
        "ms_per_step_by_rank": [round(v, 5) for v in rank_ms],
        "kernel_ms_by_rank": [round(v, 5) for v in dec_ms_by_rank],
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def _cpu_baseline(w, spec, n_rows: int) -> dict:
    """The oracle (C restatement of the reference's CPU decode, all host threads)
    on a seeded row sample of the bench workload, scaled to the full batch."""
    from oracle import oracle

    g = torch.Generator().manual_seed(4242)
    B = w.batch
    rows = sorted(torch.randperm(B, generator=g)[:min(n_rows, B)].tolist())
    q_len = w.q_len
    bs = w.key_cache.shape[2]
    rows_t = torch.tensor(rows, device=w.block_tables.device)
    lens = w.context_lens[rows_t].to(torch.int64) + q_len
    nblk = (lens + bs - 1) // bs
    maxb = int(nblk.max())
    ids, tables, c = [], torch.zeros(len(rows), maxb, dtype=torch.int32), 0
    for i in range(len(rows)):
        n = int(nblk[i])
        ids.append(w.block_tables[rows_t[i], :n].to(torch.int64))
        tables[i, :n] = torch.arange(c, c + n, dtype=torch.int32)
        c += n
    ids = torch.cat(ids)
    kc, vc = w.key_cache[ids].cpu(), w.value_cache[ids].cpu()
    qq, cl = w.query[rows_t].cpu(), w.context_lens[rows_t].cpu()
    nk, nv = w.new_key[rows_t].cpu(), w.new_value[rows_t].cpu()
    slots = oracle.slot_mapping_from_tables(tables, cl.to(torch.int64), q_len, bs)
    threads = os.cpu_count() or 1
    reps, t_tot = 0, 0.0
    while t_tot < 5.0 and reps < 50:
        t0 = time.perf_counter()
        oracle.kv_append(nk, nv, kc, vc, slots)
        oracle.paged_decode(qq, kc, vc, tables, cl, w.scale, num_threads=threads)
        t_tot += time.perf_counter() - t0
        reps += 1
    dt = t_tot / reps
    L_all = float(w.attended_lengths().sum())
    L_smp = float(lens.sum())
    value = B * q_len / (dt * L_all / L_smp)
    return {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(rows)} of {B} sequences (seeded), append + decode, {reps} reps; "
                      f"scaled to the full batch by attended tokens ({L_smp:.0f} of {L_all:.0f})"}


if __name__ == "__main__":
    main()
