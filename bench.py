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
from types import SimpleNamespace

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


# Work a CPU step may hold: sum over the sample's rows of attended tokens x query
# heads x query tokens.  Config 3's whole batch is 18.8 M (about 0.23 s on 16
# threads of the port); larger workloads take an evenly spread row sample.
CPU_STEP_WORK = 20_000_000


def _cpu_sample_rows(lens_attended: torch.Tensor, heads: int, q_len: int) -> list[int]:
    """The whole batch when its work fits one CPU step, else every k-th row of
    the batch sorted by length (so the sample's mean length tracks the batch's)."""
    work = float(lens_attended.sum()) * heads * q_len
    k = max(1, math.ceil(work / CPU_STEP_WORK))
    order = torch.argsort(lens_attended, stable=True).tolist()
    return sorted(order[k // 2::k]) if k > 1 else list(range(len(order)))


def _compact(w, rows):
    """CPU copies of what ``rows`` of workload ``w`` read: query and new rows,
    their blocks gathered into a small pool, tables renumbered into it."""
    from oracle import oracle

    q_len, bs = w.q_len, w.key_cache.shape[2]
    rows_t = torch.tensor(rows, device=w.block_tables.device)
    lens = w.context_lens[rows_t].to(torch.int64).cpu() + q_len
    nblk = (lens + bs - 1) // bs
    tables = torch.zeros(len(rows), int(nblk.max()), dtype=torch.int32)
    ids, c = [], 0
    for i in range(len(rows)):
        n = int(nblk[i])
        ids.append(w.block_tables[rows_t[i], :n].to(torch.int64))
        tables[i, :n] = torch.arange(c, c + n, dtype=torch.int32)
        c += n
    ids = torch.cat(ids)
    cl = w.context_lens[rows_t].cpu()
    return SimpleNamespace(
        query=w.query[rows_t].cpu(), key_cache=w.key_cache[ids].cpu(), value_cache=w.value_cache[ids].cpu(),
        new_key=w.new_key[rows_t].cpu(), new_value=w.new_value[rows_t].cpu(), tables=tables, context_lens=cl,
        slots=oracle.slot_mapping_from_tables(tables, cl.to(torch.int64), q_len, bs), attended=lens,
        scale=w.scale, q_len=q_len)


def _port_step_fn(c, threads):
    """One CPU step of the C restatement of the reference's decode (oracle/,
    OpenMP over rows) with the append restatement, on compact inputs ``c``."""
    from oracle import oracle

    kc, vc = c.key_cache.clone(), c.value_cache.clone()

    def step():
        oracle.kv_append(c.new_key, c.new_value, kc, vc, c.slots)
        oracle.paged_decode(c.query, kc, vc, c.tables, c.context_lens, c.scale, num_threads=threads)

    return step


def _reference_own_cpu(c, threads, seconds: float = 5.0) -> dict | None:
    """The reference's own CPU code, unmodified, from its checkout or the copy in
    baseline/_ref: GpuKVBlockPool.write_tokens_batch on a CPU pool
    (paged_kv_kernel.py:176-227) and the per-row _paged_attention_decode_torch
    (paged_attention_triton.py:663-704), torch on ``threads`` host threads.
    Times a few rows of ``c``; None when the reference is not importable or the
    step has more than one query token (that function takes q_len = 1 only)."""
    root = None
    for cand in (os.environ.get("LLM_SERVING_RUNTIME_ROOT"), str(REPO / "baseline" / "_ref")):
        if cand and (Path(cand) / "runtime" / "phase2" / "paged_attention_triton.py").exists():
            root = cand
            break
    if root is None or c.q_len != 1:
        return None
    sys.path.insert(0, root)
    try:
        import runtime.phase2.paged_attention_triton as pat
        import runtime.phase2.paged_kv_kernel as pkk
    except ImportError:
        return None
    finally:
        sys.path.remove(root)
    torch.set_num_threads(threads)
    nb, Hkv, bs, D = c.key_cache.shape
    Hq = c.query.shape[1]
    n = min(8, c.query.shape[0])
    order = torch.argsort(c.attended, stable=True)
    sel = sorted(order[torch.linspace(0, c.query.shape[0] - 1, n).round().long().unique()].tolist())
    pool = pkk.GpuKVBlockPool(num_blocks=nb, block_size_tokens=bs, num_layers=1, num_kv_heads=Hkv, head_dim=D,
                              dtype=c.key_cache.dtype, device="cpu")
    pool._grow_pools(nb)
    pool._k_pool[:, 0].copy_(c.key_cache)
    pool._v_pool[:, 0].copy_(c.value_cache)
    tables, cl = c.tables[sel], c.context_lens[sel]

    def step():
        pool.write_tokens_batch(0, tables, cl.to(torch.int64), c.new_key[sel], c.new_value[sel])
        kl, vl = pool.k_layer_view(0), pool.v_layer_view(0)
        for i, b in enumerate(sel):
            L = int(cl[i]) + 1
            nlog = math.ceil(L / bs)
            pat._paged_attention_decode_torch(c.query[b:b + 1], kl, vl, tables[i, :nlog], L, c.scale, Hq // Hkv)

    step()
    reps, t_tot = 0, 0.0
    while t_tot < seconds and reps < 100:
        t0 = time.perf_counter()
        step()
        t_tot += time.perf_counter() - t0
        reps += 1
    dt = t_tot / reps
    return {"value": len(sel) / dt, "unit": UNIT, "cores": threads, "kind": "reference",
            "ms_per_step": dt * 1e3,
            "sample": f"{len(sel)} sequences spread over the length-sorted sample (mean attended length "
                      f"{float(c.attended[sel].float().mean()):.0f}), the reference's write_tokens_batch on a "
                      f"CPU pool + _paged_attention_decode_torch per row, {reps} reps, torch threads={threads}"}


def _dtype_name(dt) -> str:
    return {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}[dt]


def _config_dict(args, spec, world, shard, GB, pg_desc="off") -> dict:
    """The config keys both arms print (the driver compares them)."""
    return {
        "workload": args.workload, "global_batch": GB, "q_len": spec.q_len, "num_q_heads": spec.num_q_heads,
        "num_kv_heads": spec.num_kv_heads, "head_dim": spec.head_dim, "block_size": spec.block_size,
        "context_lens": f"{spec.length_dist} [{spec.length_lo}, {spec.length_hi}]",
        "parallelism": ((f"kvhead-shard{world}+fused-gather" if args.gather == "fused"
                         else f"kvhead-shard{world}+allgather") if shard == "head" else f"seq-shard{world}")
        if world > 1 else "single",
        "l2": "inputs larger than L2 (no flush)",
        "launch": "cuda-graph replay" if args.graph else "eager",
        "prefix_sharing": pg_desc,
    }


def run_reference(args) -> None:
    """CPU arm: the reference's decode algorithm on this box's host cores.

    Each step runs the C restatement of the reference's CPU decode
    (oracle/pa_oracle.c, OpenMP over rows, every host thread) and the append
    restatement over one batch of the workload: the whole one-GPU batch when it
    fits CPU_STEP_WORK (configs 1-3), else an evenly spread row sample.  value
    is that step's sequences / its measured time: a rate of this one host, the
    same at every N (the host does not grow with the GPU count).  Beside it,
    the reference's own torch code on a few rows (kind "reference")."""
    world, rank, _ = _dist_setup()
    if rank != 0:
        return
    from llm_serving_runtime_b200.workloads import SPECS, make_workload, sample_lengths

    spec = SPECS[args.workload]
    if args.batch:
        spec = dataclasses.replace(spec, batch=args.batch)
    shard = _shard_mode(args, world)
    GB = spec.batch if shard == "head" else spec.batch * world
    lens = sample_lengths(spec, spec.batch) + spec.q_len
    rows = _cpu_sample_rows(lens, spec.num_q_heads, spec.q_len)
    w = make_workload(spec, device="cpu", rows=rows, global_batch=spec.batch)
    c = _compact(w, list(range(len(rows))))
    threads = os.cpu_count() or 1
    step = _port_step_fn(c, threads)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = len(rows) * spec.q_len / dt
    whole = len(rows) == spec.batch
    sample = (f"{'all' if whole else 'an evenly spread sample of'} {len(rows)} of the {spec.batch} sequences of one "
              f"{args.workload} batch per step (mean attended length {float(lens[rows].float().mean()):.0f}, batch "
              f"{float(lens.float().mean()):.0f}), append + decode, C restatement on {threads} threads; the job "
              f"holds {GB} sequences")
    pg_desc = "off"
    if spec.prefix_groups and shard != "head":
        pg_desc = f"cascade over {spec.prefix_groups} shared-prefix groups"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong" if shard == "head" else "weak", "vs_baseline": None, "dtype": _dtype_name(spec.dtype),
        "data": "synthetic (seeded; random block placement)",
        "config": _config_dict(args, spec, world, shard, GB, pg_desc),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    own = _reference_own_cpu(c, threads)
    if own is not None:
        line["reference_own_cpu"] = own
    print(json.dumps(line), flush=True)


def run_multi_token_compare(args) -> None:
    """One multi-token layer step through the reference's own cache layer and
    attention hook (BlockPagedBatchLayer.update, paged_kv_cache.py:121-170;
    block_paged_attention_forward, block_paged_attention.py:24-59) on the
    ``prefill-llama3-8b`` shapes: stock (its per-token append loop, the dense
    gather and eager attention, on the GPU) against integration.install()
    (append kernel, then the multi-query kernels over the paged cache), and the
    stock attention after the installed append (gather + eager alone).  Device
    time per step with CUDA events; one JSON line."""
    from llm_serving_runtime_b200 import integration
    from llm_serving_runtime_b200.workloads import SPECS, attention_flops, make_workload

    root = None
    for cand in (os.environ.get("LLM_SERVING_RUNTIME_ROOT"), str(REPO / "baseline" / "_ref")):
        if cand and (Path(cand) / "runtime" / "phase2" / "paged_kv_cache.py").exists():
            root = cand
            break
    if root is None:
        print(json.dumps({"multi_token_compare": "unavailable: reference runtime not importable"}))
        return
    sys.path.insert(0, root)
    import runtime.phase2.block_paged_attention as bpa
    import runtime.phase2.paged_kv_cache as pkc
    import runtime.phase2.paged_kv_kernel as pkk
    from transformers import LlamaConfig

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec = SPECS["prefill-llama3-8b"]
    w = make_workload(spec, device=dev)
    B, Hq, q, D = w.query.shape
    Hkv, bs = spec.num_kv_heads, spec.block_size
    nb = w.key_cache.shape[0]
    cfg = LlamaConfig(hidden_size=Hq * D, num_hidden_layers=1, num_attention_heads=Hq, num_key_value_heads=Hkv,
                      head_dim=D, intermediate_size=256, vocab_size=256)
    pool = pkk.GpuKVBlockPool(num_blocks=nb, block_size_tokens=bs, num_layers=1, num_kv_heads=Hkv, head_dim=D,
                              dtype=w.query.dtype, device=dev)
    pool._grow_pools(nb)
    pool._k_pool[:, 0].copy_(w.key_cache)
    pool._v_pool[:, 0].copy_(w.value_cache)
    cache = pkc.BlockPagedBatchCache(cfg, pool, block_tables=w.block_tables, seq_lens=w.context_lens,
                                     block_ids_rows=[[] for _ in range(B)])
    layer = cache.layers[0]
    start = w.context_lens.clone()

    class Attn:
        num_key_value_groups = Hq // Hkv
        training = False
        is_causal = True

    def step():
        layer._row_seq_lens = start.clone()
        cache.seq_lens = start.clone()
        k, v = layer.update(w.new_key, w.new_value)
        return bpa.block_paged_attention_forward(Attn(), w.query, k, v, None, w.scale)[0]

    def timed(fn, n):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    n = max(3, min(args.steps, 20))
    stock_ms = timed(step, n)
    integration.install(multi_query=False)  # the append kernel, the reference's gather + eager attention
    append_only_ms = timed(step, n)
    integration.uninstall()
    integration.install()
    installed_ms = timed(step, n)
    integration.uninstall()
    print(json.dumps({
        "multi_token_compare": spec.name, "batch": B, "q_len": q, "num_q_heads": Hq, "num_kv_heads": Hkv,
        "head_dim": D, "context_lens": f"{spec.length_dist} [{spec.length_lo}, {spec.length_hi}]",
        "steps": n, "ms_stock_reference": stock_ms, "ms_installed_append_stock_attention": append_only_ms,
        "ms_installed": installed_ms, "speedup_vs_stock": stock_ms / installed_ms,
        "speedup_vs_gather_eager": append_only_ms / installed_ms,
        "attention_tflops_installed": attention_flops(w) / (installed_ms / 1e3) / 1e12,
        "note": "the stock eager hook receives no mask (None) from this call, so it attends every gathered "
                "position; the installed path attends causally over the new tokens",
    }), flush=True)


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
    ap.add_argument("--multi-token-compare", action="store_true",
                    help="time a prefill layer step through the reference's cache and hook, stock vs installed")
    ap.add_argument("--no-kvhead-record", action="store_true",
                    help="skip the config-5 KV-head-sharding record added to every other workload's line")
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
    if args.multi_token_compare:
        run_multi_token_compare(args)
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
    gathered_out = torch.empty((B, spec.num_q_heads, q, spec.head_dim), dtype=w.query.dtype, device=dev) \
        if gather is not None else None
    # Shared prompt prefixes (config 4): one group description per batch
    # composition, passed with every call (paged_attention_decode(prefix_groups=)).
    pg = None
    if args.prefix_sharing != "off" and gather is None:
        pg = w.shared_prefixes()
    if args.prefix_sharing == "on" and pg is None:
        raise SystemExit("--prefix-sharing on needs a workload with shared prefixes on the sequence-sharded path")
    graph = None
    if args.graph:
        # eager calls first: the per-SM shares learn from them, and the graph
        # then keeps the shares it was captured with
        from llm_serving_runtime_b200.paged_attention import SmSpeeds

        for _ in range(2 * SmSpeeds.SAMPLES):
            paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                                   out=out, prefix_groups=pg)
            torch.cuda.synchronize()
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
                          w.slot_mapping, w.new_key, w.new_value, out=gathered_out)
        return paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens,
                                      w.scale, w.slot_mapping, w.new_key, w.new_value, out=out, prefix_groups=pg)

    def barrier():
        if world > 1:
            dist.barrier()

    # Untimed: the per-SM shares learn from the first large calls (each call's
    # timing records come back before the next one); a fixed number of calls,
    # so every rank makes the same calls.
    from llm_serving_runtime_b200.paged_attention import SmSpeeds

    share_calls = 0 if graph is not None else 2 * SmSpeeds.SAMPLES
    for _ in range(share_calls):
        step()
        torch.cuda.synchronize()
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
    # output inside the timed region (under KV-head sharding only rank 0
    # downloads the gathered output: one copy of the result per job).
    names = ("query", "new_key", "new_value", "slot_mapping", "context_lens", "block_tables")
    pg_names = ("member_offsets", "member_seqs", "prefix_lens", "seq_group") if pg is not None else ()
    inputs = {k: getattr(w, k) for k in names}
    inputs.update({k: getattr(pg, k) for k in pg_names})
    full_out_shape = (B, spec.num_q_heads, q, spec.head_dim) if shard == "head" else tuple(out.shape)

    def e2e_call(d, o):
        args_ = (d["query"], w.key_cache, w.value_cache, d["block_tables"], d["context_lens"], w.scale,
                 d["slot_mapping"], d["new_key"], d["new_value"])
        if gather is not None:
            return gather(*args_, out=o)
        pg_ = dataclasses.replace(pg, **{k: d[k] for k in pg_names}) if pg is not None else None
        return paged_attention_decode(*args_, out=o, prefix_groups=pg_)

    n_e2e = max(10, min(args.steps, 100))
    download = shard != "head" or rank == 0
    e2e_ms, h2d, d2h, last_host = _e2e_measure(dev, stream, inputs, e2e_call, full_out_shape, out.dtype,
                                               download, n_e2e, barrier, world)
    e2e_value = tokens_per_step / (e2e_ms / n_e2e / 1e3)
    ok = torch.equal(last_host, (out if gather is None else step()).cpu()) if download else None

    kvhead = None
    if not args.no_kvhead_record and args.workload != "cfg5-llama3-70b":
        del inputs
        kvhead = _kvhead_record(args, world, rank, dev, stream, barrier)

    # ---- CPU baseline (rank 0, one GPU only) ----
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline(w, spec)

    clk = clocks.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    # a cascade call moves other bytes than the plain call on the same workload
    ratio = _traffic_ratio_from_profiles(args.workload + ("+cascade" if pg is not None else ""))
    traffic = None if (ratio is None or tensor_bound) else ratio * dec_bytes
    config = _config_dict(args, spec, world, shard, GB,
                          f"cascade over {pg.num_groups} shared-prefix groups" if pg is not None else "off")
    config["bytes_per_call"] = call_bytes
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
        "dtype": _dtype_name(spec.dtype),
        "data": "synthetic (seeded; random block placement)",
        "config": config,
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
        "sm_shares": dict(_sm_shares_summary(dev), untimed_learning_calls=2 * SmSpeeds.SAMPLES),
        "ms_per_step_by_rank": [round(v, 5) for v in rank_ms],
        "kernel_ms_by_rank": [round(v, 5) for v in dec_ms_by_rank],
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if kvhead is not None:
        line["kvhead_shard"] = kvhead
    print(json.dumps(line), flush=True)


def _sm_shares_summary(dev) -> dict:
    """The per-SM share weights of the large decode calls (paged_attention.SmSpeeds)."""
    from llm_serving_runtime_b200.paged_attention import _SM_SHARES, sm_speeds

    t = sm_speeds(dev)
    w = t.weights[: t.n] if t.n else t.weights
    return {"on": bool(_SM_SHARES and t.n), "samples": t.samples, "learning": t.learning,
            "min": round(float(w.min()), 4), "max": round(float(w.max()), 4)}


def _e2e_measure(dev, stream, inputs: dict, call, out_shape, out_dtype, download: bool, n: int, barrier,
                 world: int):
    """n steps through the public API with host buffers: each step's inputs go
    up from pinned host memory on one copy stream, the call runs on ``stream``,
    and (when ``download``) its output comes back to pinned memory on another.
    Double-buffered, so step i+1's upload and step i-1's download overlap step
    i's kernels.  Returns (device ms for the n steps, max over ranks; bytes up
    per step; bytes down per step; the last downloaded output or None)."""
    import torch.distributed as dist

    host_in = [{k: v.cpu().pin_memory() for k, v in inputs.items()} for _ in range(2)]
    dev_in = [{k: torch.empty_like(v) for k, v in inputs.items()} for _ in range(2)]
    dev_out = [torch.empty(out_shape, dtype=out_dtype, device=dev) for _ in range(2)]
    host_out = [torch.empty(out_shape, dtype=out_dtype, pin_memory=True) for _ in range(2)] if download else None
    h2d = sum(v.numel() * v.element_size() for v in host_in[0].values())
    d2h = host_out[0].numel() * host_out[0].element_size() if download else 0
    up_stream, down_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]    # inputs of the slot uploaded
    ev_done = [torch.cuda.Event() for _ in range(2)]  # the call of the slot finished
    ev_out = [torch.cuda.Event() for _ in range(2)]   # download of the slot finished

    def upload(i):
        s_ = i % 2
        with torch.cuda.stream(up_stream):
            up_stream.wait_event(ev_done[s_])  # call i-2 no longer reads these inputs
            for k in inputs:
                dev_in[s_][k].copy_(host_in[s_][k], non_blocking=True)
            ev_in[s_].record(up_stream)

    def compute(i):
        s_ = i % 2
        stream.wait_event(ev_in[s_])
        stream.wait_event(ev_out[s_])  # download i-2 no longer reads this output
        res = call(dev_in[s_], dev_out[s_])
        ev_done[s_].record(stream)
        return res

    def finish(i, res):
        s_ = i % 2
        with torch.cuda.stream(down_stream):
            down_stream.wait_event(ev_done[s_])
            if download:
                host_out[s_].copy_(res, non_blocking=True)
                res.record_stream(down_stream)
            ev_out[s_].record(down_stream)

    def run(k, e_start=None):
        if e_start is not None:
            up_stream.wait_event(e_start)
        upload(0)
        for i in range(k):
            if i + 1 < k:
                upload(i + 1)
            finish(i, compute(i))
        stream.wait_event(ev_out[(k - 1) % 2])

    run(3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run(n, e0)
    e1.record(stream)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), h2d, d2h, (host_out[(n - 1) % 2] if download else None)


def _timed_ms(fn, steps: int, warmup: int, stream, barrier) -> float:
    """Mean device ms of one ``fn()`` over ``steps`` calls after ``warmup``,
    bracketed by barrier + synchronize (this rank)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    return e0.elapsed_time(e1) / steps


def _gather_floats(x: float, dev, world: int) -> list[float]:
    import torch.distributed as dist

    if world == 1:
        return [x]
    every = torch.empty(world, device=dev, dtype=torch.float64)
    dist.all_gather_into_tensor(every, torch.tensor([x], device=dev, dtype=torch.float64))
    return every.tolist()


def _kvhead_record(args, world: int, rank: int, dev, stream, barrier) -> dict:
    """Config 5 (Llama-3-70B shape) sharded by KV heads over this run's ranks,
    the output all-gathered (fused into the decode kernel over NVLink, and
    through NCCL), timed like the main step; plus the whole config 5 on one GPU
    (rank 0) as the strong-scaling baseline.  Per rank: step time, the decode
    kernel alone on its heads, and that kernel's fraction of the HBM peak.  The
    e2e uploads each rank's inputs and downloads the gathered output on rank 0
    only."""
    from llm_serving_runtime_b200 import paged_attention_decode
    from llm_serving_runtime_b200.sharding import FusedHeadGather, HeadShardedDecode, kv_head_range
    from llm_serving_runtime_b200.workloads import SPECS, algorithmic_bytes, make_workload

    spec = SPECS["cfg5-llama3-70b"]
    peak_hbm = _peaks()[0]
    steps, warmup = args.steps, args.warmup
    rec = {"workload": spec.name, "n_gpus": world, "steps": steps, "warmup": warmup, "scaling": "strong",
           "unit": UNIT, "config": {"global_batch": spec.batch, "num_q_heads": spec.num_q_heads,
                                    "num_kv_heads": spec.num_kv_heads, "head_dim": spec.head_dim,
                                    "context_lens": f"{spec.length_dist} [{spec.length_lo}, {spec.length_hi}]"}}
    B = spec.batch
    t1 = None
    if rank == 0:
        w1 = make_workload(spec, device=dev)
        o1 = torch.empty_like(w1.query)
        t1 = _timed_ms(lambda: paged_attention_decode(w1.query, w1.key_cache, w1.value_cache, w1.block_tables,
                                                      w1.context_lens, w1.scale, w1.slot_mapping, w1.new_key,
                                                      w1.new_value, out=o1), steps, warmup, stream, lambda: None)
        rec["single_gpu"] = {"ms_per_step": t1, "tokens_per_s": B / (t1 / 1e3),
                             "hbm_frac": algorithmic_bytes(w1) / (t1 / 1e3) / 1e9 / peak_hbm}
        del w1, o1
        torch.cuda.empty_cache()
    if world == 1:
        return rec
    barrier()
    w = make_workload(spec, device=dev, kv_heads=kv_head_range(spec.num_kv_heads, world, rank))
    local_out = torch.empty_like(w.query)
    t_dec = _timed_ms(lambda: paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables,
                                                     w.context_lens, w.scale, out=local_out),
                      steps, warmup, stream, barrier)
    dec_bytes = algorithmic_bytes(w, include_append=False)
    dec_by_rank = _gather_floats(t_dec, dev, world)
    rec["decode_kernel_ms_by_rank"] = [round(v, 5) for v in dec_by_rank]
    rec["decode_hbm_frac_by_rank"] = [round(dec_bytes / (v / 1e3) / 1e9 / peak_hbm, 4) for v in dec_by_rank]
    names = ("query", "new_key", "new_value", "slot_mapping", "context_lens", "block_tables")
    inputs = {k: getattr(w, k) for k in names}
    out_shape = (B, spec.num_q_heads, 1, spec.head_dim)
    for mode in ("fused", "nccl"):
        g = FusedHeadGather() if mode == "fused" else HeadShardedDecode()
        gathered = torch.empty(out_shape, dtype=w.query.dtype, device=dev)

        def call(d=None, o=None, g=g, gathered=gathered):
            d = inputs if d is None else d
            return g(d["query"], w.key_cache, w.value_cache, d["block_tables"], d["context_lens"], w.scale,
                     d["slot_mapping"], d["new_key"], d["new_value"], out=gathered if o is None else o)

        t = _timed_ms(call, steps, warmup, stream, barrier)
        by_rank = _gather_floats(t, dev, world)
        t_max = max(by_rank)
        e2e_ms, h2d, d2h, _ = _e2e_measure(dev, stream, inputs, call, out_shape, w.query.dtype, rank == 0,
                                           max(10, min(steps, 100)), barrier, world)
        entry = {"ms_per_step": t_max, "ms_per_step_by_rank": [round(v, 5) for v in by_rank],
                 "tokens_per_s": B / (t_max / 1e3),
                 "e2e": {"value": B / (e2e_ms / max(10, min(steps, 100)) / 1e3), "unit": UNIT,
                         "h2d_bytes_per_step_per_rank": h2d, "d2h_bytes_per_step": d2h,
                         "download": "rank 0 only"}}
        single = _gather_floats(t1 if t1 is not None else 0.0, dev, world)[0]
        if single > 0:
            entry["strong_scaling_eff"] = single / (world * t_max)
            entry["speedup_vs_single_gpu"] = single / t_max
        rec[mode] = entry
        if mode == "fused":
            torch.cuda.synchronize()
            g.close()
    return rec




def _cpu_baseline(w, spec) -> dict:
    """The CPU leg of this arm (rank 0, one GPU): the reference arm's step (the
    C restatement on every host thread, the whole batch or an evenly spread
    row sample) timed for about 10 s on this workload's own rows, and the
    reference's own torch code beside it."""
    rows = _cpu_sample_rows(w.attended_lengths(), spec.num_q_heads, spec.q_len)
    c = _compact(w, rows)
    threads = os.cpu_count() or 1
    step = _port_step_fn(c, threads)
    step()
    reps, t_tot = 0, 0.0
    while t_tot < 10.0 and reps < 200:
        t0 = time.perf_counter()
        step()
        t_tot += time.perf_counter() - t0
        reps += 1
    dt = t_tot / reps
    out = {"value": len(rows) * w.q_len / dt, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": f"{len(rows)} of {w.batch} sequences (mean attended length "
                     f"{float(c.attended.float().mean()):.0f}, batch {float(w.attended_lengths().float().mean()):.0f}),"
                     f" append + decode, {reps} reps of {dt * 1e3:.1f} ms"}
    own = _reference_own_cpu(c, threads)
    if own is not None:
        out["reference_own_cpu"] = own
    return out


if __name__ == "__main__":
    main()
