"""Multi-rank host logic on CPU (gloo, world size 2).

The sharded layouts of ``llm_serving_runtime_b200.sharding`` are checked end to
end with the CPU oracle as the per-rank decode (the sm_100a kernels need a
GPU): sequence sharding reassembles to the single-rank result, KV-head sharding
all-gathers to it, and a rank that leaves before the collective makes the other
rank's collective fail with an error instead of hanging.
"""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llm_serving_runtime_b200.sharding import HeadShardedDecode, kv_head_range, shard_sequences
from llm_serving_runtime_b200.workloads import WorkloadSpec, make_workload

SPEC = WorkloadSpec("gloo-small", 6, 8, 4, 64, 16, torch.float16, 2, "uniform", 3, 90, 0.5, seed=77)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_decode(query, key_cache, value_cache, block_tables, context_lens, scale, slot_mapping=None,
                   key=None, value=None, **kw):
    from oracle import oracle

    if key is not None:
        oracle.kv_append(key, value, key_cache, value_cache, slot_mapping)
    return oracle.paged_decode(query, key_cache, value_cache, block_tables, context_lens, scale).to(query.dtype)


def _rows_of(w, rows):
    """The sub-batch ``rows`` of workload ``w`` over the same pool."""
    r = torch.tensor(rows)
    q_len = w.q_len
    slots = w.slot_mapping.reshape(-1, q_len)[r].reshape(-1)
    return (w.query[r], w.block_tables[r], w.context_lens[r], w.new_key[r], w.new_value[r], slots)


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))


def _seq_worker(rank, world, port, out_q):
    _init(rank, world, port, 60)
    w = make_workload(SPEC, device="cpu")
    shards = shard_sequences((w.context_lens + w.q_len).tolist(), world)
    q, bt, cl, nk, nv, slots = _rows_of(w, shards[rank])
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    local = _oracle_decode(q, kc, vc, bt, cl, w.scale, slots, nk, nv)
    gathered = [None] * world
    dist.all_gather_object(gathered, (shards[rank], local))
    if rank == 0:
        out = torch.empty_like(w.query)
        for rows, part in gathered:
            out[torch.tensor(rows)] = part
        out_q.put(out.float().numpy())  # by value: the worker exits right after
    dist.destroy_process_group()


def _head_worker(rank, world, port, out_q):
    _init(rank, world, port, 60)
    w = make_workload(SPEC, device="cpu")
    h0, hc = kv_head_range(SPEC.num_kv_heads, world, rank)
    G = SPEC.num_q_heads // SPEC.num_kv_heads
    kc = w.key_cache[:, h0:h0 + hc].clone()
    vc = w.value_cache[:, h0:h0 + hc].clone()
    q = w.query[:, h0 * G:(h0 + hc) * G].contiguous()
    args = (q, kc, vc, w.block_tables, w.context_lens, w.scale, w.slot_mapping,
            w.new_key[:, h0:h0 + hc].contiguous(), w.new_value[:, h0:h0 + hc].contiguous())
    out = HeadShardedDecode(decode_fn=_oracle_decode)(*args)
    # out= receives the gathered [B, Hq, q, D] result, as the fused form does
    dest = torch.empty_like(out)
    kc.copy_(w.key_cache[:, h0:h0 + hc])
    vc.copy_(w.value_cache[:, h0:h0 + hc])
    assert HeadShardedDecode(decode_fn=_oracle_decode)(*args, out=dest) is dest and torch.equal(dest, out)
    if rank == 0:
        out_q.put(out.float().numpy())  # by value: the worker exits right after
    dist.destroy_process_group()


def _leaving_worker(rank, world, port, out_q):
    _init(rank, world, port, 5)
    if rank == 1:
        # leaves between steps, before the collective, without taking part
        dist.destroy_process_group()
        return
    w = make_workload(SPEC, device="cpu")
    try:
        HeadShardedDecode(decode_fn=_oracle_decode)(w.query, w.key_cache, w.value_cache, w.block_tables,
                                                    w.context_lens, w.scale)
        out_q.put("no error")
    except Exception as e:  # gloo reports the missing peer or the timeout
        out_q.put(type(e).__name__)


def _guarded(fn, rank, world, port, out_q):
    try:
        fn(rank, world, port, out_q)
    except Exception as e:  # surface worker failures at once instead of a queue timeout
        out_q.put(f"worker {rank} failed: {type(e).__name__}: {e}")
        raise


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_guarded, args=(fn, r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    result = q.get(timeout=120)
    if hasattr(result, "dtype"):
        result = torch.from_numpy(result)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return result


def _reference():
    w = make_workload(SPEC, device="cpu")
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    return _oracle_decode(w.query, kc, vc, w.block_tables, w.context_lens, w.scale, w.slot_mapping,
                          w.new_key, w.new_value)


def test_sequence_sharding_reassembles_the_batch():
    out = _run(_seq_worker)
    assert isinstance(out, torch.Tensor), out
    assert torch.equal(out, _reference().float())


def test_kv_head_sharding_all_gathers_the_heads():
    out = _run(_head_worker)
    assert isinstance(out, torch.Tensor), out
    assert torch.equal(out, _reference().float())


def test_rank_leaving_before_the_collective_is_an_error_not_a_hang():
    assert _run(_leaving_worker) != "no error"


def test_shard_sequences_balances_and_keeps_groups():
    lens = [8192, 256, 300, 4000, 4100, 512, 700, 9000]
    shards = shard_sequences(lens, 2)
    assert sorted(shards[0] + shards[1]) == list(range(8))
    loads = [sum(lens[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(lens)
    grouped = shard_sequences(list(range(1, 17)), 2, group_size=4)
    for s in grouped:
        assert all((i // 4) * 4 + k in s for i in s for k in range(4))


def test_kv_head_range():
    assert [kv_head_range(8, 8, r) for r in range(8)] == [(r, 1) for r in range(8)]
    assert kv_head_range(8, 2, 1) == (4, 4)
    with pytest.raises(ValueError):
        kv_head_range(8, 3, 0)
