"""KV-head-sharded decode with the all-gather fused into the decode kernel
(pa_decode_gather): every output row goes to every rank's gathered output and
the call ends with a flag exchange whose wait is bounded.

On one GPU the flag words of "other ranks" are plain device buffers: a layout
of one rank must equal the plain decode bit for bit, and a layout whose second
rank never raises its flag must report PA_DEVERR_WAIT_TIMEOUT within the bound
(a failure detected without a fault; the context stays usable).  With two GPUs
two processes compare the fused gather with the NCCL all-gather and check the
timeout when one rank skips a call."""

from __future__ import annotations

import dataclasses
import os
import socket
from datetime import timedelta

import pytest
import torch

from llm_serving_runtime_b200 import _lib, paged_attention_decode, read_device_errors
from llm_serving_runtime_b200.paged_attention import DeviceErrorFlags, decode_workspace
from llm_serving_runtime_b200.workloads import SPECS, make_workload

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _args(outs, flags, counters, rank, head_offset, total_heads, wait_ns):
    g = _lib.GatherArgs()
    g.num_ranks, g.rank, g.head_offset = len(outs), rank, head_offset
    g._out_ranks = torch.tensor([o.data_ptr() for o in outs], dtype=torch.int64, device=DEV)
    g._flags_ranks = torch.tensor([f.data_ptr() for f in flags], dtype=torch.int64, device=DEV)
    g.out_ranks = g._out_ranks.data_ptr()
    g.flags_ranks = g._flags_ranks.data_ptr()
    g.epoch = counters.data_ptr()
    g.done_warps = counters.data_ptr() + 4
    g.wait_ns = wait_ns
    g.total_heads = total_heads
    return g


def _workload(batch=48):
    spec = dataclasses.replace(SPECS["cfg5-llama3-70b"], batch=batch, length_lo=100, length_hi=3000)
    return make_workload(spec, device=DEV)


def test_one_rank_gather_equals_plain_decode():
    w = _workload()
    plain = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)
    out = torch.full_like(plain, float("nan"))
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    counters = torch.zeros(2, dtype=torch.int32, device=DEV)
    g = _args([out], [flags], counters, 0, 0, plain.shape[1], 2_000_000_000)
    read_device_errors(DEV)
    for call in (1, 2):
        out.fill_(float("nan"))
        paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                               out=out, gather=g, validate=True)
        assert torch.equal(out, plain)
        assert counters.tolist() == [call, 0] and flags.tolist() == [call]


_POISONED_1 = (1 | 0x80000000) - (1 << 32)  # epoch 1 with the poison bit, read back as int32


def test_missing_rank_times_out_without_a_fault():
    w = _workload(batch=24)
    plain = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)
    B, Hq, q, D = plain.shape
    outs = [torch.zeros(B, 2 * Hq, q, D, dtype=plain.dtype, device=DEV) for _ in range(2)]
    flags = [torch.zeros(2, dtype=torch.int32, device=DEV) for _ in range(2)]  # rank 1 never raises its flag
    counters = torch.zeros(2, dtype=torch.int32, device=DEV)
    g = _args(outs, flags, counters, 0, 0, 2 * Hq, 50_000_000)  # 50 ms
    read_device_errors(DEV)
    paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                           out=outs[0], gather=g)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == DeviceErrorFlags.WAIT_TIMEOUT | DeviceErrorFlags.GATHER
    for o in outs:  # rank 0's rows reached both gathered outputs
        assert torch.equal(o[:, :Hq], plain)
    # the wait ran out, so rank 0 poisoned its epoch and its flag at both ranks
    assert flags[1].tolist() == [_POISONED_1, 0] and flags[0].tolist() == [_POISONED_1, 0]
    assert counters.tolist() == [_POISONED_1, 0]
    # the next gather call reports the broken exchange at once instead of waiting again
    flags[1][1] = 2  # even a late flag of rank 1 does not revive it
    paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                           out=outs[0], gather=g)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == DeviceErrorFlags.GATHER
    assert counters.tolist() == [_POISONED_1, 0]
    again = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                                   validate=True)
    assert torch.equal(again, plain)


def test_peer_more_than_one_call_ahead_is_out_of_step():
    w = _workload(batch=16)
    plain = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)
    B, Hq, q, D = plain.shape
    outs = [torch.zeros(B, 2 * Hq, q, D, dtype=plain.dtype, device=DEV) for _ in range(2)]
    flags = [torch.zeros(2, dtype=torch.int32, device=DEV) for _ in range(2)]
    flags[0][1] = 3  # rank 1's flag claims it finished call 3 while rank 0 makes call 1
    counters = torch.zeros(2, dtype=torch.int32, device=DEV)
    g = _args(outs, flags, counters, 0, 0, 2 * Hq, 2_000_000_000)
    read_device_errors(DEV)
    paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                           out=outs[0], gather=g)
    torch.cuda.synchronize()
    assert read_device_errors(DEV) == DeviceErrorFlags.GATHER
    assert counters.tolist() == [_POISONED_1, 0]


def test_bad_block_id_raises_at_the_next_call_without_validate():
    w = _workload(batch=8)
    args = (w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)
    read_device_errors(DEV)
    bad = w.block_tables.clone()
    bad[3, 0] = w.key_cache.shape[0] + 7
    paged_attention_decode(w.query, w.key_cache, w.value_cache, bad, w.context_lens, w.scale)  # returns
    torch.cuda.synchronize()  # the error word's copy has landed
    with pytest.raises(IndexError, match="out of range"):
        paged_attention_decode(*args)
    assert read_device_errors(DEV) == 0  # raising read and cleared it
    good = paged_attention_decode(*args)
    torch.cuda.synchronize()
    assert torch.equal(paged_attention_decode(*args), good)


def test_an_error_outlives_the_check_table_eviction():
    """More workspaces than the table of deferred checks holds: the entry of
    the failing call's workspace is dropped on the way, but its device word
    keeps the error bits, so the workspace's next calls still raise."""
    w = _workload(batch=8)
    args = (w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)
    paged_attention_decode(*args)
    nbytes = decode_workspace(DEV).numel()
    spaces = [torch.zeros(nbytes, dtype=torch.uint8, device=DEV) for _ in range(130)]
    good = paged_attention_decode(*args, workspace=spaces[1])
    bad = w.block_tables.clone()
    bad[2, 0] = w.key_cache.shape[0] + 3
    paged_attention_decode(w.query, w.key_cache, w.value_cache, bad, w.context_lens, w.scale,
                           workspace=spaces[0])  # returns; the error lands in spaces[0]
    torch.cuda.synchronize()
    for ws in spaces[1:]:
        assert torch.allclose(paged_attention_decode(*args, workspace=ws), good, rtol=0, atol=2e-3)
    torch.cuda.synchronize()
    with pytest.raises(IndexError, match="out of range"):
        for _ in range(2):  # the first call raises if the entry survived, else the second
            paged_attention_decode(*args, workspace=spaces[0])
            torch.cuda.synchronize()
    assert read_device_errors(workspace=spaces[0]) == 0
    torch.cuda.synchronize()
    assert torch.allclose(paged_attention_decode(*args, workspace=spaces[0]), good, rtol=0, atol=2e-3)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_rank_worker(rank: int, port: int) -> None:
    import torch.distributed as dist

    from llm_serving_runtime_b200.sharding import FusedHeadGather, HeadShardedDecode, kv_head_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=timedelta(seconds=60), device_id=dev)
    try:
        spec = dataclasses.replace(SPECS["cfg5-llama3-70b"], batch=32, length_lo=100, length_hi=4000)
        w = make_workload(spec, device=dev, kv_heads=kv_head_range(spec.num_kv_heads, 2, rank))
        args = (w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)
        fused, nccl = FusedHeadGather(wait_s=10.0), HeadShardedDecode()
        for _ in range(3):  # both gathered buffers, twice the first
            a = fused(*args).clone()
            b = nccl(*args)
            assert torch.equal(a, b), f"rank {rank}: fused gather differs from the NCCL all-gather"
        # against the oracle: both ranks draw the same data for their own KV
        # heads, so every rank's slice of the gathered output is that decode
        from _util import TOL, max_err, oracle_rows

        rows = [0, 5, 17, 31]
        ref = oracle_rows(*args[:5], w.scale, w.q_len, rows)
        hl = w.query.shape[1]
        for r2 in range(2):
            err = max_err(a[rows][:, r2 * hl:(r2 + 1) * hl], ref)
            assert err <= TOL[torch.bfloat16], f"rank {rank}: slice of rank {r2} off the oracle by {err}"
        dest = torch.empty_like(b)
        assert fused(*args, out=dest) is dest and torch.equal(dest, b)
        # fp32 takes the NCCL form under the same call
        args32 = (w.query.float(), w.key_cache.float(), w.value_cache.float()) + args[3:]
        assert torch.allclose(fused(*args32), nccl(*args32))
        torch.cuda.synchronize()
        dist.barrier()
        fused.close()
        # failure detection: rank 1 skips one call, rank 0's wait runs out
        short = FusedHeadGather(wait_s=0.2)
        short(*args)
        torch.cuda.synchronize()
        dist.barrier()
        assert read_device_errors(dev, clear=False) == 0
        if rank == 0:
            short(*args)
            torch.cuda.synchronize()
        dist.barrier()
        # the call after the skip reports the failure on both ranks instead of
        # returning rows of different calls: rank 0 raises on the error that came
        # back; rank 1's kernel finds rank 0's poisoned flag, and its next call raises
        if rank == 0:
            with pytest.raises(RuntimeError, match="timed out"):
                short(*args)
        else:
            short(*args)
            torch.cuda.synchronize()
            with pytest.raises(RuntimeError, match="out of step"):
                short(*args)
        with pytest.raises(RuntimeError, match="close"):
            short(*args)  # broken until every rank closes
        dist.barrier()
        short.close()
        # a fresh set-up on both ranks pairs the calls up again
        for _ in range(2):
            assert torch.equal(short(*args), nccl(*args))
        torch.cuda.synchronize()
        assert read_device_errors(dev) == 0
        dist.barrier()
        short.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_fused_gather_matches_nccl_and_detects_a_missing_rank():
    import torch.multiprocessing as mp

    mp.spawn(_two_rank_worker, args=(_free_port(),), nprocs=2, join=True)
