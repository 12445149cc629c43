"""Multi-GPU layouts of the decode path (one process per GPU, torch.distributed).

Two layouts, matching how the work divides:

* Sequence sharding (independent rows).  ``shard_sequences`` gives each rank
  a greedy longest-first share of the batch, balanced by attended length, with
  prefix-sharing groups kept whole so shared blocks stay on one rank.  Each
  rank owns a pool holding only its rows' blocks and runs the decode alone —
  no collective on the data path.

* KV-head sharding (large models: few KV heads, long contexts).  Rank r holds
  KV heads [r*Hkv/N, (r+1)*Hkv/N) of every sequence and the query heads that
  read them; block tables and lengths are replicated.  ``FusedHeadGather``
  has the decode kernel itself write every output row into every rank's
  gathered [B, Hq, q_len, D] output over NVLink (CUDA IPC peer mappings) and
  end with a bounded flag exchange between the ranks; ``HeadShardedDecode`` is
  the unfused form (local decode, then an NCCL all-gather and a reorder).
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .workloads import lpt_partition

__all__ = ["shard_sequences", "kv_head_range", "HeadShardedDecode", "FusedHeadGather"]


def shard_sequences(attended_lengths, world: int, group_size: int = 0) -> list[list[int]]:
    """Row ids per rank, balanced by attended tokens (greedy longest-first).

    ``group_size > 0`` keeps consecutive groups of that many rows together
    (sequences sharing prefix blocks)."""
    n = len(attended_lengths)
    groups = None
    if group_size > 0:
        groups = [list(range(i, min(i + group_size, n))) for i in range(0, n, group_size)]
    return lpt_partition(attended_lengths, world, groups=groups)


def kv_head_range(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """(first, count) of the KV heads rank ``rank`` owns under head sharding."""
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} KV heads do not divide over {world} ranks")
    per = num_kv_heads // world
    return rank * per, per


@dataclass
class HeadShardedDecode:
    """Decode with the KV heads split over the ranks of ``group``.

    ``decode_fn`` computes the local heads' attention (defaults to the sm_100a
    op); the per-rank outputs [B, Hq/N, q, D] are all-gathered into a
    [N, B, Hq/N, q, D] buffer and returned as a [B, Hq, q, D] tensor in the
    global head order (rank r's heads are r*Hq/N .. (r+1)*Hq/N - 1).  ``out=``
    takes that [B, Hq, q, D] result, as ``FusedHeadGather`` does.
    """

    group: dist.ProcessGroup | None = None
    decode_fn: Callable | None = None
    _gather_buf: torch.Tensor | None = None

    def __call__(self, query, key_cache, value_cache, block_tables, context_lens, scale,
                 slot_mapping=None, key=None, value=None, **kw) -> torch.Tensor:
        fn = self.decode_fn
        if fn is None:
            from .paged_attention import paged_attention_decode as fn
        dest = kw.pop("out", None)
        local = fn(query, key_cache, value_cache, block_tables, context_lens, scale, slot_mapping,
                   key, value, **kw)
        world = dist.get_world_size(self.group)
        B, hl, q, D = local.shape
        shape = (world * B, hl, q, D)  # rank chunks concatenated along dim 0
        if self._gather_buf is None or tuple(self._gather_buf.shape) != shape \
                or self._gather_buf.dtype != local.dtype or self._gather_buf.device != local.device:
            self._gather_buf = torch.empty(shape, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(self._gather_buf, local.contiguous(), group=self.group)
        result = self._gather_buf.view(world, B, hl, q, D).permute(1, 0, 2, 3, 4)
        if dest is None:
            return result.reshape(B, world * hl, q, D)
        if tuple(dest.shape) != (B, world * hl, q, D):
            raise ValueError("out must be [batch, total query heads, q_len, head_dim]")
        dest.view(B, world, hl, q, D).copy_(result)
        return dest


# Peer allocations mapped into this process, by IPC handle: an allocation is
# opened once however many buffers inside it are shared, and released when the
# last user lets it go.
_ipc_bases: dict[bytes, int] = {}
_ipc_users: dict[bytes, int] = {}


def _ipc_import(handle_bytes: bytes, offset: int) -> int:
    base = _ipc_bases.get(handle_bytes)
    if base is None:
        h = _lib.IpcHandle()
        ctypes.memmove(h.bytes, handle_bytes, _lib.PA_IPC_HANDLE_BYTES)
        h.offset = 0
        ptr = ctypes.c_void_p()
        _lib.check(_lib.load().pa_ipc_import(ctypes.byref(h), ctypes.byref(ptr)), "pa_ipc_import")
        base = int(ptr.value)
        _ipc_bases[handle_bytes] = base
    _ipc_users[handle_bytes] = _ipc_users.get(handle_bytes, 0) + 1
    return base + offset


def _ipc_drop(handle_bytes: bytes) -> None:
    _ipc_users[handle_bytes] -= 1
    if _ipc_users[handle_bytes] == 0:
        _lib.check(_lib.load().pa_ipc_release(ctypes.c_void_p(_ipc_bases.pop(handle_bytes))), "pa_ipc_release")
        del _ipc_users[handle_bytes]


class _GatherState:
    def __init__(self, key, blob, outs, out_ranks, flags_ranks, counters, peer_handles):
        self.key, self.blob, self.outs = key, blob, outs
        self.out_ranks, self.flags_ranks, self.counters = out_ranks, flags_ranks, counters
        self.peer_handles = peer_handles  # IPC handles of the other ranks' allocations


class FusedHeadGather:
    """KV-head-sharded decode with the all-gather fused into the decode kernel.

    Called like ``HeadShardedDecode`` (the local heads' query and caches, the
    replicated tables and lengths) and returns [B, Hq, q_len, D] in the global
    head order.  Every rank must make the same calls in the same order.  The
    decode kernel stores each finished row of this rank's heads into every
    rank's gathered output (peer memory over NVLink), and its last warp raises
    this rank's flag at every rank and waits at most ``wait_s`` for theirs; a
    rank that does not arrive in time is reported as
    ``PA_DEVERR_WAIT_TIMEOUT`` (``read_device_errors``) instead of hanging.

    After a wait runs out the ranks no longer agree on which call is which, so
    the kernel poisons the exchange: every later call on every rank reports
    ``PA_DEVERR_GATHER``, and the call after one whose error has come back
    raises RuntimeError.  A call that raised marks this object broken: it then
    refuses calls until every rank has called ``close()``, and the next call
    sets up fresh buffers and flags on every rank together.

    The gathered outputs are two buffers used in turn: another rank may start
    writing this rank's buffer for call k+2 as soon as this rank's kernel of
    call k+1 is done, so the tensor returned must be consumed by work ordered
    on this stream before the next call.  Pass ``out=`` to get the result
    copied there (on this stream, right after the kernel) for consumers on
    other streams.  Setup (one collective to swap IPC handles) happens on the
    first call of a shape, not under a CUDA-graph capture.
    """

    def __init__(self, group: dist.ProcessGroup | None = None, wait_s: float = 2.0):
        self.group = group
        self.wait_ns = int(wait_s * 1e9)
        self._state: _GatherState | None = None
        self._calls = 0
        self._broken: str | None = None
        self._unfused = HeadShardedDecode(group=group)  # fp32: the kernel fuses fp16 / bf16 only

    def close(self) -> None:
        """Release the peer mappings and buffers (collective: every rank calls it
        after its last call; a barrier makes sure no rank still writes)."""
        was_broken, self._broken = self._broken is not None, None
        if self._state is None:
            return
        device = self._state.blob.device
        torch.cuda.synchronize(device)
        if was_broken:
            # the poisoned calls' bits: reported already, and the flags they
            # describe go away with this state
            from .paged_attention import read_device_errors

            read_device_errors(device, clear=True)
        dist.barrier(group=self.group)
        for hb in self._state.peer_handles:
            _ipc_drop(hb)
        self._state = None

    def _setup(self, B, Hq_total, q, D, dtype, device) -> _GatherState:
        world, rank = dist.get_world_size(self.group), dist.get_rank(self.group)
        key = (B, Hq_total, q, D, dtype, device)
        out_bytes = B * Hq_total * q * D * torch.tensor([], dtype=dtype).element_size()
        out_bytes = (out_bytes + 255) // 256 * 256
        flags_off = 2 * out_bytes
        blob = torch.zeros(flags_off + max(256, 4 * world), dtype=torch.uint8, device=device)
        h = _lib.IpcHandle()
        _lib.check(_lib.load().pa_ipc_export(ctypes.c_void_p(blob.data_ptr()), ctypes.byref(h)), "pa_ipc_export")
        mine = (bytes(h.bytes), int(h.offset))
        handles = [None] * world
        dist.all_gather_object(handles, mine, group=self.group)
        bases = [blob.data_ptr() if r == rank else _ipc_import(*handles[r]) for r in range(world)]
        peer_handles = [handles[r][0] for r in range(world) if r != rank]
        out_ranks = [torch.tensor([b + par * out_bytes for b in bases], dtype=torch.int64, device=device)
                     for par in (0, 1)]
        flags_ranks = torch.tensor([b + flags_off for b in bases], dtype=torch.int64, device=device)
        n = B * Hq_total * q * D
        outs = [blob[par * out_bytes:par * out_bytes + n * torch.tensor([], dtype=dtype).element_size()]
                .view(dtype).view(B, Hq_total, q, D) for par in (0, 1)]
        counters = torch.zeros(2, dtype=torch.int32, device=device)  # epoch, finished warps
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)  # every rank has mapped every buffer before any kernel writes
        return _GatherState(key, blob, outs, out_ranks, flags_ranks, counters, peer_handles)

    def __call__(self, query, key_cache, value_cache, block_tables, context_lens, scale,
                 slot_mapping=None, key=None, value=None, **kw) -> torch.Tensor:
        from .paged_attention import paged_attention_decode

        if query.dtype == torch.float32:
            dest = kw.pop("out", None)
            res = self._unfused(query, key_cache, value_cache, block_tables, context_lens, scale,
                                slot_mapping, key, value, **kw)
            return res if dest is None else dest.copy_(res)
        if self._broken is not None:
            raise RuntimeError(f"fused gather out of step ({self._broken}): call close() on every rank, "
                               "then start again")
        world, rank = dist.get_world_size(self.group), dist.get_rank(self.group)
        B, hl, q, D = query.shape
        key_ = (B, hl * world, q, D, query.dtype, query.device)
        if self._state is None or self._state.key != key_:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("run one fused-gather call of this shape before CUDA-graph capture")
            self.close()  # a new shape on every rank at once: drop the old buffers together
            self._state = self._setup(*key_)
            self._calls = 0
        st = self._state
        par = self._calls & 1
        self._calls += 1
        g = _lib.GatherArgs()
        g.num_ranks, g.rank, g.head_offset = world, rank, rank * hl
        g.out_ranks = st.out_ranks[par].data_ptr()
        g.flags_ranks = st.flags_ranks.data_ptr()
        g.epoch = st.counters.data_ptr()
        g.done_warps = st.counters.data_ptr() + 4
        g.wait_ns = self.wait_ns
        g.total_heads = hl * world
        dest = kw.pop("out", None)
        gathered = st.outs[par]
        try:
            paged_attention_decode(query, key_cache, value_cache, block_tables, context_lens, scale, slot_mapping,
                                   key, value, out=gathered, gather=g, **kw)
        except Exception as exc:
            # this rank's call did not run, or an earlier one failed: either way
            # the ranks' calls no longer pair up
            self._broken = f"{type(exc).__name__}: {exc}"
            raise
        if dest is None:
            return gathered
        if tuple(dest.shape) != tuple(gathered.shape):
            raise ValueError("out must be [batch, total query heads, q_len, head_dim]")
        dest.copy_(gathered)
        return dest
