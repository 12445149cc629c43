"""Paged decode attention with a fused KV append — the north-star call.

    out = paged_attention_decode(query, key_cache, value_cache, block_tables,
                                 context_lens, scale, slot_mapping,
                                 key=new_k, value=new_v)

* ``query``        [B, Hq, q_len, D] (HF layout; any strides with a unit last stride)
* ``key_cache``    [num_blocks, Hkv, block_size, D] (e.g. GpuKVBlockPool.k_layer_view(l))
* ``value_cache``  same shape as ``key_cache``
* ``block_tables`` int32 [B, max_blocks]: physical block of each logical block
* ``context_lens`` int32 [B]: tokens already cached BEFORE this step's q_len new
  tokens (pass ``context_lens_include_new=True`` for the reference's seq_lens,
  which include them, runtime/phase2/paged_attention_triton.py:50)
* ``scale``        softmax scale (usually head_dim ** -0.5)
* ``slot_mapping`` int64 [B * q_len] or None: cache slot (block * bs + offset) of
  each new token; -1 skips a padding token.  When None and ``key``/``value``
  are given, the slots follow from ``block_tables`` at positions
  ``context_lens[b] + t`` — the reference's ``write_tokens_batch`` arithmetic
  (runtime/phase2/paged_kv_kernel.py:217-223).
* ``key``/``value`` [B, Hkv, q_len, D] new rows, appended before attention in
  the same stream; the decode kernel overlaps its prologue with the append
  through programmatic dependent launch.

Query token t of row b attends cached positions 0 .. L_b - q_len + t with
L_b the attended length (causal over the new tokens; q_len = 1 is plain decode),
so one call also serves speculative verification.

Every call launches hand-written sm_100a kernels from ``lib/libpa_b200.so``
through its C ABI; there is no Triton and no CPU fallback.  No call allocates
device memory except the first one on a device (or a larger shape), which sizes
the shared workspace — make that call before capturing a CUDA graph.

Bad inputs (a block id outside the pool, a block table too short for its
length, a slot outside the pool) never fault: the kernels skip the access and
set a bit in the workspace's device error word.  After each call an
asynchronous copy of that word lands in pinned host memory, and the next call
on the same workspace raises ``IndexError`` (the reference's error,
runtime/phase2/paged_kv_kernel.py:118-119, :221-222) once the copy shows a bit
— no host synchronisation on the normal path.  ``validate=True`` (or
``PA_B200_VALIDATE=1``) checks synchronously at the end of the call instead;
``validate=False`` skips the check.  Calls under CUDA-graph capture are not
checked (``read_device_errors`` reads the word after a replay).
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _lib
from ._lib import CacheView, DecodeArgs, KvAppendArgs

__all__ = [
    "paged_attention_decode",
    "kv_append",
    "decode_workspace",
    "read_device_errors",
    "describe_device_errors",
    "device_error",
    "DeviceErrorFlags",
]

_DTYPE_CODE = {
    torch.float32: _lib.PA_DTYPE_FLOAT32,
    torch.float16: _lib.PA_DTYPE_FLOAT16,
    torch.bfloat16: _lib.PA_DTYPE_BFLOAT16,
}


class DeviceErrorFlags:
    BLOCK_ID_RANGE = _lib.PA_DEVERR_BLOCK_ID_RANGE
    TABLE_UNDERRUN = _lib.PA_DEVERR_TABLE_UNDERRUN
    SLOT_RANGE = _lib.PA_DEVERR_SLOT_RANGE
    WAIT_TIMEOUT = _lib.PA_DEVERR_WAIT_TIMEOUT
    PREFIX = _lib.PA_DEVERR_PREFIX
    GATHER = _lib.PA_DEVERR_GATHER


def device_error(flags: int) -> Exception:
    """The exception for a non-zero device error word: IndexError for invalid
    block ids, slots, underruns and prefix groups (the reference's error for
    them); RuntimeError when only a bounded wait ran out or a fused gather fell
    out of step."""
    text = describe_device_errors(flags)
    index_bits = (DeviceErrorFlags.BLOCK_ID_RANGE | DeviceErrorFlags.TABLE_UNDERRUN | DeviceErrorFlags.SLOT_RANGE
                  | DeviceErrorFlags.PREFIX)
    return IndexError(text) if flags & index_bits else RuntimeError(text)


def describe_device_errors(flags: int) -> str:
    parts = []
    if flags & DeviceErrorFlags.BLOCK_ID_RANGE:
        parts.append("physical block id out of range")
    if flags & DeviceErrorFlags.TABLE_UNDERRUN:
        parts.append("block table underrun")
    if flags & DeviceErrorFlags.SLOT_RANGE:
        parts.append("slot outside the pool")
    if flags & DeviceErrorFlags.WAIT_TIMEOUT:
        parts.append("a bounded wait timed out (on a bulk copy, or on a peer rank of a fused gather)")
    if flags & DeviceErrorFlags.PREFIX:
        parts.append("prefix group does not match its members' block tables or bounds")
    if flags & DeviceErrorFlags.GATHER:
        parts.append("fused gather ranks out of step (close() on every rank, then start again)")
    return "; ".join(parts)


_VALIDATE_DEFAULT = os.environ.get("PA_B200_VALIDATE", "0") == "1"

# One workspace per device: status word + merge counters + partial slots.
_ws_lock = threading.Lock()
_workspaces: dict[int, torch.Tensor] = {}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def decode_workspace(device: torch.device, nbytes: int = 256) -> torch.Tensor:
    """The device's shared workspace, grown (zero-filled) to at least ``nbytes``.

    Growing allocates, which a CUDA-graph capture forbids: size it with one
    eager call before capture.  Calls that overlap on the GPU (different streams)
    must not share a workspace — pass ``workspace=`` explicitly there.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        ws = _workspaces.get(idx)
        if ws is None or ws.numel() < nbytes:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "paged decode workspace must be sized before CUDA-graph capture: "
                    "run the same call once eagerly first"
                )
            ws = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=torch.device("cuda", idx))
            _workspaces[idx] = ws
        return ws


def read_device_errors(device: torch.device | None = None, *, clear: bool = True,
                       workspace: torch.Tensor | None = None) -> int:
    """Read (and clear) the PA_DEVERR_* bits the kernels recorded.  Synchronises.

    Clearing also drops the copy of the word that the next call would have
    checked: the bits it holds have been read here."""
    if workspace is None:
        device = device or torch.device("cuda", torch.cuda.current_device())
        workspace = decode_workspace(device)
    if clear:
        with _checks_lock:
            c = _checks.get((workspace.device.index, workspace.data_ptr()))
            if c is not None:
                c.pending = False
    flags = ctypes.c_uint32(0)
    _lib.check(
        _lib.load().pa_read_device_errors(
            workspace.data_ptr(), ctypes.byref(flags), 1 if clear else 0, _stream_ptr(workspace.device)
        ),
        "pa_read_device_errors",
    )
    return int(flags.value)


class _PendingCheck:
    """One in-flight copy of a device error word into pinned host memory."""

    __slots__ = ("host", "stream", "after_call", "landed", "pending")

    def __init__(self, device: torch.device):
        self.host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self.stream = torch.cuda.Stream(device)
        self.after_call = torch.cuda.Event()
        self.landed = torch.cuda.Event()
        self.pending = False


_checks_lock = threading.Lock()
_checks: dict[tuple[int, int], _PendingCheck] = {}


def _capturing() -> bool:
    return torch.cuda.is_current_stream_capturing()


def _raise_landed_errors(word: torch.Tensor) -> None:
    """Raise for the device errors of earlier calls on ``word`` whose copy has
    landed (the word is read again and cleared, synchronously, only then)."""
    with _checks_lock:
        c = _checks.get((word.device.index, word.data_ptr()))
        if c is None or not c.pending or not c.landed.query():
            return
        c.pending = False
        seen = int(c.host.item())
    if seen:
        flags = seen | read_device_errors(workspace=word, clear=True)
        raise device_error(flags)


def _copy_after_call(word: torch.Tensor, stream: torch.cuda.Stream) -> None:
    """Queue a copy of ``word`` to pinned host memory behind the work on
    ``stream`` (on a side stream, so ``stream`` is not held up).  While one copy
    is in flight no other is queued: the word keeps its bits until read, so the
    next copy covers every call since."""
    key = (word.device.index, word.data_ptr())
    with _checks_lock:
        c = _checks.get(key)
        if c is None:
            if len(_checks) >= 64:
                _checks.pop(next(iter(_checks)))
            c = _checks[key] = _PendingCheck(word.device)
        if c.pending:
            return
        c.after_call.record(stream)
        c.stream.wait_event(c.after_call)
        with torch.cuda.stream(c.stream):
            c.host.copy_(word[:4].view(torch.int32), non_blocking=True)
        word.record_stream(c.stream)  # a replaced workspace stays allocated until the copy has run
        c.landed.record(c.stream)
        c.pending = True


def _cache_view(t: torch.Tensor) -> CacheView:
    return CacheView(t.data_ptr(), t.shape[0], t.stride(0), t.stride(1), t.stride(2))


def _check_cache_pair(key_cache: torch.Tensor, value_cache: torch.Tensor) -> None:
    if key_cache.dim() != 4 or value_cache.dim() != 4:
        raise ValueError("key_cache/value_cache must be [num_blocks, num_kv_heads, block_size, head_dim]")
    if key_cache.shape != value_cache.shape:
        raise ValueError("key_cache and value_cache must have the same shape")
    if key_cache.dtype != value_cache.dtype:
        raise ValueError("key_cache and value_cache must have the same dtype")
    if key_cache.stride(3) != 1 or value_cache.stride(3) != 1:
        raise ValueError("cache head_dim must be contiguous")
    if not key_cache.is_cuda or key_cache.device != value_cache.device:
        raise ValueError("caches must be CUDA tensors on one device")
    if key_cache.dtype not in _DTYPE_CODE:
        raise ValueError(f"unsupported cache dtype {key_cache.dtype}")


def _check_new_rows(t: torch.Tensor, name: str, B: int, Hkv: int, q_len: int, D: int,
                    dtype: torch.dtype, device: torch.device) -> None:
    if t.dim() != 4 or tuple(t.shape) != (B, Hkv, q_len, D):
        raise ValueError(f"{name} must be [batch={B}, num_kv_heads={Hkv}, q_len={q_len}, head_dim={D}], "
                         f"got {tuple(t.shape)}")
    if t.dtype != dtype or t.device != device:
        raise ValueError(f"{name} must match the cache dtype and device")
    if t.stride(3) != 1:
        raise ValueError(f"{name} head_dim must be contiguous")


def _as_int32(t: torch.Tensor, device: torch.device, name: str) -> torch.Tensor:
    if t.dtype == torch.int32 and t.device == device:
        return t
    if torch.cuda.is_current_stream_capturing():
        raise ValueError(f"{name} must already be an int32 tensor on {device} during graph capture")
    return t.to(device=device, dtype=torch.int32)


class _with_device:
    """Make ``device`` current for the C calls (they launch on the current device)."""

    __slots__ = ("device", "prev")

    def __init__(self, device: torch.device):
        self.device = device

    def __enter__(self):
        self.prev = torch.cuda.current_device()
        if self.prev != self.device.index:
            torch.cuda.set_device(self.device)
        return self

    def __exit__(self, *exc):
        if self.prev != self.device.index:
            torch.cuda.set_device(self.prev)
        return False


_ws_bytes_cache: dict[tuple, int] = {}


def _workspace_bytes(B: int, Hq: int, Hkv: int, q_len: int, D: int, dcode: int, dev_index: int) -> int:
    key = (B, Hq, Hkv, q_len, D, dcode, dev_index)
    n = _ws_bytes_cache.get(key)
    if n is None:
        n = _lib.load().pa_decode_workspace_bytes(B, Hq, Hkv, q_len, D, dcode, dev_index)
        if n == 0:
            raise RuntimeError(f"pa_decode_workspace_bytes failed: {_lib.last_error()}")
        _ws_bytes_cache[key] = n
    return n


def kv_append(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor | None = None,
    *,
    block_tables: torch.Tensor | None = None,
    positions: torch.Tensor | None = None,
    position_offset: int = 0,
    error_word: torch.Tensor | None = None,
    validate: bool | None = None,
) -> None:
    """Scatter new rows ``key``/``value`` [B, Hkv, q_len, D] into the caches.

    With ``slot_mapping`` (int64 [B*q_len]) token b*q_len+t goes to that slot;
    otherwise to block_tables[b, p // bs] at offset p % bs with
    p = positions[b] + position_offset + t.  Bit-exact.  Invalid slots or block
    ids are skipped and flagged; the next call on the same error word raises
    IndexError (``validate=True``: this call, synchronously).
    """
    _check_cache_pair(key_cache, value_cache)
    device = key_cache.device
    if key.dim() != 4:
        raise ValueError("key must be [batch, num_kv_heads, q_len, head_dim]")
    B, _, q_len, _ = key.shape
    _, Hkv, bs, Dc = key_cache.shape
    _check_new_rows(key, "key", B, Hkv, q_len, Dc, key_cache.dtype, device)
    _check_new_rows(value, "value", B, Hkv, q_len, Dc, key_cache.dtype, device)
    args = KvAppendArgs()
    args.key = key.data_ptr()
    args.key_stride_b, args.key_stride_h, args.key_stride_t = key.stride(0), key.stride(1), key.stride(2)
    args.value = value.data_ptr()
    args.value_stride_b, args.value_stride_h, args.value_stride_t = value.stride(0), value.stride(1), value.stride(2)
    args.key_cache = _cache_view(key_cache)
    args.value_cache = _cache_view(value_cache)
    keep = []
    if slot_mapping is not None:
        if slot_mapping.dtype != torch.int64 or slot_mapping.device != device:
            if torch.cuda.is_current_stream_capturing():
                raise ValueError("slot_mapping must be int64 on the cache device during capture")
            slot_mapping = slot_mapping.to(device=device, dtype=torch.int64)
        if slot_mapping.numel() != B * q_len:
            raise ValueError(f"slot_mapping must have batch*q_len={B * q_len} entries")
        slot_mapping = slot_mapping.reshape(-1)
        if not slot_mapping.is_contiguous():
            raise ValueError("slot_mapping must be contiguous")
        keep.append(slot_mapping)
        args.slot_mapping = slot_mapping.data_ptr()
    else:
        if block_tables is None or positions is None:
            raise ValueError("kv_append needs slot_mapping, or block_tables and positions")
        block_tables = _as_int32(block_tables, device, "block_tables")
        if block_tables.dim() != 2 or block_tables.shape[0] != B or block_tables.stride(1) != 1:
            raise ValueError("block_tables must be int32 [batch, max_blocks] with contiguous rows")
        if positions.device != device or positions.dtype not in (torch.int32, torch.int64):
            positions = _as_int32(positions, device, "positions")
        positions = positions.reshape(-1)
        if positions.numel() != B or not positions.is_contiguous():
            raise ValueError("positions must be a contiguous [batch] tensor")
        keep += [block_tables, positions]
        args.block_tables = block_tables.data_ptr()
        args.block_table_stride = block_tables.stride(0)
        args.max_blocks = block_tables.shape[1]
        args.positions = positions.data_ptr()
        args.positions_is_int64 = 1 if positions.dtype == torch.int64 else 0
        args.position_offset = int(position_offset)
    args.batch, args.q_len, args.num_kv_heads, args.head_dim, args.block_size = B, q_len, Hkv, Dc, bs
    args.dtype = _DTYPE_CODE[key_cache.dtype]
    if error_word is None:
        error_word = decode_workspace(device)
    args.error_flags = error_word.data_ptr()
    deferred = validate is None and not _VALIDATE_DEFAULT and not _capturing()
    if deferred:
        _raise_landed_errors(error_word)
    with _with_device(device):
        _lib.check(_lib.load().pa_kv_append(ctypes.byref(args), _stream_ptr(device)), "pa_kv_append")
    if deferred:
        _copy_after_call(error_word, torch.cuda.current_stream(device))
    elif validate if validate is not None else _VALIDATE_DEFAULT:
        flags = read_device_errors(workspace=error_word)
        if flags:
            raise device_error(flags)


def _cascade_workspace_bytes(B: int, Hq: int, Hkv: int, q_len: int, D: int, dcode: int, dev_index: int,
                             groups) -> int:
    key = (B, Hq, Hkv, q_len, D, dcode, dev_index, groups.num_groups, int(groups.max_members),
           int(groups.max_prefix_len))
    n = _ws_bytes_cache.get(key)
    if n is None:
        n = _lib.load().pa_cascade_workspace_bytes(B, Hq, Hkv, q_len, D, dcode, dev_index, *key[7:])
        if n == 0:
            raise RuntimeError(f"pa_cascade_workspace_bytes failed: {_lib.last_error()}")
        _ws_bytes_cache[key] = n
    return n


def paged_attention_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    slot_mapping: torch.Tensor | None = None,
    key: torch.Tensor | None = None,
    value: torch.Tensor | None = None,
    *,
    out: torch.Tensor | None = None,
    context_lens_include_new: bool = False,
    workspace: torch.Tensor | None = None,
    validate: bool | None = None,
    prefix_groups=None,
    gather=None,
) -> torch.Tensor:
    """Append this step's K/V (optional) and attend; returns [B, Hq, q_len, D].

    ``prefix_groups`` (a ``prefix_sharing.PrefixGroups``) marks rows whose
    tables share leading physical blocks: the call then attends each shared
    block once per group (cascade) and returns the same result.

    ``gather`` (internal: a ``_lib.GatherArgs`` with ``total_heads`` attached,
    built by ``sharding.FusedHeadGather``) makes ``out`` this rank's gathered
    output [B, total query heads, q_len, D] and writes the local heads' rows to
    every rank's gathered output in the same kernel."""
    _check_cache_pair(key_cache, value_cache)
    device = key_cache.device
    if query.dim() != 4:
        raise ValueError("query must be [batch, num_q_heads, q_len, head_dim]")
    B, Hq, q_len, D = query.shape
    _, Hkv, bs, Dc = key_cache.shape
    if D != Dc:
        raise ValueError(f"query head_dim {D} does not match cache head_dim {Dc}")
    if query.dtype != key_cache.dtype or query.device != device:
        raise ValueError("query must match the cache dtype and device")
    if query.stride(3) != 1:
        raise ValueError("query head_dim must be contiguous")
    if Hq % Hkv != 0:
        raise ValueError(f"num_q_heads {Hq} must be a multiple of num_kv_heads {Hkv}")
    if block_tables.dim() != 2 or block_tables.shape[0] != B:
        # paged_attention_triton.py:752-753
        raise ValueError("query batch size must match block_tables rows")
    block_tables = _as_int32(block_tables, device, "block_tables")
    if block_tables.stride(1) != 1:
        raise ValueError("block_tables rows must be contiguous")
    context_lens = _as_int32(context_lens.reshape(-1), device, "context_lens")
    if context_lens.numel() != B or not context_lens.is_contiguous():
        raise ValueError("context_lens must be a contiguous [batch] tensor")
    if (key is None) != (value is None):
        raise ValueError("key and value must be given together")
    if slot_mapping is not None and key is None:
        raise ValueError("slot_mapping needs key and value")
    out_heads = Hq if gather is None else gather.total_heads
    if out is None:
        if gather is not None:
            raise ValueError("the fused gather writes into the gathered output given as out")
        out = torch.empty((B, Hq, q_len, D), dtype=query.dtype, device=device)
    elif tuple(out.shape) != (B, out_heads, q_len, D) or out.dtype != query.dtype or out.device != device \
            or out.stride(3) != 1:
        raise ValueError("out must be [batch, num_q_heads, q_len, head_dim] in the query dtype")
    if B == 0:
        return out

    lib = _lib.load()
    dcode = _DTYPE_CODE[query.dtype]
    cascade = prefix_groups is not None and prefix_groups.num_groups > 0
    if cascade:
        if prefix_groups.seq_group.numel() != B or prefix_groups.seq_group.device != device:
            raise ValueError("prefix_groups must describe this batch on the cache's device")
        need = _cascade_workspace_bytes(B, Hq, Hkv, q_len, D, dcode, device.index, prefix_groups)
    else:
        need = _workspace_bytes(B, Hq, Hkv, q_len, D, dcode, device.index)
    if workspace is None:
        workspace = decode_workspace(device, need)
    deferred = validate is None and not _VALIDATE_DEFAULT and not _capturing()
    if deferred:
        _raise_landed_errors(workspace)

    appended = False
    if key is not None:
        kv_append(
            key, value, key_cache, value_cache, slot_mapping,
            block_tables=block_tables, positions=context_lens,
            position_offset=-q_len if context_lens_include_new else 0,
            error_word=workspace, validate=False,
        )
        appended = True

    args = DecodeArgs()
    args.query = query.data_ptr()
    args.query_stride_b, args.query_stride_h, args.query_stride_t = query.stride(0), query.stride(1), query.stride(2)
    args.key_cache = _cache_view(key_cache)
    args.value_cache = _cache_view(value_cache)
    args.block_tables = block_tables.data_ptr()
    args.block_table_stride = block_tables.stride(0)
    args.max_blocks = block_tables.shape[1]
    args.context_lens = context_lens.data_ptr()
    args.len_offset = 0 if context_lens_include_new else q_len
    args.out = out.data_ptr()
    args.out_stride_b, args.out_stride_h, args.out_stride_t = out.stride(0), out.stride(1), out.stride(2)
    args.batch, args.q_len, args.num_q_heads, args.num_kv_heads = B, q_len, Hq, Hkv
    args.head_dim, args.block_size = D, bs
    args.dtype = dcode
    args.scale = float(scale)
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel()
    args.allow_overlap_with_previous = 1 if appended else 0
    with _with_device(device):
        if gather is not None:
            _lib.check(lib.pa_decode_gather(ctypes.byref(args), ctypes.byref(gather), _stream_ptr(device)),
                       "pa_decode_gather")
        elif cascade:
            groups = prefix_groups.to_args()
            _lib.check(lib.pa_decode_cascade(ctypes.byref(args), ctypes.byref(groups), _stream_ptr(device)),
                       "pa_decode_cascade")
        else:
            _lib.check(lib.pa_decode(ctypes.byref(args), _stream_ptr(device)), "pa_decode")
    if deferred:
        _copy_after_call(workspace, torch.cuda.current_stream(device))
    elif validate if validate is not None else _VALIDATE_DEFAULT:
        flags = read_device_errors(workspace=workspace)
        if flags:
            raise device_error(flags)
    return out
