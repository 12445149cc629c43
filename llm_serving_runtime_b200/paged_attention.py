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

import numpy as np
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
    "SmSpeeds",
    "sm_speeds",
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
# Per-SM shares of large decode calls (SmSpeeds); PA_B200_SM_SHARES=0 keeps
# every SM's share equal.
_SM_SHARES = os.environ.get("PA_B200_SM_SHARES", "1") != "0"

# One workspace per device: status word + merge counters + partial slots.
_ws_lock = threading.Lock()
_workspaces: dict[int, torch.Tensor] = {}


def _stream_ptr(device: torch.device) -> int:
    """The current stream's raw handle (no Stream object per call)."""
    return torch._C._cuda_getCurrentRawStream(device.index if device.index is not None
                                              else torch.cuda.current_device())


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


# The workspace's first bytes: the device error word at 0, then (at
# PA_WS_SM_TIMING_OFFSET) one pa_sm_timing record per SM.
_TIMING_DTYPE = np.dtype([("t0", "<u8"), ("t1", "<u8"), ("cost", "<u4"), ("smid", "<u4"), ("tag", "<u4"),
                          ("pad", "<u4")])
_HEAD_BYTES = _lib.PA_WS_SM_TIMING_OFFSET + _lib.PA_MAX_SM_WEIGHTS * _TIMING_DTYPE.itemsize


class SmSpeeds:
    """Relative streaming speed of each SM of one device.

    The decode kernel gives every SM of a large call a share of the work in
    proportion to these weights (pa_decode_args.sm_weights): SMs stream at
    speeds up to ~10 % apart, in a pattern fixed by where they sit, and equal
    shares would leave the call waiting on the slowest.  The weights start
    equal.  The first SAMPLES large calls on the device each write one timing
    record per SM (pa_sm_timing: its share and how long it took), which comes
    back with the error word's asynchronous copy.  An SM's speed varies a
    little from call to call (two calls' speeds correlate about 0.87 on B200),
    so the weights are the mean of the relative speeds over the samples so far.
    After SAMPLES samples they stay fixed, so later calls split their work
    identically and give bit-identical results on identical inputs.  A call too
    small for per-SM shares writes no records; after one, the next calls are
    tagged only every 2, 4, ... 1024 calls, so small calls pay almost nothing."""

    SAMPLES = 8

    def __init__(self, num_sms: int):
        self.n = num_sms if 0 < num_sms <= _lib.PA_MAX_SM_WEIGHTS else 0
        self.weights = torch.ones(max(self.n, 1), dtype=torch.float32)  # host memory the C call reads
        self.weights_ptr = self.weights.data_ptr()  # updated in place, so the address stays
        self.samples = 0
        self._tag = 0
        self._sum = np.zeros(max(self.n, 1))
        self._misses = 0
        self._skip = 0

    @property
    def learning(self) -> bool:
        return self.n > 0 and self.samples < self.SAMPLES

    def want_sample(self) -> bool:
        """Whether the next call should carry a tag (backs off after misses)."""
        if not self.learning:
            return False
        if self._skip > 0:
            self._skip -= 1
            return False
        return True

    def new_tag(self) -> int:
        self._tag = self._tag % 0x7FFFFFFF + 1
        return self._tag

    def absorb(self, tag: int, raw: np.ndarray) -> bool:
        """Take one call's timing records (raw bytes); False when they are not
        that call's (a call too small for per-SM shares writes none)."""
        rec = raw.view(_TIMING_DTYPE)[: self.n]
        if rec.shape[0] != self.n or (rec["tag"] != tag).any():
            self._misses = min(self._misses + 1, 10)
            self._skip = 1 << self._misses
            return False
        self._misses = 0
        smid = rec["smid"].astype(np.int64)
        if smid.max() >= self.n or np.unique(smid).size != self.n:
            return False  # a CTA ran off its own SM: the records do not say which SM was how fast
        busy = (rec["t1"].astype(np.int64) - rec["t0"].astype(np.int64)).astype(np.float64)
        if (busy <= 0).any() or (rec["cost"] == 0).any():
            return False
        speed = rec["cost"].astype(np.float64) / busy
        rel = np.empty(self.n)
        rel[smid] = speed / speed.mean()
        self._sum += np.clip(rel, 0.6, 1.6)
        self.samples += 1
        w = self._sum / self.samples
        w = w / w.mean()
        self.weights.copy_(torch.from_numpy(w.astype(np.float32)))
        return True


_speeds_lock = threading.Lock()
_speeds: dict[int, SmSpeeds] = {}


def sm_speeds(device: torch.device) -> SmSpeeds:
    """The device's per-SM speed table (created on first use)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _speeds.get(idx)
    if t is not None:
        return t
    with _speeds_lock:
        t = _speeds.get(idx)
        if t is None:
            t = _speeds[idx] = SmSpeeds(torch.cuda.get_device_properties(idx).multi_processor_count)
        return t


class _PendingCheck:
    """One in-flight copy of a workspace's first bytes (the device error word,
    and after a tagged call the per-SM timing records) into pinned memory.

    The copy runs on a side stream behind an event recorded on the call's
    stream, through raw CUDA runtime calls on the handles (a few microseconds
    of host time per call; torch's stream and event wrappers cost ten times
    that).  The workspace tensor is held until the copy has landed, so the
    caching allocator cannot hand its memory out meanwhile."""

    __slots__ = ("host", "host_ptr", "side", "side_ptr", "ev_call", "ev_landed", "pending", "tag", "speeds",
                 "word")

    def __init__(self, device: torch.device, rt):
        self.host = torch.zeros(_HEAD_BYTES, dtype=torch.uint8, pin_memory=True)
        self.host_ptr = self.host.data_ptr()
        with torch.cuda.device(device):
            self.side = torch.cuda.Stream(device)
            self.side_ptr = self.side.cuda_stream
            evs = []
            for _ in range(2):
                ev = ctypes.c_void_p()
                if rt.cudaEventCreateWithFlags(ctypes.byref(ev), 0x2) != 0:  # cudaEventDisableTiming
                    raise RuntimeError("cudaEventCreateWithFlags failed")
                evs.append(ev.value)
        self.ev_call, self.ev_landed = evs
        self.pending = False
        self.tag = 0
        self.speeds = None
        self.word = None


_checks_lock = threading.Lock()
_checks: dict[tuple[int, int], _PendingCheck] = {}


def _capturing() -> bool:
    return torch.cuda.is_current_stream_capturing()


def _raise_landed_errors(word: torch.Tensor) -> None:
    """Raise for the device errors of earlier calls on ``word`` whose copy has
    landed (the word is read again and cleared, synchronously, only then)."""
    c = _checks.get((word.device.index, word.data_ptr()))
    if c is None or not c.pending:
        return
    with _checks_lock:
        if not c.pending:
            return
        q = _lib.cudart().cudaEventQuery(c.ev_landed)
        if q == 600:  # cudaErrorNotReady
            return
        if q != 0:
            raise RuntimeError(f"cudaEventQuery on the error-word copy failed ({q})")
        c.pending = False
        c.word = None
        seen = int(c.host[:4].view(torch.int32).item())
        if c.tag:
            n = c.speeds.n
            c.speeds.absorb(c.tag, c.host.numpy()[_lib.PA_WS_SM_TIMING_OFFSET:][: n * _TIMING_DTYPE.itemsize])
            c.tag = 0
    if seen:
        flags = seen | read_device_errors(workspace=word, clear=True)
        raise device_error(flags)


def _copy_is_free(word: torch.Tensor) -> bool:
    """No copy of ``word``'s workspace is in flight (the next one may carry timing)."""
    c = _checks.get((word.device.index, word.data_ptr()))
    return c is None or not c.pending


def _copy_after_call(word: torch.Tensor, stream_ptr: int, tag: int = 0, speeds: "SmSpeeds | None" = None) -> None:
    """Queue a copy of ``word`` to pinned host memory behind the work on the
    stream ``stream_ptr`` (on a side stream, so that stream is not held up).
    While one copy is in flight no other is queued: the word keeps its bits
    until read, so the next copy covers every call since.  After a call tagged
    ``tag`` the copy also takes the call's per-SM timing records, for
    ``speeds``."""
    rt = _lib.cudart()
    if rt is None:
        return  # no runtime to queue the copy with: the synchronous checks still work
    key = (word.device.index, word.data_ptr())
    with _checks_lock:
        c = _checks.get(key)
        if c is None:
            if len(_checks) >= 64:
                # drop the oldest entry whose copy is not in flight (its pinned
                # buffer may then be freed; a landed but unread error stays in
                # the device word, which only a read clears, so the workspace's
                # next call reports it); with every copy in flight, skip this check
                idle = next((k for k, v in _checks.items()
                             if not v.pending or rt.cudaEventQuery(v.ev_landed) == 0), None)
                if idle is None:
                    return
                old = _checks.pop(idle)
                rt.cudaEventDestroy(old.ev_call)
                rt.cudaEventDestroy(old.ev_landed)
            c = _checks[key] = _PendingCheck(word.device, rt)
        if c.pending:
            return
        nbytes = 4
        if tag and speeds is not None and word.numel() >= _lib.PA_WS_SM_TIMING_OFFSET + speeds.n * 32:
            nbytes = _lib.PA_WS_SM_TIMING_OFFSET + speeds.n * _TIMING_DTYPE.itemsize
            c.tag, c.speeds = tag, speeds
        if (rt.cudaEventRecord(c.ev_call, stream_ptr) or rt.cudaStreamWaitEvent(c.side_ptr, c.ev_call, 0)
                or rt.cudaMemcpyAsync(c.host_ptr, word.data_ptr(), nbytes, 2, c.side_ptr)  # device to host
                or rt.cudaEventRecord(c.ev_landed, c.side_ptr)):
            raise RuntimeError("queueing the error-word copy failed")
        c.word = word
        c.pending = True


def _cache_view(t: torch.Tensor) -> CacheView:
    st = t.stride()
    return CacheView(t.data_ptr(), t.shape[0], st[0], st[1], st[2])


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
# pa_decode's message for a batch beyond its per-sequence shared-memory tables
_BATCH_LIMIT_TEXT = "too large for the decode kernel's shared memory"


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
    args.key_stride_b, args.key_stride_h, args.key_stride_t = key.stride()[:3]
    args.value = value.data_ptr()
    args.value_stride_b, args.value_stride_h, args.value_stride_t = value.stride()[:3]
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
        _copy_after_call(error_word, _stream_ptr(device))
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
    stream_ptr = _stream_ptr(device)

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
    args.query_stride_b, args.query_stride_h, args.query_stride_t = query.stride()[:3]
    args.key_cache = _cache_view(key_cache)
    args.value_cache = _cache_view(value_cache)
    args.block_tables = block_tables.data_ptr()
    args.block_table_stride = block_tables.stride(0)
    args.max_blocks = block_tables.shape[1]
    args.context_lens = context_lens.data_ptr()
    args.len_offset = 0 if context_lens_include_new else q_len
    args.out = out.data_ptr()
    args.out_stride_b, args.out_stride_h, args.out_stride_t = out.stride()[:3]
    args.batch, args.q_len, args.num_q_heads, args.num_kv_heads = B, q_len, Hq, Hkv
    args.head_dim, args.block_size = D, bs
    args.dtype = dcode
    args.scale = float(scale)
    args.workspace = workspace.data_ptr()
    args.workspace_bytes = workspace.numel()
    args.allow_overlap_with_previous = 1 if appended else 0
    speeds = sm_speeds(device)
    tag = 0
    if speeds.n and _SM_SHARES:
        args.sm_weights = speeds.weights_ptr
        args.num_sm_weights = speeds.n
        if deferred and speeds.learning and query.dtype != torch.float32 and _copy_is_free(workspace) \
                and speeds.want_sample():
            tag = speeds.new_tag()
            args.sm_timing_tag = tag
    with _with_device(device):
        if gather is not None:
            _lib.check(lib.pa_decode_gather(ctypes.byref(args), ctypes.byref(gather), stream_ptr),
                       "pa_decode_gather")
        elif cascade:
            groups = prefix_groups.to_args()
            _lib.check(lib.pa_decode_cascade(ctypes.byref(args), ctypes.byref(groups), stream_ptr),
                       "pa_decode_cascade")
        else:
            rc = lib.pa_decode(ctypes.byref(args), stream_ptr)
            if rc == _lib.PA_ERR_UNSUPPORTED and B > 1 and _BATCH_LIMIT_TEXT in _lib.last_error():
                # More sequences than the kernel's shared-memory tables hold:
                # the rows are independent, so attend the two halves one after
                # the other (the append above already covered every row).
                half = B // 2
                for lo, hi in ((0, half), (half, B)):
                    paged_attention_decode(query[lo:hi], key_cache, value_cache, block_tables[lo:hi],
                                           context_lens[lo:hi], scale, out=out[lo:hi],
                                           context_lens_include_new=context_lens_include_new,
                                           workspace=workspace, validate=False)
            else:
                _lib.check(rc, "pa_decode")
    if deferred:
        _copy_after_call(workspace, stream_ptr, tag, speeds)
    elif validate if validate is not None else _VALIDATE_DEFAULT:
        flags = read_device_errors(workspace=workspace)
        if flags:
            raise device_error(flags)
    return out
