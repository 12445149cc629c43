"""ctypes binding of ``libpa_b200.so`` (the C ABI in include/paged_attention_b200.h).

The structures below mirror the header field for field.  Loading fails loudly
(``RuntimeError``) when the library has not been built: there is no fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libpa_b200.so"

PA_OK = 0
PA_ERR_INVALID_ARGUMENT = 1
PA_ERR_UNSUPPORTED = 2
PA_ERR_WORKSPACE = 3
PA_ERR_CUDA = 4
PA_ERR_DEVICE = 5

PA_DTYPE_FLOAT32 = 0
PA_DTYPE_FLOAT16 = 1
PA_DTYPE_BFLOAT16 = 2

PA_DEVERR_BLOCK_ID_RANGE = 0x1
PA_DEVERR_TABLE_UNDERRUN = 0x2
PA_DEVERR_SLOT_RANGE = 0x4
PA_DEVERR_WAIT_TIMEOUT = 0x8
PA_DEVERR_PREFIX = 0x10
PA_DEVERR_GATHER = 0x20

PA_STATIC_WORKSPACE_BYTES = 16 << 20

EXPORTED_SYMBOLS = (
    "pa_kv_append",
    "pa_decode",
    "pa_decode_static_workspace",
    "pa_decode_cascade",
    "pa_cascade_workspace_bytes",
    "pa_decode_gather",
    "pa_ipc_export",
    "pa_ipc_import",
    "pa_ipc_release",
    "pa_decode_workspace_bytes",
    "pa_workspace_init",
    "pa_read_device_errors",
    "pa_last_error",
    "pa_last_kernel",
    "pa_version",
)

_i32, _i64, _vp, _sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t


class CacheView(ctypes.Structure):
    _fields_ = [
        ("data", _vp),
        ("num_blocks", _i64),
        ("stride_block", _i64),
        ("stride_head", _i64),
        ("stride_token", _i64),
    ]


class KvAppendArgs(ctypes.Structure):
    _fields_ = [
        ("key", _vp),
        ("key_stride_b", _i64), ("key_stride_h", _i64), ("key_stride_t", _i64),
        ("value", _vp),
        ("value_stride_b", _i64), ("value_stride_h", _i64), ("value_stride_t", _i64),
        ("key_cache", CacheView),
        ("value_cache", CacheView),
        ("slot_mapping", _vp),
        ("block_tables", _vp),
        ("block_table_stride", _i64),
        ("max_blocks", _i32),
        ("positions", _vp),
        ("positions_is_int64", _i32),
        ("position_offset", _i32),
        ("batch", _i32), ("q_len", _i32), ("num_kv_heads", _i32), ("head_dim", _i32),
        ("block_size", _i32),
        ("dtype", _i32),
        ("error_flags", _vp),
    ]


class DecodeArgs(ctypes.Structure):
    _fields_ = [
        ("query", _vp),
        ("query_stride_b", _i64), ("query_stride_h", _i64), ("query_stride_t", _i64),
        ("key_cache", CacheView),
        ("value_cache", CacheView),
        ("block_tables", _vp),
        ("block_table_stride", _i64),
        ("max_blocks", _i32),
        ("context_lens", _vp),
        ("len_offset", _i32),
        ("out", _vp),
        ("out_stride_b", _i64), ("out_stride_h", _i64), ("out_stride_t", _i64),
        ("batch", _i32), ("q_len", _i32), ("num_q_heads", _i32), ("num_kv_heads", _i32),
        ("head_dim", _i32), ("block_size", _i32),
        ("dtype", _i32),
        ("scale", ctypes.c_float),
        ("workspace", _vp),
        ("workspace_bytes", _sz),
        ("allow_overlap_with_previous", _i32),
        ("sm_weights", _vp),
        ("num_sm_weights", _i32),
        ("sm_timing_tag", ctypes.c_uint32),
    ]


class SmTiming(ctypes.Structure):
    """pa_sm_timing: one SM's share of a large decode call."""

    _fields_ = [
        ("t_start_ns", ctypes.c_uint64),
        ("t_end_ns", ctypes.c_uint64),
        ("cost", ctypes.c_uint32),
        ("smid", ctypes.c_uint32),
        ("tag", ctypes.c_uint32),
        ("pad", ctypes.c_uint32),
    ]


PA_WS_SM_TIMING_OFFSET = 256
PA_MAX_SM_WEIGHTS = 160


class PrefixGroupsArgs(ctypes.Structure):
    _fields_ = [
        ("num_groups", _i32),
        ("max_members", _i32),
        ("max_prefix_len", _i32),
        ("member_offsets", _vp),
        ("member_seqs", _vp),
        ("prefix_lens", _vp),
        ("seq_group", _vp),
    ]


PA_IPC_HANDLE_BYTES = 64


class IpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * PA_IPC_HANDLE_BYTES), ("offset", _i64)]


class GatherArgs(ctypes.Structure):
    _fields_ = [
        ("num_ranks", _i32),
        ("rank", _i32),
        ("head_offset", _i32),
        ("out_ranks", _vp),
        ("flags_ranks", _vp),
        ("epoch", _vp),
        ("done_warps", _vp),
        ("wait_ns", _i64),
    ]


_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once; raise RuntimeError when it is missing."""
    global _handle
    with _lock:
        if _handle is not None:
            return _handle
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -c \"import __graft_entry__ as g; g.build()\"` "
                "(or python llm_serving_runtime_b200/_build.py). There is no CPU fallback."
            )
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.pa_kv_append.restype = ctypes.c_int
        lib.pa_kv_append.argtypes = [ctypes.POINTER(KvAppendArgs), _vp]
        lib.pa_decode.restype = ctypes.c_int
        lib.pa_decode.argtypes = [ctypes.POINTER(DecodeArgs), _vp]
        lib.pa_decode_static_workspace.restype = ctypes.c_int
        lib.pa_decode_static_workspace.argtypes = [ctypes.POINTER(DecodeArgs), _vp]
        lib.pa_decode_cascade.restype = ctypes.c_int
        lib.pa_decode_cascade.argtypes = [ctypes.POINTER(DecodeArgs), ctypes.POINTER(PrefixGroupsArgs), _vp]
        lib.pa_cascade_workspace_bytes.restype = _sz
        lib.pa_cascade_workspace_bytes.argtypes = [_i32] * 10
        lib.pa_decode_gather.restype = ctypes.c_int
        lib.pa_decode_gather.argtypes = [ctypes.POINTER(DecodeArgs), ctypes.POINTER(GatherArgs), _vp]
        lib.pa_ipc_export.restype = ctypes.c_int
        lib.pa_ipc_export.argtypes = [_vp, ctypes.POINTER(IpcHandle)]
        lib.pa_ipc_import.restype = ctypes.c_int
        lib.pa_ipc_import.argtypes = [ctypes.POINTER(IpcHandle), ctypes.POINTER(_vp)]
        lib.pa_ipc_release.restype = ctypes.c_int
        lib.pa_ipc_release.argtypes = [_vp]
        lib.pa_decode_workspace_bytes.restype = _sz
        lib.pa_decode_workspace_bytes.argtypes = [_i32, _i32, _i32, _i32, _i32, _i32, _i32]
        lib.pa_workspace_init.restype = ctypes.c_int
        lib.pa_workspace_init.argtypes = [_vp, _sz, _vp]
        lib.pa_read_device_errors.restype = ctypes.c_int
        lib.pa_read_device_errors.argtypes = [_vp, ctypes.POINTER(ctypes.c_uint32), _i32, _vp]
        lib.pa_last_error.restype = ctypes.c_char_p
        lib.pa_last_error.argtypes = []
        lib.pa_last_kernel.restype = ctypes.c_char_p
        lib.pa_last_kernel.argtypes = []
        lib.pa_version.restype = _i32
        lib.pa_version.argtypes = []
        _handle = lib
        return lib


_cudart_handle: ctypes.CDLL | None = None
_cudart_tried = False


def cudart() -> ctypes.CDLL | None:
    """The CUDA runtime this process already uses (libcudart.so.12), for the
    few raw stream, event and copy calls of the host path (no torch wrapper
    per call); None when it cannot be loaded."""
    global _cudart_handle, _cudart_tried
    with _lock:
        if _cudart_tried:
            return _cudart_handle
        _cudart_tried = True
        try:
            rt = ctypes.CDLL("libcudart.so.12")
        except OSError:
            return None
        rt.cudaEventCreateWithFlags.argtypes = [ctypes.POINTER(_vp), ctypes.c_uint]
        rt.cudaEventRecord.argtypes = [_vp, _vp]
        rt.cudaStreamWaitEvent.argtypes = [_vp, _vp, ctypes.c_uint]
        rt.cudaMemcpyAsync.argtypes = [_vp, _vp, _sz, ctypes.c_int, _vp]
        rt.cudaEventQuery.argtypes = [_vp]
        rt.cudaEventDestroy.argtypes = [_vp]
        for f in (rt.cudaEventCreateWithFlags, rt.cudaEventRecord, rt.cudaStreamWaitEvent, rt.cudaMemcpyAsync,
                  rt.cudaEventQuery, rt.cudaEventDestroy):
            f.restype = ctypes.c_int
        _cudart_handle = rt
        return rt


def last_error() -> str:
    msg = load().pa_last_error()
    return msg.decode() if msg else ""


def last_kernel() -> str:
    """Kernel launched by the last pa_decode call on this host thread."""
    name = load().pa_last_kernel()
    return name.decode() if name else ""


def check(status: int, what: str) -> None:
    """Map a pa_status to the reference's exception types."""
    if status == PA_OK:
        return
    msg = f"{what}: {last_error()}"
    if status in (PA_ERR_INVALID_ARGUMENT, PA_ERR_UNSUPPORTED):
        raise ValueError(msg)
    if status == PA_ERR_DEVICE:
        raise IndexError(msg)
    raise RuntimeError(msg)
