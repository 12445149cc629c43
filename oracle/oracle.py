"""CPU oracle for the paged-attention decode path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` import this module, and only as the checker /
the reported CPU baseline.  The product (``llm_serving_runtime_b200``) never
imports it and has no CPU fallback.

Contents
  * ``paged_decode``   — ctypes front end of ``pa_oracle.c``: the reference's
    per-row CPU decode (runtime/phase2/paged_attention_triton.py:663-704),
    extended causally to q_len > 1 (runtime/phase2/block_paged_attention.py:50-59).
  * ``kv_append``      — the slot-mapping scatter, restated with numpy on raw
    element bits (bit-exact by construction).
  * ``write_tokens_batch`` — the reference's batched append
    (runtime/phase2/paged_kv_kernel.py:176-227) on a 5-D pool, numpy.
  * ``slot_mapping_from_tables`` — slot = table[b, p // bs] * bs + p % bs, the
    integer math of paged_kv_kernel.py:217-223.

Parity of this oracle is pinned against the reference itself: the fixtures in
``tests/golden/`` were produced by importing the reference
(``tests/golden/make_golden.py``) and ``tests/test_oracle_golden.py`` checks
this module against every one of them.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from pathlib import Path

import numpy as np
import torch

ORACLE_DIR = Path(__file__).resolve().parent
_SRC = ORACLE_DIR / "pa_oracle.c"
_LIB = ORACLE_DIR / "_build" / "libpa_oracle.so"
_lock = threading.Lock()
_lib_handle = None

_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def build_oracle(force: bool = False) -> Path:
    """Compile ``pa_oracle.c`` with gcc (-O2 -fopenmp) into ``oracle/_build``."""
    if not force and _LIB.exists() and _LIB.stat().st_mtime >= _SRC.stat().st_mtime:
        return _LIB
    _LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = _LIB.with_suffix(".so.tmp")
    cmd = ["gcc", "-O2", "-fopenmp", "-shared", "-fPIC", "-o", str(tmp), str(_SRC), "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{proc.stderr}")
    os.replace(tmp, _LIB)
    return _LIB


def _lib():
    global _lib_handle
    with _lock:
        if _lib_handle is None:
            lib = ctypes.CDLL(str(build_oracle()))
            i64, i32 = ctypes.c_int64, ctypes.c_int32
            vp = ctypes.c_void_p
            lib.oracle_paged_decode.restype = ctypes.c_int
            lib.oracle_paged_decode.argtypes = [
                vp, i64, i64, i64,          # query + strides
                vp, vp, i64, i64, i64, i64,  # caches, num_blocks, strides
                vp, i64, i32,               # block tables, stride, max_blocks
                vp, i32,                    # context_lens, len_offset
                vp,                         # out (fp32)
                i32, i32, i32, i32, i32, i32, i32,  # B, q_len, Hq, Hkv, D, bs, dtype
                ctypes.c_float, i32,        # scaling, threads
            ]
            _lib_handle = lib
        return _lib_handle


def paged_decode(
    query: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    context_lens: torch.Tensor,
    scale: float,
    *,
    len_offset: int | None = None,
    num_threads: int = 0,
) -> torch.Tensor:
    """fp32 decode output [B, Hq, q_len, D] for CPU tensors.

    ``context_lens[b] + len_offset`` tokens are attended (default
    ``len_offset = q_len``: context_lens counts tokens cached before the step).
    The caller casts to the query dtype, as the reference does at :703.
    """
    for t in (query, key_cache, value_cache, block_tables, context_lens):
        if t.device.type != "cpu":
            raise ValueError("oracle inputs must be CPU tensors")
    if key_cache.stride() != value_cache.stride() or key_cache.shape != value_cache.shape:
        raise ValueError("oracle expects key and value caches with one layout")
    if query.dtype != key_cache.dtype:
        raise ValueError("query and cache dtypes differ")
    B, Hq, q_len, D = query.shape
    nb, Hkv, bs, D2 = key_cache.shape
    if D2 != D or query.stride(3) != 1 or key_cache.stride(3) != 1:
        raise ValueError("head_dim mismatch or non-unit innermost stride")
    bt = block_tables.to(torch.int32)
    lens = context_lens.to(torch.int32).contiguous()
    out = torch.empty(B, Hq, q_len, D, dtype=torch.float32)
    off = q_len if len_offset is None else int(len_offset)
    rc = _lib().oracle_paged_decode(
        query.data_ptr(), query.stride(0), query.stride(1), query.stride(2),
        key_cache.data_ptr(), value_cache.data_ptr(), nb,
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        bt.data_ptr(), bt.stride(0), bt.shape[1],
        lens.data_ptr(), off,
        out.data_ptr(),
        B, q_len, Hq, Hkv, D, bs, _DTYPE_CODE[query.dtype],
        float(scale), int(num_threads),
    )
    if rc != 0:
        raise IndexError("block id out of range or block table underrun")
    return out


def _bits(t: torch.Tensor) -> np.ndarray:
    """Raw element bits of a CPU tensor as a numpy view (no copy)."""
    view_dtype = {2: torch.int16, 4: torch.int32}[t.element_size()]
    return t.view(view_dtype).numpy()


def slot_mapping_from_tables(
    block_tables: torch.Tensor, positions: torch.Tensor, q_len: int, block_size: int
) -> torch.Tensor:
    """slot[b*q_len + t] = table[b, p // bs] * bs + p % bs with p = positions[b] + t."""
    bt = block_tables.to(torch.int64).numpy()
    pos = positions.to(torch.int64).numpy()[:, None] + np.arange(q_len)[None, :]
    lb = pos // block_size
    if (lb >= bt.shape[1]).any():
        raise IndexError("block table underrun")
    phys = np.take_along_axis(bt, lb, axis=1)
    return torch.from_numpy((phys * block_size + pos % block_size).reshape(-1).copy())


def kv_append(
    key: torch.Tensor,
    value: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """In place: cache[slot // bs, h, slot % bs, :] = new[b, h, t, :] (bit copy).

    ``key``/``value`` are [B, Hkv, q_len, D]; slot i = b * q_len + t; a negative
    slot is a padding token and is skipped.
    """
    B, Hkv, q_len, D = key.shape
    bs = key_cache.shape[2]
    slots = slot_mapping.to(torch.int64).numpy().reshape(B, q_len)
    kc, vc = _bits(key_cache), _bits(value_cache)
    kn, vn = _bits(key), _bits(value)
    for b in range(B):
        for t in range(q_len):
            s = int(slots[b, t])
            if s < 0:
                continue
            blk, off = divmod(s, bs)
            if blk >= kc.shape[0]:
                raise IndexError(f"slot {s} outside the pool")
            kc[blk, :, off, :] = kn[b, :, t, :]
            vc[blk, :, off, :] = vn[b, :, t, :]


def write_tokens_batch(
    k_pool: torch.Tensor,
    v_pool: torch.Tensor,
    layer_idx: int,
    block_tables: torch.Tensor,
    start_positions: torch.Tensor,
    key_states: torch.Tensor,
    value_states: torch.Tensor,
) -> None:
    """The reference's batched append on 5-D pools [num_blocks, L, Hkv, bs, D].

    For t in range(kv_len): pos = start + t; physical = table[row, pos // bs];
    pool[physical, layer, :, pos % bs, :] = states[:, :, t, :]
    (runtime/phase2/paged_kv_kernel.py:217-227); IndexError on underrun (:221-222).
    """
    bs = k_pool.shape[3]
    kv_len = key_states.shape[2]
    bt = block_tables.to(torch.int64).numpy()
    start = start_positions.to(torch.int64).numpy()
    kp, vp = _bits(k_pool), _bits(v_pool)
    kn, vn = _bits(key_states), _bits(value_states)
    rows = np.arange(bt.shape[0])
    for t in range(kv_len):
        pos = start + t
        logical = pos // bs
        if (logical >= bt.shape[1]).any():
            raise IndexError("block table underrun during batched write")
        physical = bt[rows, logical]
        if (physical < 0).any() or (physical >= k_pool.shape[0]).any():
            raise IndexError("physical block id out of range")
        offset = pos % bs
        for r in range(bt.shape[0]):
            kp[physical[r], layer_idx, :, offset[r], :] = kn[r, :, t, :]
            vp[physical[r], layer_idx, :, offset[r], :] = vn[r, :, t, :]
