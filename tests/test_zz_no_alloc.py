"""pa_decode_static_workspace: the decode entry point for callers that cannot
allocate device memory (a plugin host that passes only inputs and outputs, a
serving loop whose free HBM all belongs to the KV pool).  Its scratch is a
fixed array inside the library, so it takes no workspace argument.

Called through the C ABI (ctypes).  Each call is compared with the regular
entry point pa_decode (caller-provided workspace), which launches the same
deterministic kernel, so the two must agree bit for bit; one call is also
checked against the CPU oracle.  The calls come in a row with different
shapes and dtypes, so scratch left by one call must not leak into the next.
After its first call on a device the entry point needs no free device memory
at all: a call made with all but a sliver of HBM handed to a stand-in KV pool
must succeed and leave the free memory unchanged.
Collected last on purpose; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from _util import TOL, max_err, oracle_rows
from llm_serving_runtime_b200 import _lib, paged_attention_decode
from llm_serving_runtime_b200.paged_attention import sm_speeds
from llm_serving_runtime_b200.workloads import make_workload

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
_DT = {torch.float32: _lib.PA_DTYPE_FLOAT32, torch.float16: _lib.PA_DTYPE_FLOAT16,
       torch.bfloat16: _lib.PA_DTYPE_BFLOAT16}


def _view(t):
    return _lib.CacheView(t.data_ptr(), t.shape[0], t.stride(0), t.stride(1), t.stride(2))


def _args(w, out) -> _lib.DecodeArgs:
    a = _lib.DecodeArgs()
    q = w.query
    a.query = q.data_ptr()
    a.query_stride_b, a.query_stride_h, a.query_stride_t = q.stride(0), q.stride(1), q.stride(2)
    a.key_cache, a.value_cache = _view(w.key_cache), _view(w.value_cache)
    a.block_tables = w.block_tables.data_ptr()
    a.block_table_stride = w.block_tables.stride(0)
    a.max_blocks = w.block_tables.shape[1]
    a.context_lens = w.context_lens.data_ptr()
    a.len_offset = w.q_len
    a.out = out.data_ptr()
    a.out_stride_b, a.out_stride_h, a.out_stride_t = out.stride(0), out.stride(1), out.stride(2)
    a.batch, a.q_len = q.shape[0], q.shape[2]
    a.num_q_heads, a.num_kv_heads = q.shape[1], w.key_cache.shape[1]
    a.head_dim, a.block_size = q.shape[3], w.key_cache.shape[2]
    a.dtype = _DT[q.dtype]
    a.scale = w.scale
    a.workspace = None      # ignored by the static-workspace entry point
    a.workspace_bytes = 0
    # the per-SM shares paged_attention_decode passes, so both entry points
    # split large calls the same way
    speeds = sm_speeds(DEV)
    if speeds.n:
        a.sm_weights = speeds.weights.data_ptr()
        a.num_sm_weights = speeds.n
    return a


def _static_decode(w, out=None) -> torch.Tensor:
    out = torch.empty_like(w.query) if out is None else out
    args = _args(w, out)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    rc = _lib.load().pa_decode_static_workspace(ctypes.byref(args), stream)
    assert rc == _lib.PA_OK, _lib.last_error()
    return out


def _expected(w):
    return paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)


def test_static_workspace_equals_pa_decode_on_calls_in_a_row():
    torch.cuda.set_device(DEV)
    cases = [
        make_workload("cfg3-llama3-8b", device=DEV, rows=list(range(48))),   # bf16, rows cut by the split
        make_workload("cfg5-llama3-70b", device=DEV, rows=list(range(24))),  # bf16, G = 8
        make_workload("cfg2-qwen2-0.5b", device=DEV),                        # fp16, D = 64
        make_workload("cfg1-fp32-small", device=DEV),                        # fp32 kernel
        make_workload("cfg3-llama3-8b", device=DEV, rows=list(range(100, 148))),
    ]
    for w in cases:
        expected = _expected(w)
        got = _static_decode(w)
        torch.cuda.synchronize()
        assert torch.equal(got, expected), f"{w.spec.name}: differs from pa_decode"


def test_static_workspace_against_the_oracle():
    torch.cuda.set_device(DEV)
    w = make_workload("cfg2-qwen2-0.5b", device=DEV)
    got = _static_decode(w)
    torch.cuda.synchronize()
    rows = list(range(w.batch))
    ref = oracle_rows(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale, w.q_len, rows)
    assert max_err(got, ref) <= TOL[w.query.dtype]


def test_static_workspace_needs_no_free_memory_after_its_first_call():
    torch.cuda.set_device(DEV)
    w = make_workload("cfg3-llama3-8b", device=DEV, rows=list(range(32)))
    expected = _expected(w)
    out = torch.empty_like(w.query)
    _static_decode(w, out)  # first call on this device: the library's device code and array are set up
    torch.cuda.synchronize()
    free, _ = torch.cuda.mem_get_info(DEV)
    margin = 256 << 20
    pool_stand_in = torch.empty(max(0, free - margin), dtype=torch.uint8, device=DEV) if free > margin else None
    try:
        out.zero_()
        torch.cuda.synchronize()
        before, _ = torch.cuda.mem_get_info(DEV)
        for _ in range(2):
            _static_decode(w, out)
            torch.cuda.synchronize()
            assert torch.equal(out, expected)
        after, _ = torch.cuda.mem_get_info(DEV)
        assert after == before, f"free device memory changed by {before - after} bytes"
    finally:
        del pool_stand_in
        torch.cuda.empty_cache()


def test_static_workspace_rejects_shapes_beyond_its_size():
    torch.cuda.set_device(DEV)
    # 4 query tokens x 4 query heads per KV head at head_dim 128: 16 rows of
    # partial state per warp, more scratch than the 16 MiB array holds.
    w = make_workload("cfg4-prefix-verify", device=DEV, rows=list(range(4)))
    out = torch.empty_like(w.query)
    args = _args(w, out)
    rc = _lib.load().pa_decode_static_workspace(ctypes.byref(args), torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.PA_ERR_WORKSPACE
    assert "static workspace holds" in _lib.last_error()
