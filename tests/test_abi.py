"""The C ABI: the library loads, exports exactly what include/*.h declares, the
ctypes mirror has the header's layout, and argument errors are reported
without touching a GPU."""

from __future__ import annotations

import ctypes
import re
import subprocess

import pytest

from conftest import REPO
from llm_serving_runtime_b200 import _lib

HEADER = REPO / "include" / "paged_attention_b200.h"


def _declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"PA_API\s+[\w\s\*]+?\b(pa_\w+)\s*\(", text))


def test_header_declares_the_exported_symbols():
    assert _declared_functions() == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in _declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}
    assert exported == _declared_functions()


def test_header_constants_match_the_binding():
    text = HEADER.read_text()
    defines = dict(re.findall(r"#define (PA_DEVERR_\w+) (0x[0-9a-fA-F]+)u", text))
    assert defines, "no PA_DEVERR_ bits found"
    for name, value in defines.items():
        assert getattr(_lib, name) == int(value, 16), name
    statuses = dict(re.findall(r"(PA_(?:OK|ERR_\w+)) = (\d+)", text))
    for name, value in statuses.items():
        assert getattr(_lib, name) == int(value), name


def test_version():
    assert _lib.load().pa_version() == 10000


_LAYOUT_PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "paged_attention_b200.h"
#define F(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("pa_cache_view %zu\n", sizeof(pa_cache_view));
  printf("pa_kv_append_args %zu\n", sizeof(pa_kv_append_args));
  printf("pa_decode_args %zu\n", sizeof(pa_decode_args));
  F(pa_kv_append_args, key_cache) F(pa_kv_append_args, slot_mapping) F(pa_kv_append_args, positions)
  F(pa_kv_append_args, position_offset) F(pa_kv_append_args, batch) F(pa_kv_append_args, error_flags)
  F(pa_decode_args, key_cache) F(pa_decode_args, block_tables) F(pa_decode_args, context_lens)
  F(pa_decode_args, out) F(pa_decode_args, batch) F(pa_decode_args, scale) F(pa_decode_args, workspace)
  F(pa_decode_args, workspace_bytes) F(pa_decode_args, allow_overlap_with_previous)
  F(pa_decode_args, sm_weights) F(pa_decode_args, num_sm_weights) F(pa_decode_args, sm_timing_tag)
  printf("pa_sm_timing %zu\n", sizeof(pa_sm_timing));
  F(pa_sm_timing, cost) F(pa_sm_timing, tag)
  printf("pa_prefix_groups %zu\n", sizeof(pa_prefix_groups));
  F(pa_prefix_groups, max_prefix_len) F(pa_prefix_groups, member_offsets) F(pa_prefix_groups, seq_group)
  printf("pa_gather_args %zu\n", sizeof(pa_gather_args));
  printf("pa_ipc_handle %zu\n", sizeof(pa_ipc_handle));
  F(pa_gather_args, head_offset) F(pa_gather_args, out_ranks) F(pa_gather_args, flags_ranks)
  F(pa_gather_args, done_warps) F(pa_gather_args, wait_ns) F(pa_ipc_handle, offset)
  return 0;
}
"""


def test_ctypes_structs_match_header_layout(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(_LAYOUT_PROBE)
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-I", str(REPO / "include"), str(src), "-o", str(exe)], check=True)
    lines = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    c = dict(line.rsplit(" ", 1) for line in lines if line)
    assert int(c["pa_cache_view"]) == ctypes.sizeof(_lib.CacheView)
    assert int(c["pa_kv_append_args"]) == ctypes.sizeof(_lib.KvAppendArgs)
    assert int(c["pa_decode_args"]) == ctypes.sizeof(_lib.DecodeArgs)
    assert int(c["pa_prefix_groups"]) == ctypes.sizeof(_lib.PrefixGroupsArgs)
    assert int(c["pa_gather_args"]) == ctypes.sizeof(_lib.GatherArgs)
    assert int(c["pa_ipc_handle"]) == ctypes.sizeof(_lib.IpcHandle)
    assert int(c["pa_sm_timing"]) == ctypes.sizeof(_lib.SmTiming)
    classes = {"pa_kv_append_args": _lib.KvAppendArgs, "pa_decode_args": _lib.DecodeArgs,
               "pa_sm_timing": _lib.SmTiming,
               "pa_prefix_groups": _lib.PrefixGroupsArgs, "pa_gather_args": _lib.GatherArgs,
               "pa_ipc_handle": _lib.IpcHandle}
    for key, val in c.items():
        if "." not in key:
            continue
        struct, field = key.split(".")
        cls = classes[struct]
        assert getattr(cls, field).offset == int(val), key


def test_null_arguments_are_rejected_without_a_gpu():
    lib = _lib.load()
    assert lib.pa_decode(None, None) == _lib.PA_ERR_INVALID_ARGUMENT
    assert "null" in _lib.last_error()
    assert lib.pa_kv_append(None, None) == _lib.PA_ERR_INVALID_ARGUMENT
    args = _lib.DecodeArgs()
    args.batch, args.q_len, args.num_q_heads, args.num_kv_heads = 1, 1, 6, 4
    args.head_dim, args.block_size, args.dtype = 64, 16, _lib.PA_DTYPE_BFLOAT16
    assert lib.pa_decode(ctypes.byref(args), None) == _lib.PA_ERR_INVALID_ARGUMENT
    assert "multiple" in _lib.last_error()
    args.dtype = 7
    assert lib.pa_decode(ctypes.byref(args), None) == _lib.PA_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        _lib.check(_lib.PA_ERR_UNSUPPORTED, "pa_decode")
    with pytest.raises(IndexError):
        _lib.check(_lib.PA_ERR_DEVICE, "pa_decode")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.PA_ERR_WORKSPACE, "pa_decode")


def test_cascade_argument_errors_without_a_gpu():
    lib = _lib.load()
    args = _lib.DecodeArgs()
    assert lib.pa_decode_cascade(ctypes.byref(args), None, None) == _lib.PA_ERR_INVALID_ARGUMENT
    groups = _lib.PrefixGroupsArgs()
    groups.num_groups = 2
    assert lib.pa_decode_cascade(ctypes.byref(args), ctypes.byref(groups), None) == _lib.PA_ERR_INVALID_ARGUMENT
    assert "member_offsets" in _lib.last_error()
    groups.num_groups = -1
    assert lib.pa_decode_cascade(ctypes.byref(args), ctypes.byref(groups), None) == _lib.PA_ERR_INVALID_ARGUMENT


def test_gather_argument_errors_without_a_gpu():
    lib = _lib.load()
    args = _lib.DecodeArgs()
    g = _lib.GatherArgs()
    assert lib.pa_decode_gather(ctypes.byref(args), None, None) == _lib.PA_ERR_INVALID_ARGUMENT
    g.num_ranks, g.rank = 2, 2
    assert lib.pa_decode_gather(ctypes.byref(args), ctypes.byref(g), None) == _lib.PA_ERR_INVALID_ARGUMENT
    g.rank = 1
    assert lib.pa_decode_gather(ctypes.byref(args), ctypes.byref(g), None) == _lib.PA_ERR_INVALID_ARGUMENT
    assert "out_ranks" in _lib.last_error()
    assert lib.pa_ipc_export(None, None) == _lib.PA_ERR_INVALID_ARGUMENT


def test_empty_batch_is_a_no_op():
    lib = _lib.load()
    args = _lib.DecodeArgs()
    args.batch, args.q_len, args.num_q_heads, args.num_kv_heads = 0, 1, 8, 2
    args.head_dim, args.block_size, args.dtype = 64, 16, _lib.PA_DTYPE_FLOAT16
    assert lib.pa_decode(ctypes.byref(args), None) == _lib.PA_OK
