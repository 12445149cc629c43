"""Wire the sm_100a kernels under the reference runtime without changing it.

``install()`` replaces, inside an importable copy of the reference
(``runtime.phase2``), the decode dispatcher and the pool's batched append:

  runtime.phase2.paged_attention_triton._paged_attention_decode_batched_triton
  runtime.phase2.paged_attention_triton.paged_attention_decode_batched
  runtime.phase2.paged_attention_triton.paged_attention_decode
  runtime.phase2.paged_attention_triton.triton_available
  runtime.phase2.block_paged_attention.paged_attention_decode_batched
      (bound by name at import time, block_paged_attention.py:8-11)
  runtime.phase2.paged_kv_kernel.GpuKVBlockPool.write_tokens_batch

so the reference's scheduler, BlockPagedBatchCache.update, prefix cache and
CUDA-graph decode manager run unchanged on top.  ``uninstall()`` restores the
originals.  Nothing is imported from the reference unless ``install`` is called.

Inputs on the CPU (a query tensor, or a pool, that is not on a CUDA device) keep
the reference's own function: the sm_100a kernels serve CUDA tensors, and the
reference's CPU path is its own code, not a stand-in for them.  CUDA inputs only
ever reach the kernels, which fail loudly when the library is missing.
"""

from __future__ import annotations

import importlib
from types import ModuleType

from . import reference_api
from .kv_block_pool import write_tokens_batch_into

__all__ = ["install", "uninstall", "PATCH_POINTS"]

PATCH_POINTS = (
    ("runtime.phase2.paged_attention_triton", "_paged_attention_decode_batched_triton"),
    ("runtime.phase2.paged_attention_triton", "paged_attention_decode_batched"),
    ("runtime.phase2.paged_attention_triton", "paged_attention_decode"),
    ("runtime.phase2.paged_attention_triton", "triton_available"),
    ("runtime.phase2.block_paged_attention", "paged_attention_decode_batched"),
    ("runtime.phase2.paged_kv_kernel", "GpuKVBlockPool.write_tokens_batch"),
)

_saved: dict[tuple[str, str], object] = {}


def _replacement(module: str, name: str, original):
    if name == "GpuKVBlockPool.write_tokens_batch":
        def write_tokens_batch(self, layer_idx, block_tables, start_positions, key_states, value_states):
            if self.device.type != "cuda":
                return original(self, layer_idx, block_tables, start_positions, key_states, value_states)
            write_tokens_batch_into(self, layer_idx, block_tables, start_positions, key_states, value_states)

        write_tokens_batch.__doc__ = write_tokens_batch_into.__doc__
        return write_tokens_batch
    ours = getattr(reference_api, name)
    if name == "triton_available":
        return ours

    def by_device(*args, **kwargs):
        query = kwargs.get("query", args[0] if args else None)
        if query is not None and not query.is_cuda:
            return original(*args, **kwargs)
        return ours(*args, **kwargs)

    by_device.__name__, by_device.__doc__ = ours.__name__, ours.__doc__
    by_device.b200_impl = ours
    return by_device


def _resolve(mod: ModuleType, dotted: str):
    owner = mod
    parts = dotted.split(".")
    for p in parts[:-1]:
        owner = getattr(owner, p)
    return owner, parts[-1]


def install() -> list[str]:
    """Patch the reference modules in place; returns the patched names."""
    done = []
    for module_name, dotted in PATCH_POINTS:
        mod = importlib.import_module(module_name)
        owner, attr = _resolve(mod, dotted)
        key = (module_name, dotted)
        if key not in _saved:
            _saved[key] = getattr(owner, attr)
        setattr(owner, attr, _replacement(module_name, dotted, _saved[key]))
        done.append(f"{module_name}.{dotted}")
    return done


def uninstall() -> None:
    for (module_name, dotted), original in list(_saved.items()):
        mod = importlib.import_module(module_name)
        owner, attr = _resolve(mod, dotted)
        setattr(owner, attr, original)
        del _saved[(module_name, dotted)]
