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
CUDA-graph decode manager run unchanged on top.

Multi-token steps (chunked or batched prefill, speculative verify) also stay on
the paged cache (``multi_query=True``, the default).  The reference's cache
layers gather every row's K/V into a dense padded tensor for such steps
(paged_kv_cache.py:80-81, :168-169; paged_kv_kernel.py:252-309) and its hook
then runs eager attention over it (block_paged_attention.py:50-59).  Here:

  * ``BlockPagedLayer.update`` / ``BlockPagedBatchLayer.update`` run the
    reference's own update (the append goes to the append kernel), but the
    gather it ends with is deferred: the layer publishes a
    ``MultiQueryMetadata`` (pool, layer, block tables, lengths including the
    new tokens, q_len) and returns the step's own K/V rows;
  * the hook (``block_paged_attention_forward``, also re-registered as HF's
    ``"block_paged"`` attention when that name is registered) runs the causal
    multi-query kernels over the paged KV when the attention mask asks for
    exactly that: each new token t of row b attends positions
    0 .. L_b - q_len + t.  HF passes no mask (None) when causal attention is
    implied; a given mask is compared with that pattern once per mask tensor.
    Any other mask (padding inside a row, a custom pattern) gathers the K/V
    then and calls the reference's own hook, so those batches keep the
    reference's eager path.

``uninstall()`` restores the originals.  Nothing is imported from the reference
unless ``install`` is called.

Inputs on the CPU (a query tensor, or a pool, that is not on a CUDA device) keep
the reference's own function: the sm_100a kernels serve CUDA tensors, and the
reference's CPU path is its own code, not a stand-in for them.  CUDA inputs only
ever reach the kernels, which fail loudly when the library is missing.
"""

from __future__ import annotations

import contextvars
import importlib
import math
from dataclasses import dataclass
from types import ModuleType
from typing import Any

import torch

from . import reference_api
from .kv_block_pool import write_tokens_batch_into

__all__ = ["install", "uninstall", "PATCH_POINTS", "MULTI_QUERY_PATCH_POINTS", "MultiQueryMetadata"]

PATCH_POINTS = (
    ("runtime.phase2.paged_attention_triton", "_paged_attention_decode_batched_triton"),
    ("runtime.phase2.paged_attention_triton", "paged_attention_decode_batched"),
    ("runtime.phase2.paged_attention_triton", "paged_attention_decode"),
    ("runtime.phase2.paged_attention_triton", "triton_available"),
    ("runtime.phase2.block_paged_attention", "paged_attention_decode_batched"),
    ("runtime.phase2.paged_kv_kernel", "GpuKVBlockPool.write_tokens_batch"),
)

MULTI_QUERY_PATCH_POINTS = (
    ("runtime.phase2.paged_kv_kernel", "GpuKVBlockPool.gather_layer"),
    ("runtime.phase2.paged_kv_kernel", "GpuKVBlockPool.gather_layer_batch"),
    ("runtime.phase2.paged_kv_cache", "BlockPagedLayer.update"),
    ("runtime.phase2.paged_kv_cache", "BlockPagedBatchLayer.update"),
    ("runtime.phase2.block_paged_attention", "block_paged_attention_forward"),
)

_saved: dict[tuple[str, str], object] = {}
_saved_registration: list = []


@dataclass(frozen=True)
class MultiQueryMetadata:
    """What a cache layer publishes for a multi-token step over the paged KV."""

    pool: Any
    layer_idx: int
    block_tables: torch.Tensor  # [B, max_blocks] int32
    seq_lens: torch.Tensor      # [B] int32, including this step's q_len tokens
    q_len: int


# Set while a cache layer's own update runs: the gather it ends with records
# its arguments here instead of gathering.
_deferred_gather: contextvars.ContextVar[list | None] = contextvars.ContextVar("b200_deferred_gather",
                                                                             default=None)


def _ref(name: str) -> ModuleType:
    return importlib.import_module(f"runtime.phase2.{name}")


def _deferring_gather_layer(original):
    def gather_layer(self, layer_idx, block_ids, seq_len):
        box = _deferred_gather.get()
        if box is None:
            return original(self, layer_idx, block_ids, seq_len)
        n = math.ceil(seq_len / self.block_size_tokens)
        if n > len(block_ids):
            raise IndexError("block table underrun during gather")  # paged_kv_kernel.py:263-264
        table = torch.tensor([list(block_ids[:n])], dtype=torch.int32, device=self.device)
        lens = torch.tensor([seq_len], dtype=torch.int32, device=self.device)
        box.append((self, layer_idx, table, lens))
        return None, None

    gather_layer.__doc__ = original.__doc__
    return gather_layer


def _deferring_gather_layer_batch(original):
    def gather_layer_batch(self, layer_idx, block_tables, seq_lens):
        box = _deferred_gather.get()
        if box is None:
            return original(self, layer_idx, block_tables, seq_lens)
        box.append((self, layer_idx, block_tables, seq_lens))
        return None, None

    gather_layer_batch.__doc__ = original.__doc__
    return gather_layer_batch


def _multi_query_update(original):
    def update(self, key_states, value_states, *args, **kwargs):
        pool = getattr(self, "pool", None)
        kv_len = int(key_states.shape[-2])
        if kv_len <= 1 or pool is None or pool.device.type != "cuda" or not key_states.is_cuda:
            return original(self, key_states, value_states, *args, **kwargs)
        box: list = []
        token = _deferred_gather.set(box)
        try:
            result = original(self, key_states, value_states, *args, **kwargs)
        finally:
            _deferred_gather.reset(token)
        if not box:  # the update ended without its gather
            return result
        pool_, layer_idx, tables, lens = box[-1]
        if tables.dtype != torch.int32 or tables.device != key_states.device:
            tables = tables.to(device=key_states.device, dtype=torch.int32)
        if lens.dtype != torch.int32 or lens.device != key_states.device:
            lens = lens.to(device=key_states.device, dtype=torch.int32)
        _ref("paged_attention_triton").set_paged_decode_batch_metadata(
            MultiQueryMetadata(pool=pool_, layer_idx=layer_idx, block_tables=tables, seq_lens=lens, q_len=kv_len))
        return key_states, value_states

    update.__doc__ = original.__doc__
    return update


_mask_checks: dict[tuple, bool] = {}


def _mask_is_plain_causal(meta: MultiQueryMetadata, mask: torch.Tensor | None, module) -> bool:
    """True when ``mask`` lets new token t of row b attend exactly positions
    0 .. L_b - q_len + t of the columns it covers (what the paged kernels do)."""
    if mask is None:
        return bool(getattr(module, "is_causal", True))
    if mask.dim() != 4 or mask.shape[0] != meta.seq_lens.shape[0] or mask.shape[-2] != meta.q_len:
        return False
    key = (mask.data_ptr(), mask._version, tuple(mask.shape), mask.dtype, meta.seq_lens.data_ptr(),
           meta.seq_lens._version, meta.q_len)
    hit = _mask_checks.get(key)
    if hit is not None:
        return hit
    allowed = mask if mask.dtype == torch.bool else mask > torch.finfo(mask.dtype).min / 2
    cols = torch.arange(mask.shape[-1], device=mask.device)
    last = meta.seq_lens.to(mask.device).long()[:, None] - meta.q_len + torch.arange(meta.q_len,
                                                                                      device=mask.device)[None, :]
    want = cols[None, None, :] <= last[:, :, None]  # [B, q, cols]
    ok = bool(torch.equal(allowed, want[:, None].expand_as(allowed)))
    if len(_mask_checks) > 256:
        _mask_checks.clear()
    _mask_checks[key] = ok
    return ok


def _hook(original):
    def block_paged_attention_forward(module, query, key, value, attention_mask, scaling, dropout=0.0, **kwargs):
        meta = _ref("paged_attention_triton").get_paged_decode_batch_metadata()
        if isinstance(meta, MultiQueryMetadata) and query.is_cuda:
            if query.shape[-2] == meta.q_len and _mask_is_plain_causal(meta, attention_mask, module):
                out = reference_api.paged_attention_verify_batched(
                    query, meta, getattr(module, "num_key_value_groups", 1), scaling)
                return out.transpose(1, 2).contiguous(), None
            # any other mask: the reference's gather and its own eager attention
            key, value = meta.pool.gather_layer_batch(meta.layer_idx, meta.block_tables, meta.seq_lens)
        return original(module, query, key, value, attention_mask, scaling, dropout, **kwargs)

    block_paged_attention_forward.__doc__ = original.__doc__
    block_paged_attention_forward.b200_impl = True
    return block_paged_attention_forward


def _replacement(module: str, name: str, original):
    if name == "GpuKVBlockPool.write_tokens_batch":
        def write_tokens_batch(self, layer_idx, block_tables, start_positions, key_states, value_states):
            if self.device.type != "cuda":
                return original(self, layer_idx, block_tables, start_positions, key_states, value_states)
            write_tokens_batch_into(self, layer_idx, block_tables, start_positions, key_states, value_states)

        write_tokens_batch.__doc__ = write_tokens_batch_into.__doc__
        return write_tokens_batch
    if name == "GpuKVBlockPool.gather_layer":
        return _deferring_gather_layer(original)
    if name == "GpuKVBlockPool.gather_layer_batch":
        return _deferring_gather_layer_batch(original)
    if name.endswith(".update"):
        return _multi_query_update(original)
    if name == "block_paged_attention_forward":
        return _hook(original)
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


def _attention_registry():
    try:
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
    except Exception:  # noqa: BLE001 - transformers absent or too old: nothing registered
        return None
    return ALL_ATTENTION_FUNCTIONS


def install(multi_query: bool = True) -> list[str]:
    """Patch the reference modules in place; returns the patched names."""
    done = []
    points = PATCH_POINTS + (MULTI_QUERY_PATCH_POINTS if multi_query else ())
    for module_name, dotted in points:
        mod = importlib.import_module(module_name)
        owner, attr = _resolve(mod, dotted)
        key = (module_name, dotted)
        if key not in _saved:
            _saved[key] = getattr(owner, attr)
        setattr(owner, attr, _replacement(module_name, dotted, _saved[key]))
        done.append(f"{module_name}.{dotted}")
    if multi_query:
        registry = _attention_registry()
        if registry is not None and "block_paged" in registry:
            if not _saved_registration:
                _saved_registration.append(registry["block_paged"])
            hook = _ref("block_paged_attention").block_paged_attention_forward
            registry.register("block_paged", hook)
            done.append("transformers ALL_ATTENTION_FUNCTIONS['block_paged']")
    return done


def uninstall() -> None:
    for (module_name, dotted), original in list(_saved.items()):
        mod = importlib.import_module(module_name)
        owner, attr = _resolve(mod, dotted)
        setattr(owner, attr, original)
        del _saved[(module_name, dotted)]
    if _saved_registration:
        registry = _attention_registry()
        if registry is not None:
            registry.register("block_paged", _saved_registration[0])
        _saved_registration.clear()
    _mask_checks.clear()
