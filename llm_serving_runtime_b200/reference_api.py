"""Drop-in replacement of the reference's decode module public API.

Same names, arguments, return shapes and error behaviour as
runtime/phase2/paged_attention_triton.py, with every decode call routed to the
sm_100a kernel of ``paged_attention.paged_attention_decode``:

  PagedDecodeBatchMetadata / PagedDecodeContext       (:43-54)
  set/reset/get_paged_decode_batch_metadata,
  set/get_paged_decode_context                        (:57-75)
  triton_available                                    (:78-79)
  warmup_paged_attention_kernel                       (:118-143)
  _paged_attention_decode_batched_triton              (:460-552)
  paged_attention_decode_batched                      (:745-775)
  paged_attention_decode                              (:778-802)
  reference_sdpa_attention                            (:805-817, dense helper)

Beyond the reference: ``paged_attention_verify_batched`` attends k draft
tokens per sequence over the same paged cache in one batched call (causal over
the drafts).  The reference runs speculative verification one sequence at a
time outside the batch (worker_server.py:1522) because its batched decode
accepts only q_len = 1.

Differences on purpose: the output is a fresh tensor, never an alias of a
cached scratch buffer (the reference returns its fp32 scratch for fp32
queries, :533-535); long rows are split across the whole batch in one launch
instead of falling back to per-row launches with a host sync each (:537-552).
"""

from __future__ import annotations

import contextvars
import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.nn.functional as F

from . import _lib
from .paged_attention import paged_attention_decode as _decode

__all__ = [
    "PagedDecodeBatchMetadata",
    "PagedDecodeContext",
    "set_paged_decode_batch_metadata",
    "reset_paged_decode_batch_metadata",
    "get_paged_decode_batch_metadata",
    "set_paged_decode_context",
    "get_paged_decode_context",
    "triton_available",
    "warmup_paged_attention_kernel",
    "paged_attention_decode_batched",
    "paged_attention_decode",
    "paged_attention_verify_batched",
    "reference_sdpa_attention",
]

_decode_batch_metadata: contextvars.ContextVar[PagedDecodeBatchMetadata | None] = contextvars.ContextVar(
    "paged_decode_batch_metadata", default=None
)


@dataclass(frozen=True)
class PagedDecodeBatchMetadata:
    """Batched decode metadata passed explicitly to the kernel."""

    pool: Any  # the reference's GpuKVBlockPool, or any pool with k_layer_view / v_layer_view
    layer_idx: int
    block_tables: torch.Tensor  # [B, max_blocks] int32
    seq_lens: torch.Tensor  # [B] int32 — KV length to attend over (includes current token)


PagedDecodeContext = PagedDecodeBatchMetadata


def set_paged_decode_batch_metadata(meta: PagedDecodeBatchMetadata | None) -> contextvars.Token:
    return _decode_batch_metadata.set(meta)


def reset_paged_decode_batch_metadata(token: contextvars.Token) -> None:
    _decode_batch_metadata.reset(token)


def get_paged_decode_batch_metadata() -> PagedDecodeBatchMetadata | None:
    return _decode_batch_metadata.get()


def set_paged_decode_context(ctx: PagedDecodeBatchMetadata | None) -> None:
    _decode_batch_metadata.set(ctx)


def get_paged_decode_context() -> PagedDecodeBatchMetadata | None:
    return get_paged_decode_batch_metadata()


def triton_available() -> bool:
    """True when the fused GPU decode path is usable (the sm_100a library loads
    and CUDA is available) — the question the reference's callers ask."""
    if not torch.cuda.is_available():
        return False
    try:
        _lib.load()
    except RuntimeError:
        return False
    return True


def _paged_attention_decode_batched_triton(
    query: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    scaling: float,
    num_kv_groups: int,
) -> torch.Tensor:
    """Same contract as the reference's Triton dispatcher: query [B, heads, 1, dim],
    seq_lens including the current token; returns [B, heads, 1, dim]."""
    batch_size, num_heads, q_len, head_dim = query.shape
    if q_len != 1:
        raise ValueError("Triton paged decode expects q_len=1")
    if num_heads != num_kv_groups * k_cache.shape[1]:
        raise ValueError("num_heads must equal num_kv_groups * num_kv_heads")
    return _decode(query, k_cache, v_cache, block_tables, seq_lens, scaling,
                   context_lens_include_new=True)


def paged_attention_decode_batched(
    query: torch.Tensor,
    metadata: PagedDecodeBatchMetadata,
    num_kv_groups: int,
    scaling: float,
) -> torch.Tensor:
    """Batched decode: ``query [B, heads, 1, dim]``."""
    if query.shape[0] != metadata.block_tables.shape[0]:
        raise ValueError("query batch size must match block_tables rows")
    pool = metadata.pool
    k_layer = pool.k_layer_view(metadata.layer_idx)
    v_layer = pool.v_layer_view(metadata.layer_idx)
    if not query.is_cuda:
        raise RuntimeError("the B200 paged decode needs CUDA tensors (no CPU fallback)")
    seq_lens = metadata.seq_lens
    if seq_lens.dtype != torch.int32 or seq_lens.device != query.device:
        seq_lens = seq_lens.to(device=query.device, dtype=torch.int32)
    return _paged_attention_decode_batched_triton(
        query, k_layer, v_layer, metadata.block_tables, seq_lens, scaling, num_kv_groups
    )


def paged_attention_verify_batched(
    query: torch.Tensor,
    metadata: PagedDecodeBatchMetadata,
    num_kv_groups: int,
    scaling: float,
    prefix_groups=None,
) -> torch.Tensor:
    """Batched speculative verify: ``query [B, heads, k, dim]`` holds each
    sequence's k draft tokens, whose K/V the cache update already appended, so
    ``metadata.seq_lens`` counts them.  Draft t of row b attends positions
    0 .. seq_lens[b] - k + t.  Returns [B, heads, k, dim].  ``prefix_groups``
    (``prefix_sharing.PrefixGroups``) attends prefixes that rows share through
    the same blocks once per group."""
    if query.dim() != 4 or query.shape[0] != metadata.block_tables.shape[0]:
        raise ValueError("query must be [batch, heads, k, dim] with the batch of block_tables")
    pool = metadata.pool
    k_layer = pool.k_layer_view(metadata.layer_idx)
    v_layer = pool.v_layer_view(metadata.layer_idx)
    if query.shape[1] != num_kv_groups * k_layer.shape[1]:
        raise ValueError("num_heads must equal num_kv_groups * num_kv_heads")
    if not query.is_cuda:
        raise RuntimeError("the B200 paged decode needs CUDA tensors (no CPU fallback)")
    seq_lens = metadata.seq_lens
    if seq_lens.dtype != torch.int32 or seq_lens.device != query.device:
        seq_lens = seq_lens.to(device=query.device, dtype=torch.int32)
    return _decode(query, k_layer, v_layer, metadata.block_tables, seq_lens, scaling,
                   context_lens_include_new=True, prefix_groups=prefix_groups)


def paged_attention_decode(
    query: torch.Tensor,
    pool: Any,
    layer_idx: int,
    block_ids: list[int],
    seq_len: int,
    num_kv_groups: int,
    scaling: float,
    block_table: torch.Tensor | None = None,
) -> torch.Tensor:
    """Decode-step attention for batch=1 (back-compat wrapper)."""
    if seq_len <= 0:
        raise ValueError("seq_len must be positive for paged decode")
    num_logical = math.ceil(seq_len / pool.block_size_tokens)
    if block_table is None:
        table = torch.tensor(block_ids[:num_logical], device=query.device, dtype=torch.int32)
    else:
        table = block_table[:num_logical]
    meta = PagedDecodeBatchMetadata(
        pool=pool,
        layer_idx=layer_idx,
        block_tables=table.unsqueeze(0),
        seq_lens=torch.tensor([seq_len], device=query.device, dtype=torch.int32),
    )
    return paged_attention_decode_batched(query, meta, num_kv_groups, scaling)


def warmup_paged_attention_kernel(
    pool: Any,
    *,
    num_heads: int,
    num_kv_groups: int,
    head_dim: int,
    block_ids: list[int],
    seq_len: int = 16,
) -> None:
    """One B=1 call at backend start-up: loads the library, sizes the workspace
    and sets the kernel's shared-memory attribute before any graph capture."""
    if not triton_available():
        return
    device = pool.device
    query = torch.zeros(1, num_heads, 1, head_dim, device=device, dtype=pool.dtype)
    paged_attention_decode(
        query=query,
        pool=pool,
        layer_idx=0,
        block_ids=block_ids,
        seq_len=seq_len,
        num_kv_groups=num_kv_groups,
        scaling=head_dim**-0.5,
        block_table=torch.tensor(block_ids, device=device, dtype=torch.int32),
    )
    if device.type == "cuda":
        torch.cuda.synchronize()


def reference_sdpa_attention(
    query: torch.Tensor,
    keys: torch.Tensor,
    values: torch.Tensor,
    scaling: float,
    num_kv_groups: int,
) -> torch.Tensor:
    """Dense attention helper of the reference (used by its parity tests).
    Not on the decode path; kept so imports of the module keep working."""
    if num_kv_groups > 1:
        keys = keys.repeat_interleave(num_kv_groups, dim=1)
        values = values.repeat_interleave(num_kv_groups, dim=1)
    attn = torch.matmul(query, keys.transpose(2, 3)) * scaling
    attn = F.softmax(attn, dim=-1, dtype=torch.float32).to(query.dtype)
    return torch.matmul(attn, values)
