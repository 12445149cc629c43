"""The KV-cache append of a block pool, on the sm_100a append kernel.

``write_tokens_batch_into(pool, layer_idx, block_tables, start_positions,
key_states, value_states)`` has the contract of the reference's
``GpuKVBlockPool.write_tokens_batch`` (runtime/phase2/paged_kv_kernel.py:176-227):
row b's token t lands in block ``block_tables[b, p // bs]`` at offset ``p % bs``,
with ``p = start_positions[b] + t``, in layer ``layer_idx`` of the pool.  One
``pa_kv_append`` launch moves every row instead of a Python loop of indexed
assignments per token.

The pool is any object with the reference pool's public surface: ``device``,
``block_size_tokens`` and the per-layer views ``k_layer_view(l)`` /
``v_layer_view(l)`` ([num_blocks, kv_heads, block_size, head_dim], strided
views of the pool are fine).  ``integration.install()`` binds this function as
the reference pool's ``write_tokens_batch``; a pool that records the blocks it
hands out and grows on first touch (the reference's ``_touch_blocks``,
paged_kv_kernel.py:117-122, :229-231) has that hook called before the views are
taken, so a grown pool is written in place.
"""

from __future__ import annotations

import torch

from .paged_attention import kv_append

__all__ = ["write_tokens_batch_into"]


def _capturing(device: torch.device) -> bool:
    return bool(device.type == "cuda" and torch.cuda.is_available() and torch.cuda.is_current_stream_capturing())


def write_tokens_batch_into(
    pool,
    layer_idx: int,
    block_tables: torch.Tensor,
    start_positions: torch.Tensor,
    key_states: torch.Tensor,
    value_states: torch.Tensor,
) -> None:
    """Batched KV write: states [B, kv_heads, kv_len, dim] at positions
    start_positions[b] + t through block_tables [B, max_blocks].

    Outside graph capture the reference's host checks stay (paged_kv_kernel.py:
    199-227): tables and positions move to the pool's device, a table too short
    for the positions raises IndexError, and the pool's block bookkeeping (when
    it has one) sees the touched blocks.  Under capture only the kernel runs,
    as in the reference's capture branch.
    """
    if key_states.shape != value_states.shape:
        raise ValueError("key_states and value_states must match shape")
    batch_size = int(key_states.shape[0])
    kv_len = int(key_states.shape[-2])
    if block_tables.shape[0] != batch_size or start_positions.shape[0] != batch_size:
        raise ValueError("batch dimension mismatch in write_tokens_batch")
    device = pool.device
    if device.type != "cuda":
        raise RuntimeError("the B200 paged KV append needs a CUDA pool (no CPU fallback)")
    if not _capturing(device):
        block_tables = block_tables.to(device=device, dtype=torch.int32)
        start_positions = start_positions.to(device=device, dtype=torch.int64)
        # the last position each row writes decides the underrun, as in the
        # reference's per-token check; one host synchronisation, as there
        if kv_len == 0:
            return
        bs = pool.block_size_tokens
        first = torch.div(start_positions, bs, rounding_mode="floor")
        logical_last = torch.div(start_positions + (kv_len - 1), bs, rounding_mode="floor")
        top, span = torch.stack([logical_last.max(), (logical_last - first).max()]).tolist()
        if top >= block_tables.shape[1]:
            raise IndexError("block table underrun during batched write")
        touch = getattr(pool, "_touch_blocks", None)
        if touch is not None:
            logical = (first[:, None] + torch.arange(span + 1, device=device)[None, :]).clamp_max(logical_last[:, None])
            touch(torch.gather(block_tables.to(torch.int64), 1, logical).reshape(-1))
    kv_append(
        key_states,
        value_states,
        pool.k_layer_view(layer_idx),
        pool.v_layer_view(layer_idx),
        None,
        block_tables=block_tables,
        positions=start_positions,
    )
