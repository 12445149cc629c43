"""Transformers attention hook for a block-paged cache, on the sm_100a decode kernel.

Mirrors runtime/phase2/block_paged_attention.py:14-60: with batch metadata
published by the cache's ``update`` and a single query token, attention runs in
the fused paged decode kernel; otherwise (prefill, q_len > 1 without metadata)
it is eager masked attention over the K/V the cache returned.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .reference_api import get_paged_decode_batch_metadata, paged_attention_decode_batched

__all__ = ["repeat_kv", "block_paged_attention_forward"]


def repeat_kv(hidden_states: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return hidden_states
    batch, num_key_value_heads, slen, head_dim = hidden_states.shape
    hidden_states = hidden_states[:, :, None, :, :].expand(batch, num_key_value_heads, n_rep, slen, head_dim)
    return hidden_states.reshape(batch, num_key_value_heads * n_rep, slen, head_dim)


def block_paged_attention_forward(
    module,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attention_mask: torch.Tensor | None,
    scaling: float,
    dropout: float = 0.0,
    **kwargs,
):
    """Fused paged decode when q_len=1 (returns [B, q, heads, dim], None), else eager."""
    num_kv_groups = getattr(module, "num_key_value_groups", 1)
    meta = get_paged_decode_batch_metadata()
    if meta is not None and query.shape[-2] == 1 and query.is_cuda:
        attn_output = paged_attention_decode_batched(
            query=query,
            metadata=meta,
            num_kv_groups=num_kv_groups,
            scaling=scaling,
        )
        return attn_output.transpose(1, 2).contiguous(), None

    key_states = repeat_kv(key, num_kv_groups)
    value_states = repeat_kv(value, num_kv_groups)
    attn_weights = torch.matmul(query, key_states.transpose(2, 3)) * scaling
    if attention_mask is not None:
        attn_weights = attn_weights + attention_mask
    attn_weights = F.softmax(attn_weights, dim=-1, dtype=torch.float32).to(query.dtype)
    if dropout > 0.0 and getattr(module, "training", False):
        attn_weights = F.dropout(attn_weights, p=dropout)
    attn_output = torch.matmul(attn_weights, value_states)
    return attn_output.transpose(1, 2).contiguous(), attn_weights
