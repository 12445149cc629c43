"""A minimal paged KV store for the GPU tests.

Holds K and V as [num_blocks, num_layers, kv_heads, block_size, head_dim]
tensors, allocated whole up front, and offers the surface the decode path reads
from a pool: ``device``, ``dtype``, ``block_size_tokens`` and the per-layer
views ``k_layer_view`` / ``v_layer_view``.  Its ``write_tokens_batch`` is the
library's append (``kv_block_pool.write_tokens_batch_into``); ``copy_blocks``
copies whole blocks for copy-on-write.  It keeps no block bookkeeping: the
tests that need the reference's pool use the reference's own class.
"""

from __future__ import annotations

import torch

from llm_serving_runtime_b200.kv_block_pool import write_tokens_batch_into


class LayeredKV:
    def __init__(self, num_blocks: int, num_layers: int, num_kv_heads: int, block_size: int, head_dim: int,
                 dtype: torch.dtype, device):
        shape = (num_blocks, num_layers, num_kv_heads, block_size, head_dim)
        self.device = torch.device(device)
        self.dtype = dtype
        self.block_size_tokens = block_size
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)

    def k_layer_view(self, layer: int) -> torch.Tensor:
        return self.k[:, layer]

    def v_layer_view(self, layer: int) -> torch.Tensor:
        return self.v[:, layer]

    def write_tokens_batch(self, layer_idx, block_tables, start_positions, key_states, value_states) -> None:
        write_tokens_batch_into(self, layer_idx, block_tables, start_positions, key_states, value_states)

    def copy_blocks(self, src_ids, dst_ids) -> None:
        """Whole blocks (every layer), the copy a copy-on-write needs."""
        if len(src_ids) != len(dst_ids):
            raise ValueError("copy_blocks needs as many destinations as sources")
        if not src_ids:
            return
        src = torch.as_tensor(list(src_ids), dtype=torch.long, device=self.device)
        dst = torch.as_tensor(list(dst_ids), dtype=torch.long, device=self.device)
        self.k[dst] = self.k[src]
        self.v[dst] = self.v[src]
