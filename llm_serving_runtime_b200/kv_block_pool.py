"""``GpuKVBlockPool`` with its KV append on the sm_100a append kernel.

Mirrors the reference's pool (runtime/phase2/paged_kv_kernel.py:15-315): same
constructor, lazy zero-initialised growth, per-layer views, statistics and
error behaviour.  ``write_tokens_batch`` launches ``pa_kv_append`` instead of a
per-token Python loop of advanced-index assignments; ``write_tokens`` (batch 1)
delegates to it as the reference does.  The gather helpers and ``copy_blocks``
keep the reference's torch semantics (they serve prefill / prefix snapshots,
not the decode path).

``write_tokens_batch_into(pool, ...)`` is the same append as a free function
over any object with the reference pool's attributes, so the reference's own
``GpuKVBlockPool`` can be patched to it (see ``integration.install``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .paged_attention import kv_append, read_device_errors, describe_device_errors

__all__ = ["PoolShape", "GpuKVBlockPool", "write_tokens_batch_into"]


@dataclass(frozen=True)
class PoolShape:
    num_blocks: int
    block_size_tokens: int
    num_layers: int
    num_kv_heads: int
    head_dim: int


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

    Outside graph capture it keeps the reference's host checks and bookkeeping
    (paged_kv_kernel.py:199-231): block tables / positions are moved to the pool
    device, an underrun raises IndexError, touched blocks are recorded and the
    pool grows to cover them.  Under capture it only launches the kernel.
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
    block_size = pool.block_size_tokens
    pool._ensure_pools()
    capturing = _capturing(device)
    if not capturing:
        block_tables = block_tables.to(device=device, dtype=torch.int32)
        start_positions = start_positions.to(device=device, dtype=torch.int64)
        # Host bookkeeping of the reference (one synchronisation, as there).
        pos = start_positions[:, None] + torch.arange(kv_len, device=device)[None, :]
        logical = torch.div(pos, block_size, rounding_mode="floor")
        if int(logical.max().item()) >= block_tables.shape[1]:
            raise IndexError("block table underrun during batched write")
        physical = torch.gather(block_tables.to(torch.int64), 1, logical)
        pool._touch_blocks(physical.reshape(-1))
    k_pool, v_pool = pool._k_pool, pool._v_pool
    kv_append(
        key_states,
        value_states,
        k_pool[:, layer_idx],
        v_pool[:, layer_idx],
        None,
        block_tables=block_tables,
        positions=start_positions,
        validate=False,
    )


class GpuKVBlockPool:
    """Shared GPU block pool with lazy physical block allocation."""

    _POOL_GROWTH_BLOCKS = 8

    def __init__(
        self,
        *,
        num_blocks: int,
        block_size_tokens: int,
        num_layers: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: str | torch.device,
    ) -> None:
        if num_blocks <= 0 or block_size_tokens <= 0:
            raise ValueError("num_blocks and block_size_tokens must be positive")
        self.shape = PoolShape(
            num_blocks=num_blocks,
            block_size_tokens=block_size_tokens,
            num_layers=num_layers,
            num_kv_heads=num_kv_heads,
            head_dim=head_dim,
        )
        self.dtype = dtype
        self.device = torch.device(device)
        self._block_shape = (num_layers, num_kv_heads, block_size_tokens, head_dim)
        self._k_pool: torch.Tensor | None = None
        self._v_pool: torch.Tensor | None = None
        self._used_blocks: set[int] = set()
        self._peak_allocated_blocks = 0

    # ---- accounting (paged_kv_kernel.py:55-79) ----
    @property
    def block_size_tokens(self) -> int:
        return self.shape.block_size_tokens

    def allocated_block_count(self) -> int:
        return len(self._used_blocks)

    def peak_allocated_block_count(self) -> int:
        return self._peak_allocated_blocks

    def bytes_per_block(self) -> int:
        s = self.shape
        elems = s.num_layers * s.num_kv_heads * s.block_size_tokens * s.head_dim * 2
        return elems * torch.empty((), dtype=self.dtype).element_size()

    def bytes_for_blocks(self, block_count: int) -> int:
        return block_count * self.bytes_per_block()

    def peak_allocated_bytes(self) -> int:
        return self.bytes_for_blocks(self._peak_allocated_blocks)

    # ---- storage (paged_kv_kernel.py:81-134) ----
    def _ensure_pools(self) -> None:
        if self._k_pool is not None:
            return
        self._grow_pools(min(1, self.shape.num_blocks))

    def reserve(self, num_blocks: int | None = None) -> None:
        """Allocate the pool up front (e.g. before CUDA-graph capture)."""
        self._grow_pools(self.shape.num_blocks if num_blocks is None else num_blocks)

    def _grow_pools(self, min_blocks: int) -> None:
        needed = min(self.shape.num_blocks, max(min_blocks, 1))
        if self._k_pool is not None and self._k_pool.shape[0] >= needed:
            return
        if self._k_pool is None:
            target = needed
        else:
            target = min(self.shape.num_blocks, max(needed, self._k_pool.shape[0] + self._POOL_GROWTH_BLOCKS))
        shape = (target, *self._block_shape)
        k_new = torch.zeros(shape, dtype=self.dtype, device=self.device)
        v_new = torch.zeros(shape, dtype=self.dtype, device=self.device)
        if self._k_pool is not None:
            existing = self._k_pool.shape[0]
            k_new[:existing].copy_(self._k_pool)
            v_new[:existing].copy_(self._v_pool)
        self._k_pool = k_new
        self._v_pool = v_new

    def _touch_block(self, physical: int) -> None:
        if physical < 0 or physical >= self.shape.num_blocks:
            raise IndexError(f"physical block id out of range: {physical}")
        self._grow_pools(physical + 1)
        self._used_blocks.add(physical)
        self._peak_allocated_blocks = max(self._peak_allocated_blocks, len(self._used_blocks))

    def _touch_blocks(self, physical_ids: torch.Tensor) -> None:
        for physical in physical_ids.unique().tolist():
            self._touch_block(int(physical))

    def k_layer_view(self, layer_idx: int) -> torch.Tensor:
        """Per-layer K blocks: ``[num_blocks, num_kv_heads, block_size, head_dim]``."""
        self._ensure_pools()
        return self._k_pool[:, layer_idx]

    def v_layer_view(self, layer_idx: int) -> torch.Tensor:
        """Per-layer V blocks: ``[num_blocks, num_kv_heads, block_size, head_dim]``."""
        self._ensure_pools()
        return self._v_pool[:, layer_idx]

    # ---- append (paged_kv_kernel.py:136-227) ----
    def write_tokens(
        self,
        layer_idx: int,
        block_ids: list[int],
        start_pos: int,
        key_states: torch.Tensor,
        value_states: torch.Tensor,
    ) -> None:
        """Write key/value states for token positions [start_pos, start_pos + kv_len)."""
        if key_states.dim() == 3:
            key_states = key_states.unsqueeze(0)
            value_states = value_states.unsqueeze(0)
        if key_states.shape[0] != 1:
            raise ValueError("write_tokens expects a single sequence; use write_tokens_batch")
        self.write_tokens_batch(
            layer_idx,
            torch.tensor([block_ids], device=self.device, dtype=torch.int32),
            torch.tensor([start_pos], device=self.device, dtype=torch.int64),
            key_states,
            value_states,
        )

    def write_tokens_batch(
        self,
        layer_idx: int,
        block_tables: torch.Tensor,
        start_positions: torch.Tensor,
        key_states: torch.Tensor,
        value_states: torch.Tensor,
    ) -> None:
        """Vectorized KV write for batch rows.

        ``block_tables`` [B, max_blocks], ``start_positions`` [B], states [B, kv_heads, kv_len, dim].
        """
        write_tokens_batch_into(self, layer_idx, block_tables, start_positions, key_states, value_states)

    def check_device_errors(self) -> None:
        """Raise IndexError if an append recorded an invalid slot or block id."""
        flags = read_device_errors(self.device)
        if flags:
            raise IndexError(describe_device_errors(flags))

    # ---- prefix snapshots and prefill gathers (torch semantics of the reference) ----
    def copy_blocks(self, src_block_ids: list[int], dst_block_ids: list[int]) -> None:
        """Copy full physical blocks (all layers) from src ids to dst ids."""
        if len(src_block_ids) != len(dst_block_ids):
            raise ValueError(
                f"copy_blocks length mismatch: src={len(src_block_ids)} dst={len(dst_block_ids)}"
            )
        if not src_block_ids:
            return
        self._ensure_pools()
        for src, dst in zip(src_block_ids, dst_block_ids):
            if src == dst:
                continue
            self._touch_block(int(src))
            self._touch_block(int(dst))
            self._k_pool[int(dst)].copy_(self._k_pool[int(src)])
            self._v_pool[int(dst)].copy_(self._v_pool[int(src)])

    def gather_layer(self, layer_idx: int, block_ids: list[int], seq_len: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Gather K/V for attention as [batch=1, heads, seq_len, head_dim] (prefill / parity)."""
        if seq_len <= 0:
            raise ValueError("seq_len must be positive")
        bs = self.block_size_tokens
        num_logical_blocks = math.ceil(seq_len / bs)
        if num_logical_blocks > len(block_ids):
            raise IndexError("block table underrun during gather")
        self._ensure_pools()
        for physical in block_ids[:num_logical_blocks]:
            self._touch_block(int(physical))
        ids = torch.tensor(block_ids[:num_logical_blocks], device=self.device, dtype=torch.long)
        k = self._k_pool[ids, layer_idx]  # [nblk, Hkv, bs, D]
        v = self._v_pool[ids, layer_idx]
        H, D = self.shape.num_kv_heads, self.shape.head_dim
        keys = k.permute(1, 0, 2, 3).reshape(H, -1, D)[:, :seq_len].unsqueeze(0)
        values = v.permute(1, 0, 2, 3).reshape(H, -1, D)[:, :seq_len].unsqueeze(0)
        return keys, values

    def gather_layer_batch(self, layer_idx: int, block_tables: torch.Tensor, seq_lens: torch.Tensor):
        """Gather K/V for batched prefill: [B, kv_heads, max_seq, head_dim] padded."""
        batch_size = int(block_tables.shape[0])
        max_seq = int(seq_lens.max().item())
        if max_seq <= 0:
            raise ValueError("seq_len must be positive")
        keys = torch.zeros(batch_size, self.shape.num_kv_heads, max_seq, self.shape.head_dim,
                           device=self.device, dtype=self.dtype)
        values = torch.zeros_like(keys)
        for b in range(batch_size):
            seq_len = int(seq_lens[b].item())
            num_logical = math.ceil(seq_len / self.block_size_tokens)
            row_ids = [int(x) for x in block_tables[b, :num_logical].tolist()]
            k, v = self.gather_layer(layer_idx, row_ids, seq_len)
            keys[b, :, :seq_len] = k[0]
            values[b, :, :seq_len] = v[0]
        return keys, values

    def reset(self) -> None:
        self._k_pool = None
        self._v_pool = None
        self._used_blocks.clear()
        self._peak_allocated_blocks = 0
