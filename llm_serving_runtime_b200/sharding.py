"""Multi-GPU layouts of the decode path (one process per GPU, torch.distributed).

Two layouts, matching how the work divides:

* Sequence sharding (independent rows).  ``shard_sequences`` gives each rank
  a greedy longest-first share of the batch, balanced by attended length, with
  prefix-sharing groups kept whole so shared blocks stay on one rank.  Each
  rank owns a pool holding only its rows' blocks and runs the decode alone —
  no collective on the data path.

* KV-head sharding (large models: few KV heads, long contexts).  Rank r holds
  KV heads [r*Hkv/N, (r+1)*Hkv/N) of every sequence and the query heads that
  read them; block tables and lengths are replicated.  ``HeadShardedDecode``
  runs the local decode and all-gathers the per-rank outputs (NCCL over
  NVLink) into the full [B, Hq, q_len, D] result.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .workloads import lpt_partition

__all__ = ["shard_sequences", "kv_head_range", "HeadShardedDecode"]


def shard_sequences(attended_lengths, world: int, group_size: int = 0) -> list[list[int]]:
    """Row ids per rank, balanced by attended tokens (greedy longest-first).

    ``group_size > 0`` keeps consecutive groups of that many rows together
    (sequences sharing prefix blocks)."""
    n = len(attended_lengths)
    groups = None
    if group_size > 0:
        groups = [list(range(i, min(i + group_size, n))) for i in range(0, n, group_size)]
    return lpt_partition(attended_lengths, world, groups=groups)


def kv_head_range(num_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """(first, count) of the KV heads rank ``rank`` owns under head sharding."""
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} KV heads do not divide over {world} ranks")
    per = num_kv_heads // world
    return rank * per, per


@dataclass
class HeadShardedDecode:
    """Decode with the KV heads split over the ranks of ``group``.

    ``decode_fn`` computes the local heads' attention (defaults to the sm_100a
    op); the per-rank outputs [B, Hq/N, q, D] are all-gathered into a
    [N, B, Hq/N, q, D] buffer and returned as a [B, Hq, q, D] tensor in the
    global head order (rank r's heads are r*Hq/N .. (r+1)*Hq/N - 1).
    """

    group: dist.ProcessGroup | None = None
    decode_fn: Callable | None = None
    _gather_buf: torch.Tensor | None = None

    def __call__(self, query, key_cache, value_cache, block_tables, context_lens, scale,
                 slot_mapping=None, key=None, value=None, **kw) -> torch.Tensor:
        fn = self.decode_fn
        if fn is None:
            from .paged_attention import paged_attention_decode as fn
        local = fn(query, key_cache, value_cache, block_tables, context_lens, scale, slot_mapping,
                   key, value, **kw)
        world = dist.get_world_size(self.group)
        B, hl, q, D = local.shape
        shape = (world * B, hl, q, D)  # rank chunks concatenated along dim 0
        if self._gather_buf is None or tuple(self._gather_buf.shape) != shape \
                or self._gather_buf.dtype != local.dtype or self._gather_buf.device != local.device:
            self._gather_buf = torch.empty(shape, dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(self._gather_buf, local.contiguous(), group=self.group)
        return self._gather_buf.view(world, B, hl, q, D).permute(1, 0, 2, 3, 4).reshape(B, world * hl, q, D)
