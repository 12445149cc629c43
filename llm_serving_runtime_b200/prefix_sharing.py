"""Shared prompt prefixes for cascade decoding (``pa_decode_cascade``).

When a prefix cache hands several sequences the SAME physical blocks for a
common prompt prefix, instead of copying them per sequence as the reference
does on a hit (``GpuKVBlockPool.copy_blocks``, runtime/phase2/paged_kv_kernel.py:233-250,
called from worker_server.py:1266-1272 and :1446), one decode call can read each
shared block once per group instead of once per member:

    groups = find_shared_prefixes(block_tables, context_lens, block_size=16)
    out = paged_attention_decode(query, k_cache, v_cache, block_tables,
                                 context_lens, scale, prefix_groups=groups)

``PrefixGroups`` holds the group description the C ABI takes (``pa_prefix_groups``):
member rows per group (CSR), each group's shared-prefix length in tokens, the
group of every batch row (-1: none) and two host bounds that size the launch.
Build it once per batch composition (when sequences join or leave), not per
step: the tensors stay valid while the tables grow, so one CUDA graph can
replay it.  The result equals the plain call's; the kernels flag a member whose
table does not match its group's in the prefix (``PA_DEVERR_PREFIX``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

__all__ = ["PrefixGroups", "find_shared_prefixes"]


@dataclass
class PrefixGroups:
    member_offsets: torch.Tensor  # int32 [num_groups + 1]
    member_seqs: torch.Tensor     # int32 [members]
    prefix_lens: torch.Tensor     # int32 [num_groups], tokens
    seq_group: torch.Tensor       # int32 [batch], -1 for rows in no group
    max_members: int
    max_prefix_len: int

    @property
    def num_groups(self) -> int:
        return int(self.member_offsets.numel()) - 1

    @classmethod
    def from_members(cls, groups: list[list[int]], prefix_lens: list[int], batch: int,
                     device: torch.device | str) -> "PrefixGroups":
        """Groups given as lists of batch rows plus each group's shared token count."""
        if len(groups) != len(prefix_lens):
            raise ValueError("one prefix length per group")
        seq_group = np.full(batch, -1, dtype=np.int32)
        offsets = [0]
        members: list[int] = []
        for gi, rows in enumerate(groups):
            if not rows:
                raise ValueError(f"group {gi} has no members")
            for r in rows:
                if not 0 <= r < batch:
                    raise ValueError(f"group {gi}: row {r} outside the batch")
                if seq_group[r] != -1:
                    raise ValueError(f"row {r} is in more than one group")
                seq_group[r] = gi
            members.extend(rows)
            offsets.append(len(members))
        if any(int(p) < 0 for p in prefix_lens):
            raise ValueError("prefix lengths must not be negative")
        dev = torch.device(device)

        def t(a):
            return torch.as_tensor(np.asarray(a, dtype=np.int32)).to(dev)

        return cls(
            member_offsets=t(offsets), member_seqs=t(members if members else [0]),
            prefix_lens=t(list(prefix_lens) if prefix_lens else [0]), seq_group=t(seq_group),
            max_members=max((len(g) for g in groups), default=1),
            max_prefix_len=max((int(p) for p in prefix_lens), default=0),
        )

    def to_args(self) -> _lib.PrefixGroupsArgs:
        a = _lib.PrefixGroupsArgs()
        a.num_groups = self.num_groups
        a.max_members = int(self.max_members)
        a.max_prefix_len = int(self.max_prefix_len)
        a.member_offsets = self.member_offsets.data_ptr()
        a.member_seqs = self.member_seqs.data_ptr()
        a.prefix_lens = self.prefix_lens.data_ptr()
        a.seq_group = self.seq_group.data_ptr()
        return a


def find_shared_prefixes(block_tables, cached_lens, *, block_size: int, min_shared_tokens: int = 256,
                         min_members: int = 2, device: torch.device | str | None = None) -> PrefixGroups:
    """Group rows whose block tables start with the same physical blocks.

    ``cached_lens`` counts each row's tokens cached before the step (the
    north-star ``context_lens``): only those can be shared.  Rows are grouped by
    their first block id; a group's prefix is the longest run of leading blocks
    common to all its members, capped by the shortest member's cached tokens.
    Groups sharing fewer than ``min_shared_tokens`` tokens or with fewer than
    ``min_members`` rows are dropped.  Runs on the host (numpy).
    """
    if device is None:
        device = block_tables.device if isinstance(block_tables, torch.Tensor) else "cpu"
    tables = block_tables.cpu().numpy() if isinstance(block_tables, torch.Tensor) else np.asarray(block_tables)
    lens = cached_lens.cpu().numpy() if isinstance(cached_lens, torch.Tensor) else np.asarray(cached_lens)
    lens = lens.reshape(-1).astype(np.int64)
    B = tables.shape[0]
    full_blocks = lens // block_size
    by_first: dict[int, list[int]] = {}
    for b in range(B):
        if full_blocks[b] > 0:
            by_first.setdefault(int(tables[b, 0]), []).append(b)
    groups, prefix = [], []
    for rows in by_first.values():
        if len(rows) < min_members:
            continue
        limit = int(min(full_blocks[r] for r in rows))
        sub = tables[rows, :limit]
        same = np.all(sub == sub[0:1], axis=0)
        n = int(limit if same.all() else np.argmin(same))
        if n * block_size < max(min_shared_tokens, 1):
            continue
        groups.append(rows)
        prefix.append(n * block_size)
    return PrefixGroups.from_members(groups, prefix, B, device)
