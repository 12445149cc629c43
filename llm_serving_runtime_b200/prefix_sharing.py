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
    north-star ``context_lens``): only those can be shared, in whole blocks.
    A row belongs to at most one group (the kernels take one prefix per row),
    and a group's prefix is the run of leading blocks common to all its
    members.  Prefix caches hand out prefixes of many depths (one entry per
    cached block depth), so the rows form a trie over their leading block ids;
    ``_choose_groups`` picks the groups that save the most prefix reads,
    (members - 1) x prefix tokens summed over the groups.  Groups sharing fewer
    than ``min_shared_tokens`` tokens or with fewer than ``min_members`` rows
    are not formed.  Runs on the host (numpy), once per batch composition.
    """
    if device is None:
        device = block_tables.device if isinstance(block_tables, torch.Tensor) else "cpu"
    tables = block_tables.cpu().numpy() if isinstance(block_tables, torch.Tensor) else np.asarray(block_tables)
    lens = cached_lens.cpu().numpy() if isinstance(cached_lens, torch.Tensor) else np.asarray(cached_lens)
    tables = tables.astype(np.int64)
    lens = lens.reshape(-1).astype(np.int64)
    B = tables.shape[0]
    full_blocks = np.minimum(np.maximum(lens, 0) // block_size, tables.shape[1])
    chosen = _choose_groups(tables, full_blocks, block_size, max(int(min_shared_tokens), 1),
                            max(int(min_members), 2))
    chosen.sort(key=lambda g: g[0][0])
    return PrefixGroups.from_members([rows for rows, _ in chosen], [d * block_size for _, d in chosen], B, device)


def _choose_groups(tables: np.ndarray, full_blocks: np.ndarray, bs: int, min_tokens: int,
                   min_members: int) -> list[tuple[list[int], int]]:
    """(sorted member rows, shared blocks) of the groups that save the most
    prefix reads, sum over groups of (members - 1) x shared tokens.

    The rows form a trie over their leading block ids, built with path
    compression: a node holds the rows that share its first ``depth`` blocks,
    ``depth`` taken as far as all of them agree and all still have cached
    blocks; rows whose cached blocks end there are its enders, the others split
    into children by their next block.  A group formed at a node has that
    node's depth as its prefix.  Two groups at one node are worth less than
    their union, so a node forms at most one; every row not in a group deeper
    down may join it, and rows that join no group are worth nothing below and
    the ancestor's depth above.  So a subtree is summarised by ``f[k]``: the
    best value of its groups when exactly k of its rows stay free for an
    ancestor.  Children combine by (max, +) convolution over k, and a node
    that forms a group of j rows turns g[k + j] into f[k] plus (j - 1) x its
    prefix tokens.  Nodes whose depth is under ``min_tokens`` form no group,
    and neither do their ancestors (shallower still), so there only the
    children's best values add up.  Exact; O(rows^2) at worst, on the host.
    """
    NEG = -np.inf
    # node: [rows, depth, enders, children]; built top-down (parents first)
    nodes: list[list] = []

    def split(rows: np.ndarray, col: int, parent: int) -> None:
        keys = tables[rows, col]
        order = np.argsort(keys, kind="stable")
        rows, keys = rows[order], keys[order]
        for part in np.split(rows, np.flatnonzero(np.diff(keys)) + 1):
            nodes.append([part, col + 1, None, []])  # the part shares blocks [0, col]
            nodes[parent][3].append(len(nodes) - 1)

    root_rows = np.flatnonzero(full_blocks > 0)
    nodes.append([root_rows, 0, np.empty(0, dtype=np.int64), []])
    if root_rows.size:
        split(root_rows, 0, 0)
    i = 0
    while i + 1 < len(nodes):  # ``nodes`` grows while this runs
        i += 1
        rows, start = nodes[i][0], nodes[i][1]
        if rows.size == 1:
            nodes[i][2] = rows
            continue
        limit = int(full_blocks[rows].min())
        sub = tables[rows, start:limit]
        same = np.all(sub == sub[0:1], axis=0)
        depth = start + (int(same.size) if same.all() else int(np.argmin(same)))
        nodes[i][1] = depth
        nodes[i][2] = rows[full_blocks[rows] == depth]
        cont = rows[full_blocks[rows] > depth]
        if cont.size:
            split(cont, depth, i)

    def formable(i: int) -> bool:
        return i > 0 and nodes[i][0].size > 1 and nodes[i][1] * bs >= min_tokens

    # bottom-up: f per formable node, with what backtracking needs
    f_of: dict[int, np.ndarray] = {}
    steps_of: dict[int, list] = {}    # per merge: (length before, argmax split per k)
    join_of: dict[int, np.ndarray] = {}  # per k: rows of the group formed here (0: none)
    best_of: dict[int, float] = {}    # value of a subtree that no ancestor can use
    for i in range(len(nodes) - 1, -1, -1):
        rows, depth, enders, children = nodes[i]
        if not formable(i):
            if i > 0 and rows.size == 1:
                f_of[i] = np.array([NEG, 0.0])  # a lone row: free
                steps_of[i], join_of[i] = [], np.zeros(2, dtype=np.int64)
            best_of[i] = sum(float(f_of[c].max()) if c in f_of else best_of[c] for c in children)
            continue
        g = np.full(enders.size + 1, NEG)
        g[enders.size] = 0.0  # enders stay free unless they join here
        steps = []
        for c in children:
            fc = f_of[c]
            merged = np.full(g.size + fc.size - 1, NEG)
            arg = np.zeros(merged.size, dtype=np.int64)
            for kc in range(fc.size):  # k = k_acc + kc
                if fc[kc] == NEG:
                    continue
                cand = g + fc[kc]
                seg = merged[kc:kc + g.size]
                better = cand > seg
                seg[better] = cand[better]
                arg[kc:kc + g.size][better] = kc
            steps.append((c, arg))
            g = merged
        n = g.size - 1
        f = g.copy()
        join = np.zeros(n + 1, dtype=np.int64)
        gain = depth * bs
        for j in range(min_members, n + 1):
            cand = g[j:] + (j - 1) * gain
            better = cand > f[:n + 1 - j]
            f[:n + 1 - j][better] = cand[better]
            join[:n + 1 - j][better] = j
        f_of[i], steps_of[i], join_of[i] = f, steps, join

    # top-down: how many free rows each node hands up, and the groups formed
    want: dict[int, int] = {}
    for i in range(len(nodes)):
        if i in f_of and i not in want:  # a formable subtree under a non-formable parent
            want[i] = int(np.argmax(f_of[i]))
        if not formable(i):
            continue
        k = want[i] + int(join_of[i][want[i]])
        for c, arg in reversed(steps_of[i]):
            kc = int(arg[k])
            want[c] = kc
            k -= kc
    groups: list[tuple[list[int], int]] = []
    free_of: dict[int, list[int]] = {}
    for i in range(len(nodes) - 1, 0, -1):
        rows, depth, enders, children = nodes[i]
        free = [int(r) for r in enders] + [r for c in children for r in free_of.pop(c, [])]
        if formable(i):
            j = int(join_of[i][want[i]])
            if j:
                groups.append((sorted(free[:j]), depth))
                free = free[j:]
        free_of[i] = free
    return groups
