"""Host logic of cascade decoding (no GPU): building prefix groups and finding
shared prefixes from block tables."""

from __future__ import annotations

import pytest
import torch

from llm_serving_runtime_b200.prefix_sharing import PrefixGroups, find_shared_prefixes
from llm_serving_runtime_b200.workloads import make_workload


def test_from_members_builds_the_csr_and_row_groups():
    g = PrefixGroups.from_members([[4, 0, 2], [1, 5]], [512, 256], batch=7, device="cpu")
    assert g.num_groups == 2 and g.max_members == 3 and g.max_prefix_len == 512
    assert g.member_offsets.tolist() == [0, 3, 5]
    assert g.member_seqs.tolist() == [4, 0, 2, 1, 5]
    assert g.prefix_lens.tolist() == [512, 256]
    assert g.seq_group.tolist() == [0, 1, 0, -1, 0, 1, -1]
    assert g.member_offsets.dtype == torch.int32 and g.seq_group.dtype == torch.int32


@pytest.mark.parametrize("groups,lens,err", [
    ([[0, 1], [1, 2]], [16, 16], "more than one group"),
    ([[0, 9]], [16], "outside the batch"),
    ([[]], [16], "no members"),
    ([[0, 1]], [16, 32], "one prefix length per group"),
    ([[0, 1]], [-16], "must not be negative"),
])
def test_from_members_rejects_bad_groups(groups, lens, err):
    with pytest.raises(ValueError, match=err):
        PrefixGroups.from_members(groups, lens, batch=4, device="cpu")


def test_no_groups_is_empty():
    g = PrefixGroups.from_members([], [], batch=3, device="cpu")
    assert g.num_groups == 0 and g.seq_group.tolist() == [-1, -1, -1]


def test_find_shared_prefixes_takes_the_longest_common_run():
    bs = 16
    tables = torch.tensor([
        [7, 8, 9, 10, 11, 0],    # group A: shares 7, 8, 9 with rows 2 and 4
        [20, 21, 22, 0, 0, 0],   # alone
        [7, 8, 9, 30, 31, 32],
        [40, 41, 42, 43, 0, 0],  # shares its first block with row 5 only for one block (too short)
        [7, 8, 9, 10, 50, 0],
        [40, 60, 0, 0, 0, 0],
    ], dtype=torch.int32)
    cached = torch.tensor([80, 40, 96, 60, 75, 20])  # tokens cached before the step
    g = find_shared_prefixes(tables, cached, block_size=bs, min_shared_tokens=32)
    assert g.num_groups == 1
    assert sorted(g.member_seqs.tolist()) == [0, 2, 4] and g.prefix_lens.tolist() == [3 * bs]
    assert g.seq_group.tolist() == [0, -1, 0, -1, 0, -1]
    # a shorter member caps the prefix at its own cached (whole) blocks
    cached2 = torch.tensor([80, 40, 96, 60, 35, 20])
    g2 = find_shared_prefixes(tables, cached2, block_size=bs, min_shared_tokens=16)
    assert g2.prefix_lens[g2.seq_group[0]].item() == 2 * bs
    # at a one-block threshold rows 3 and 5 (block 40) form a group too
    assert g2.num_groups == 2 and g2.seq_group[3] == g2.seq_group[5] != -1
    assert g2.prefix_lens[g2.seq_group[3]].item() == bs
    # at four blocks only rows 0 and 4 still share enough (7, 8, 9, 10)
    g3 = find_shared_prefixes(tables, cached, block_size=bs, min_shared_tokens=64)
    assert g3.num_groups == 1 and g3.member_seqs.tolist() == [0, 4] and g3.prefix_lens.tolist() == [4 * bs]
    # the threshold drops short prefixes
    assert find_shared_prefixes(tables, cached, block_size=bs, min_shared_tokens=80).num_groups == 0


def test_find_shared_prefixes_on_the_prefix_workload():
    w = make_workload("cfg4-prefix-verify", device="cpu", rows=list(range(96)), global_batch=512)
    found = find_shared_prefixes(w.block_tables, w.context_lens, block_size=w.key_cache.shape[2])
    given = w.shared_prefixes()
    assert found.num_groups == given.num_groups == 3
    assert found.prefix_lens.tolist() == given.prefix_lens.tolist() == [1024] * 3
    assert torch.equal(found.seq_group, given.seq_group)


def _table(rows_blocks, width):
    t = torch.zeros(len(rows_blocks), width, dtype=torch.int32)
    for i, r in enumerate(rows_blocks):
        t[i, :len(r)] = torch.tensor(r, dtype=torch.int32)
    return t


def test_a_row_sharing_less_does_not_shorten_the_group():
    """A prefix cache hands out entries of every depth: three rows borrowed a
    64-block entry, a fourth only its first two blocks.  The three keep their
    64 blocks; grouping by the first block alone would have given all four 2
    blocks (and, under the threshold, no group)."""
    bs = 16
    shared = list(range(64))
    rows = [shared + [100 + i] for i in range(3)] + [shared[:2] + [200, 201]]
    tables = _table(rows, 66)
    cached = torch.tensor([64 * bs + 5] * 3 + [4 * bs])
    g = find_shared_prefixes(tables, cached, block_size=bs)
    assert g.num_groups == 1 and g.member_seqs.tolist() == [0, 1, 2] and g.prefix_lens.tolist() == [64 * bs]


def test_rows_left_by_a_deep_group_join_a_shallow_one():
    """Rows a, b share 100 blocks; c, d share 11; e, f only the first 10 with
    all of them.  Best: {a, b} at 100 and {c, d, e, f} at 10 (1x100 + 3x10),
    not {c, d} at 11 (1x11) beside {a, b}, nor all six at 10 (5x10)."""
    bs = 1
    base = list(range(10))
    ab = base + list(range(1000, 1090))
    rows = [ab + [5000], ab + [5001], base + [300, 301], base + [300, 302], base + [400], base + [500]]
    tables = _table(rows, 101)
    cached = torch.tensor([101, 101, 12, 12, 11, 11])
    g = find_shared_prefixes(tables, cached, block_size=bs, min_shared_tokens=1)
    got = sorted((g.prefix_lens[g.seq_group[m[0]]].item(), m) for m in
                 ([r for r in range(6) if g.seq_group[r] == k] for k in range(g.num_groups)))
    assert got == [(10, [2, 3, 4, 5]), (100, [0, 1])]


def _brute_force_value(tables, full, bs, min_tokens, min_members):
    def partitions(items):
        if not items:
            yield []
            return
        first, rest = items[0], items[1:]
        for p in partitions(rest):
            for i in range(len(p)):
                yield p[:i] + [[first] + p[i]] + p[i + 1:]
            yield [[first]] + p

    def lcp(rows):
        lim = min(full[r] for r in rows)
        d = 0
        while d < lim and all(tables[r, d] == tables[rows[0], d] for r in rows):
            d += 1
        return d

    best = 0
    for part in partitions(list(range(tables.shape[0]))):
        v = 0
        for grp in part:
            d = lcp(grp) if len(grp) > 1 else 0
            if len(grp) >= min_members and d * bs >= min_tokens:
                v += (len(grp) - 1) * d * bs
        best = max(best, v)
    return best


def test_grouping_is_optimal_on_small_random_tries():
    """Against every partition of the rows, on seeded random tables whose rows
    copy leading blocks from earlier rows (nested prefixes of many depths)."""
    import random

    import numpy as np

    rng = random.Random(11)
    for _ in range(250):
        B, W, bs = rng.randint(2, 6), 6, 16
        tables = np.zeros((B, W), dtype=np.int64)
        nxt = 1
        for r in range(B):
            k = rng.randint(1, W) if r and rng.random() < 0.8 else 0
            if k:
                tables[r, :k] = tables[rng.randrange(r), :k]
            tables[r, k:] = np.arange(nxt, nxt + W - k)
            nxt += W - k
        full = np.array([rng.randint(0, W) for _ in range(B)])
        min_tokens, min_members = rng.choice([16, 32, 48]), rng.choice([2, 2, 3])
        g = find_shared_prefixes(torch.tensor(tables), torch.tensor(full * bs + rng.randint(0, bs - 1)),
                                 block_size=bs, min_shared_tokens=min_tokens, min_members=min_members)
        value = 0
        for k in range(g.num_groups):
            members = g.member_seqs[g.member_offsets[k]:g.member_offsets[k + 1]].tolist()
            prefix = int(g.prefix_lens[k])
            assert len(members) >= min_members and prefix >= min_tokens
            for m in members:  # every member really holds the shared blocks
                assert full[m] * bs >= prefix
                assert (tables[m, :prefix // bs] == tables[members[0], :prefix // bs]).all()
            value += (len(members) - 1) * prefix
        assert value == _brute_force_value(tables, full, bs, min_tokens, min_members)
