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
    # the threshold drops short prefixes
    assert find_shared_prefixes(tables, cached, block_size=bs, min_shared_tokens=64).num_groups == 0


def test_find_shared_prefixes_on_the_prefix_workload():
    w = make_workload("cfg4-prefix-verify", device="cpu", rows=list(range(96)), global_batch=512)
    found = find_shared_prefixes(w.block_tables, w.context_lens, block_size=w.key_cache.shape[2])
    given = w.shared_prefixes()
    assert found.num_groups == given.num_groups == 3
    assert found.prefix_lens.tolist() == given.prefix_lens.tolist() == [1024] * 3
    assert torch.equal(found.seq_group, given.seq_group)
