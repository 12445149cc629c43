"""Cascade decoding over shared prompt prefixes (pa_decode_cascade): rows whose
block tables start with the same physical blocks attend those blocks once per
group.  The result must match the oracle (the reference's per-row algorithm,
which attends every member's prefix separately) and the plain call."""

from __future__ import annotations

import pytest
import torch

from _util import excess_err, max_err, oracle_rows
from llm_serving_runtime_b200 import PrefixGroups, find_shared_prefixes, paged_attention_decode
from llm_serving_runtime_b200.paged_attention import DeviceErrorFlags, read_device_errors
from llm_serving_runtime_b200.workloads import make_workload
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _shared_batch(groups, prefix_lens, lone, cached, Hq, Hkv, D, bs, dtype, q_len, seed):
    """A batch whose groups share their first prefix_lens[g] tokens (whole
    blocks) through the same physical blocks; rows are numbered in a shuffled
    order so members are not adjacent.  ``cached[i]`` = tokens cached before the
    step for the i-th row in (members of group 0, group 1, ..., lone rows)."""
    g = torch.Generator().manual_seed(seed)
    n_rows = sum(groups) + lone
    perm = torch.randperm(n_rows, generator=g).tolist()
    L = [c + q_len for c in cached]
    nblk = [(x + bs - 1) // bs for x in L]
    maxb = max(nblk)
    tables = torch.zeros(n_rows, maxb, dtype=torch.int32)
    lens = torch.zeros(n_rows, dtype=torch.int32)
    next_block = 0
    members, i = [], 0
    for gi, size in enumerate(groups):
        pblk = prefix_lens[gi] // bs
        shared = torch.arange(next_block, next_block + pblk, dtype=torch.int32)
        next_block += pblk
        rows = []
        for _ in range(size):
            r = perm[i]
            assert cached[i] + q_len >= prefix_lens[gi]
            tables[r, :pblk] = shared
            n_priv = nblk[i] - pblk
            tables[r, pblk:pblk + n_priv] = torch.arange(next_block, next_block + n_priv, dtype=torch.int32)
            next_block += n_priv
            lens[r] = cached[i]
            rows.append(r)
            i += 1
        members.append(rows)
    for _ in range(lone):
        r = perm[i]
        tables[r, :nblk[i]] = torch.arange(next_block, next_block + nblk[i], dtype=torch.int32)
        next_block += nblk[i]
        lens[r] = cached[i]
        i += 1
    num_blocks = next_block + 3
    kc = (torch.randn(num_blocks, Hkv, bs, D, generator=g) * 0.5).to(dtype)
    vc = (torch.randn(num_blocks, Hkv, bs, D, generator=g) * 0.5).to(dtype)
    q = (torch.randn(n_rows, Hq, q_len, D, generator=g) * 0.5).to(dtype)
    return q, kc, vc, tables, lens, members


CASES = [
    # (groups, prefix_lens, lone, cached, Hq, Hkv, D, bs, dtype, q_len)
    ([3, 2], [320, 160], 2, [320, 400, 777, 160, 161, 50, 900], 32, 8, 128, 16, torch.bfloat16, 4),
    ([4], [200], 1, [200, 216, 233, 1000, 64], 14, 2, 64, 8, torch.float16, 1),   # prefix not a unit multiple
    ([4], [4096], 0, [4096, 4100, 5000, 4200], 32, 8, 128, 16, torch.bfloat16, 1),  # few tiles: split prefix
    ([6], [512], 0, [512] * 6, 32, 8, 128, 32, torch.bfloat16, 4),                 # suffix = new tokens only
    ([2, 2], [128, 96], 1, [128, 300, 96, 97, 10], 8, 2, 128, 16, torch.bfloat16, 1),
    ([3], [256], 0, [300, 256, 999], 64, 8, 128, 16, torch.bfloat16, 2),           # G = 8
    ([3, 2], [256, 128], 1, [256, 300, 500, 128, 200, 60], 32, 8, 80, 16, torch.bfloat16, 2),  # head_dim 80
    ([3, 2], [256, 128], 1, [256, 300, 700, 128, 200, 60], 32, 8, 128, 64, torch.bfloat16, 1),  # 64-token blocks
    ([4], [512], 0, [512, 600, 1000, 530], 32, 8, 128, 128, torch.float16, 2),  # 128-token blocks
]


@pytest.mark.parametrize("groups,prefix_lens,lone,cached,Hq,Hkv,D,bs,dtype,q_len", CASES)
def test_cascade_matches_oracle_and_plain_call(groups, prefix_lens, lone, cached, Hq, Hkv, D, bs, dtype, q_len):
    q, kc, vc, bt, cl, members = _shared_batch(groups, prefix_lens, lone, cached, Hq, Hkv, D, bs, dtype, q_len,
                                               seed=sum(cached) + D)
    pg = PrefixGroups.from_members(members, prefix_lens, q.shape[0], DEV)
    args = (q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), D ** -0.5)
    out = paged_attention_decode(*args, prefix_groups=pg, validate=True)
    plain = paged_attention_decode(*args, validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5, len_offset=q_len)
    assert excess_err(out, ref) <= 0, f"cascade max abs err {max_err(out, ref)}"
    assert excess_err(plain, ref) <= 0


def test_prefix_covering_the_whole_row():
    """q_len = 1 with the reference's lengths (which include the new token): a
    prefix that reaches the new token leaves the member no units of its own."""
    q, kc, vc, bt, cl, members = _shared_batch([3], [128], 0, [127, 127, 200], 32, 8, 128, 16, torch.bfloat16, 1,
                                               seed=5)
    seq_lens = cl + 1
    pg = PrefixGroups.from_members(members, [128], q.shape[0], DEV)
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), seq_lens.to(DEV), 128 ** -0.5,
                                 context_lens_include_new=True, prefix_groups=pg, validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, seq_lens, 128 ** -0.5, len_offset=0)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_cascade_with_append_on_prefix_workload():
    w = make_workload("cfg4-prefix-verify", device=DEV)
    pg = w.shared_prefixes()
    out = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                                 w.slot_mapping, w.new_key, w.new_value, prefix_groups=pg, validate=True)
    plain = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                                   validate=True)
    rows = list(range(w.batch))  # the whole batch: 16 groups of 32 rows, q_len 4
    ref = oracle_rows(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale, w.q_len, rows)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"
    assert (out.float() - plain.float()).abs().max().item() <= 4e-3


def test_detected_groups_match_the_workload():
    w = make_workload("cfg4-prefix-verify", device=DEV)
    found = find_shared_prefixes(w.block_tables, w.context_lens, block_size=w.key_cache.shape[2])
    given = w.shared_prefixes()
    assert found.num_groups == given.num_groups and found.max_prefix_len == given.max_prefix_len
    assert torch.equal(found.seq_group, given.seq_group)


def test_member_with_a_different_table_is_flagged():
    q, kc, vc, bt, cl, members = _shared_batch([3], [256], 0, [256, 300, 400], 32, 8, 128, 16, torch.bfloat16, 1,
                                               seed=9)
    bt[members[0][1], 3] = bt[members[0][1], 3] + 1  # one prefix block differs for the second member
    pg = PrefixGroups.from_members(members, [256], q.shape[0], DEV)
    read_device_errors(DEV)
    with pytest.raises(IndexError, match="prefix group"):
        paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 128 ** -0.5,
                               prefix_groups=pg, validate=True)
    assert read_device_errors(DEV) == 0


def test_no_groups_is_the_plain_call():
    q, kc, vc, bt, cl, _ = _shared_batch([], [], 3, [10, 500, 64], 32, 8, 128, 16, torch.bfloat16, 1, seed=2)
    pg = PrefixGroups.from_members([], [], q.shape[0], DEV)
    args = (q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 128 ** -0.5)
    assert torch.equal(paged_attention_decode(*args, prefix_groups=pg), paged_attention_decode(*args))
    assert DeviceErrorFlags.PREFIX == 0x10


def test_cascade_inside_a_cuda_graph():
    """One capture of the cascade call replays correctly after the lengths grow
    (the kernels read lengths, tables and groups on the device)."""
    from llm_serving_runtime_b200.cuda_graph import DecodeStepGraph

    q, kc, vc, bt, cl, members = _shared_batch([3, 2], [256, 128], 1, [256, 300, 500, 128, 140, 90], 32, 8, 128,
                                               16, torch.bfloat16, 1, seed=21)
    B, maxb = bt.shape
    pg = PrefixGroups.from_members(members, [256, 128], B, DEV)
    kcd, vcd = kc.to(DEV), vc.to(DEV)
    graph = DecodeStepGraph([kcd], [vcd], batch=B, max_blocks=maxb, num_q_heads=32, q_len=1, scale=128 ** -0.5,
                            prefix_groups=pg)
    for grow in (0, 5):
        lens = cl - 5 + grow
        graph.query[0].copy_(q.to(DEV))
        graph.block_tables.copy_(bt.to(DEV))
        graph.context_lens.copy_(lens.to(DEV))
        out = graph.replay()[0]
        torch.cuda.synchronize()
        ref = oracle.paged_decode(q, kc, vc, bt, lens, 128 ** -0.5, len_offset=1)
        assert excess_err(out, ref) <= 0, f"step {grow}: max abs err {max_err(out, ref)}"


def _random_cascade(seed):
    import random

    rnd = random.Random(seed)
    dtype = rnd.choice([torch.bfloat16, torch.float16])
    D = rnd.choice([64, 128, 128, 80])
    bs = rnd.choice([8, 16, 16, 32, 64, 128])
    Hkv = rnd.choice([1, 2, 8])
    G = rnd.choice([1, 4, 4, 7, 8])
    q_len = rnd.choice([1, 1, 2, 4])
    n_groups = rnd.randint(1, 5)
    groups = [rnd.randint(1, 12) for _ in range(n_groups)]
    prefix_lens = [bs * rnd.randint(1, max(1, 1536 // bs)) for _ in range(n_groups)]
    lone = rnd.randint(0, 4)
    cached = []
    for gi, size in enumerate(groups):
        for _ in range(size):
            # a member holds the whole prefix; its own part may be empty
            cached.append(prefix_lens[gi] + rnd.choice([0, 0, rnd.randint(0, bs), rnd.randint(0, 900)]))
    cached += [rnd.randint(0, 1500) for _ in range(lone)]
    return groups, prefix_lens, lone, cached, G * Hkv, Hkv, D, bs, dtype, q_len


@pytest.mark.parametrize("seed", range(80))
def test_random_cascades_vs_oracle(seed):
    """Seeded random groups (sizes, prefix lengths, members with empty or short
    own parts, lone rows) over random shapes: the cascade, with the groups given
    and with the groups found from the block tables, against the oracle."""
    groups, prefix_lens, lone, cached, Hq, Hkv, D, bs, dtype, q_len = _random_cascade(seed)
    q, kc, vc, bt, cl, members = _shared_batch(groups, prefix_lens, lone, cached, Hq, Hkv, D, bs, dtype, q_len,
                                               seed=7000 + seed)
    args = (q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), D ** -0.5)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5, len_offset=q_len)
    given = PrefixGroups.from_members(members, prefix_lens, q.shape[0], DEV)
    found = find_shared_prefixes(bt, cl, block_size=bs, min_shared_tokens=bs, device=DEV)
    for pg in (given, found):
        out = paged_attention_decode(*args, prefix_groups=pg, validate=True)
        assert excess_err(out, ref) <= 0, f"seed {seed}: max abs err {max_err(out, ref)}"
