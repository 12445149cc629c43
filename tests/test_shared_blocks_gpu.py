"""Zero-copy prefix blocks end to end on the GPU.

A prompt is written through the pool's append kernel, the prefix cache
snapshots its blocks by reference, later requests borrow them, one request
rewrites a cached position (copy-on-write), and one decode step with the
append runs through the cascade over the groups found from the tables.  The
output must match the oracle on the pool's contents, and the shared blocks
must be unchanged by the rewrite."""

from __future__ import annotations

import pytest
import torch

from _pool import LayeredKV
from _util import excess_err, max_err
from llm_serving_runtime_b200 import find_shared_prefixes, paged_attention_decode
from llm_serving_runtime_b200.shared_blocks import BlockRefAllocator
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_borrowed_prefix_blocks_through_the_cascade():
    bs, Hkv, Hq, D, dtype, layer = 16, 2, 16, 128, torch.bfloat16, 1
    pool = LayeredKV(96, 2, Hkv, bs, D, dtype, DEV)
    alloc = BlockRefAllocator(total_blocks=96, block_size_tokens=bs)
    g = torch.Generator().manual_seed(11)

    def rand(*shape):
        return (torch.randn(*shape, generator=g) * 0.5).to(dtype).to(DEV)

    def write(a, start, n):
        table = torch.tensor([a.block_ids], dtype=torch.int32, device=DEV)
        pool.write_tokens_batch(layer, table, torch.tensor([start], device=DEV), rand(1, Hkv, n, D),
                                rand(1, Hkv, n, D))

    prefix = 256
    w = alloc.allocate_for_tokens("w", prefix + 8)
    write(w, 0, prefix + 5)
    used = alloc.stats()["used_blocks"]
    entry = alloc.snapshot_blocks(w.block_ids[:prefix // bs])
    assert alloc.stats()["used_blocks"] == used  # the snapshot copied nothing
    alloc.free_request("w")

    suffix = [40, 0, 100, 17, 64]
    rows = []
    for i, s in enumerate(suffix):
        r = alloc.allocate_for_tokens(f"r{i}", prefix + s + 1, borrowed_block_ids=entry)
        assert r.block_ids[:len(entry)] == entry
        if s:
            write(r, prefix, s)
        rows.append(r)
    shared_k = pool.k_layer_view(layer)[entry].clone()
    shared_v = pool.v_layer_view(layer)[entry].clone()
    # row 1 rewrites its last prompt token: its copy of the last prefix block first
    (old, new), = alloc.make_writable("r1", prefix - 1, 1, pool.copy_blocks)
    assert old == entry[-1] and rows[1].block_ids[len(entry) - 1] == new
    write(rows[1], prefix - 1, 1)
    assert torch.equal(pool.k_layer_view(layer)[entry], shared_k)
    assert torch.equal(pool.v_layer_view(layer)[entry], shared_v)
    k_new = pool.k_layer_view(layer)[new]
    assert torch.equal(k_new[:, :bs - 1], shared_k[-1][:, :bs - 1])
    assert not torch.equal(k_new[:, bs - 1], shared_k[-1][:, bs - 1])

    lone = alloc.allocate_for_tokens("lone", 301)
    write(lone, 0, 300)
    allocs = rows + [lone]
    cached = [prefix + s for s in suffix] + [300]
    for a, c in zip(allocs, cached):  # the decode step's positions are private
        assert alloc.make_writable(a.request_id, c, 1, pool.copy_blocks) == []
    width = max(len(a.block_ids) for a in allocs)
    bt = torch.zeros(len(allocs), width, dtype=torch.int32)
    for i, a in enumerate(allocs):
        bt[i, :len(a.block_ids)] = torch.tensor(a.block_ids, dtype=torch.int32)
    cl = torch.tensor(cached, dtype=torch.int32)
    groups = find_shared_prefixes(bt, cl, block_size=bs, min_shared_tokens=64, device=DEV)
    # row 1's last prefix block is its own now, so the group shares one block fewer
    assert groups.num_groups == 1 and groups.prefix_lens.tolist() == [prefix - bs]
    assert groups.member_seqs.tolist() == [0, 1, 2, 3, 4]

    B = len(allocs)
    q, new_k, new_v = rand(B, Hq, 1, D), rand(B, Hkv, 1, D), rand(B, Hkv, 1, D)
    slot = torch.tensor([int(bt[i, c // bs]) * bs + c % bs for i, c in enumerate(cached)], dtype=torch.int64,
                        device=DEV)
    kc, vc = pool.k_layer_view(layer), pool.v_layer_view(layer)
    bt_d, cl_d = bt.to(DEV), cl.to(DEV)
    out = paged_attention_decode(q, kc, vc, bt_d, cl_d, D ** -0.5, slot, new_k, new_v, prefix_groups=groups,
                                 validate=True)
    plain = paged_attention_decode(q, kc, vc, bt_d, cl_d, D ** -0.5, validate=True)
    ref = oracle.paged_decode(q.cpu(), kc.cpu(), vc.cpu(), bt, cl, D ** -0.5, len_offset=1)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"
    assert excess_err(plain, ref) <= 0
    assert alloc.stats()["cow_copies_total"] == 1
