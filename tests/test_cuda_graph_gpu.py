"""A captured decode step replays correctly for later steps (growing lengths,
new tokens appended through slot_mapping), matching eager calls bit for bit."""

from __future__ import annotations

import pytest
import torch

from llm_serving_runtime_b200 import paged_attention_decode
from llm_serving_runtime_b200.cuda_graph import DecodeStepGraph, bucket_max_blocks
from oracle import oracle

DEV = torch.device("cuda", 0)


@pytest.mark.gpu
def test_graph_replays_consecutive_steps_like_eager():
    g = torch.Generator().manual_seed(5)
    layers, B, Hq, Hkv, D, bs = 3, 6, 32, 8, 128, 16
    ctx = torch.tensor([3, 15, 16, 200, 511, 77])
    steps = 4
    max_blocks = bucket_max_blocks(int(((ctx + steps + bs - 1) // bs).max()))
    nb = B * max_blocks
    pool_k = (torch.randn(nb, layers, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    pool_v = (torch.randn(nb, layers, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    ref_k, ref_v = pool_k.clone(), pool_v.clone()
    tables = torch.randperm(nb, generator=g)[: B * max_blocks].reshape(B, max_blocks).to(torch.int32).to(DEV)
    graph = DecodeStepGraph([pool_k[:, l] for l in range(layers)], [pool_v[:, l] for l in range(layers)],
                            batch=B, max_blocks=max_blocks, num_q_heads=Hq, scale=D ** -0.5)
    for s in range(steps):
        lens = (ctx + s).to(torch.int32).to(DEV)
        slots = oracle.slot_mapping_from_tables(tables.cpu(), lens.cpu().to(torch.int64), 1, bs).to(DEV)
        qs = [(torch.randn(B, Hq, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(layers)]
        ks = [(torch.randn(B, Hkv, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(layers)]
        vs = [(torch.randn(B, Hkv, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(layers)]
        outs = graph.step(block_tables=tables, context_lens=lens, slot_mapping=slots, queries=qs, new_keys=ks,
                          new_values=vs)
        for l in range(layers):
            eager = paged_attention_decode(qs[l], ref_k[:, l], ref_v[:, l], tables, lens, D ** -0.5, slots,
                                           ks[l], vs[l])
            assert torch.equal(outs[l], eager), (s, l)
    torch.cuda.synchronize()
    assert torch.equal(pool_k, ref_k) and torch.equal(pool_v, ref_v)


def test_bucket_max_blocks():
    assert [bucket_max_blocks(x) for x in (1, 2, 3, 33, 64, 65)] == [1, 2, 4, 64, 64, 128]


@pytest.mark.gpu
def test_graph_replays_the_cascade_like_eager():
    """Shared-prefix groups under capture: the prefix pass, its split counters
    and the folding decode replay for later steps exactly as eager calls."""
    from _util import excess_err, max_err
    from llm_serving_runtime_b200 import PrefixGroups

    g = torch.Generator().manual_seed(8)
    layers, B, Hq, Hkv, D, bs = 2, 8, 32, 8, 128, 16
    ctx = torch.tensor([530, 70, 600, 100, 700, 50, 512, 20])
    # the 512-token prefix with only 16 prefix tiles takes two splits
    groups, prefix = [[0, 2, 4, 6], [1, 3]], [512, 64]
    steps = 3
    max_blocks = bucket_max_blocks(int(((ctx + steps + bs - 1) // bs).max()))
    nb = B * max_blocks
    pool_k = (torch.randn(nb, layers, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    pool_v = (torch.randn(nb, layers, Hkv, bs, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
    ref_k, ref_v = pool_k.clone(), pool_v.clone()
    tables = torch.randperm(nb, generator=g).reshape(B, max_blocks).to(torch.int32)
    for rows, p in zip(groups, prefix):
        for r in rows[1:]:
            tables[r, :p // bs] = tables[rows[0], :p // bs]
    tables = tables.to(DEV)
    pg = PrefixGroups.from_members(groups, prefix, B, DEV)
    graph = DecodeStepGraph([pool_k[:, l] for l in range(layers)], [pool_v[:, l] for l in range(layers)],
                            batch=B, max_blocks=max_blocks, num_q_heads=Hq, scale=D ** -0.5, prefix_groups=pg)
    for s in range(steps):
        lens = (ctx + s).to(torch.int32).to(DEV)
        slots = oracle.slot_mapping_from_tables(tables.cpu(), lens.cpu().to(torch.int64), 1, bs).to(DEV)
        qs = [(torch.randn(B, Hq, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(layers)]
        ks = [(torch.randn(B, Hkv, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(layers)]
        vs = [(torch.randn(B, Hkv, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV) for _ in range(layers)]
        outs = graph.step(block_tables=tables, context_lens=lens, slot_mapping=slots, queries=qs, new_keys=ks,
                          new_values=vs)
        for l in range(layers):
            eager = paged_attention_decode(qs[l], ref_k[:, l], ref_v[:, l], tables, lens, D ** -0.5, slots,
                                           ks[l], vs[l], prefix_groups=pg)
            assert torch.equal(outs[l], eager), (s, l)
            if s == steps - 1:
                ref = oracle.paged_decode(qs[l].cpu(), pool_k[:, l].cpu(), pool_v[:, l].cpu(), tables.cpu(),
                                          lens.cpu(), D ** -0.5, len_offset=1)
                assert excess_err(outs[l], ref) <= 0, f"max abs err {max_err(outs[l], ref)}"
    torch.cuda.synchronize()
    assert torch.equal(pool_k, ref_k) and torch.equal(pool_v, ref_v)
