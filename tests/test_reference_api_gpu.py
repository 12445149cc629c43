"""The drop-in modules on the GPU: the reference's own parity tests replayed
through reference_api / kv_block_pool, the HF hook, and the batched cache flow
(append -> metadata -> hook) the reference's BlockPagedBatchLayer.update drives."""

from __future__ import annotations

import math

import pytest
import torch

from _util import excess_err
from llm_serving_runtime_b200 import reference_api as ra
from llm_serving_runtime_b200.block_paged_attention import block_paged_attention_forward
from llm_serving_runtime_b200.kv_block_pool import GpuKVBlockPool
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _run_parity(*, dtype, num_kv_heads, num_kv_groups, head_dim, block_size, seq_len):
    """tests/test_paged_attention_kernel_parity.py:19-79 with the CUDA branch."""
    num_heads = num_kv_heads * num_kv_groups
    num_blocks = math.ceil(seq_len / block_size) + 1
    pool = GpuKVBlockPool(num_blocks=num_blocks, block_size_tokens=block_size, num_layers=1,
                          num_kv_heads=num_kv_heads, head_dim=head_dim, dtype=dtype, device=DEV)
    block_ids = list(range(num_blocks))
    torch.manual_seed(42)
    k = torch.randn(1, num_kv_heads, seq_len, head_dim, device=DEV, dtype=dtype)
    v = torch.randn(1, num_kv_heads, seq_len, head_dim, device=DEV, dtype=dtype)
    pool.write_tokens(0, block_ids, 0, k, v)
    query = torch.randn(1, num_heads, 1, head_dim, device=DEV, dtype=dtype)
    scaling = head_dim ** -0.5
    keys, values = pool.gather_layer(0, block_ids, seq_len)
    expected = ra.reference_sdpa_attention(query, keys, values, scaling, num_kv_groups)
    actual = ra.paged_attention_decode(query=query, pool=pool, layer_idx=0, block_ids=block_ids,
                                       seq_len=seq_len, num_kv_groups=num_kv_groups, scaling=scaling)
    assert actual.shape == (1, num_heads, 1, head_dim)
    assert (expected - actual).abs().max().item() < 1e-2
    # and the tighter bar against the fp32 oracle
    nlog = math.ceil(seq_len / block_size)
    ref = oracle.paged_decode(query.cpu(), pool.k_layer_view(0).cpu(), pool.v_layer_view(0).cpu(),
                              torch.tensor([block_ids[:nlog]], dtype=torch.int32),
                              torch.tensor([seq_len], dtype=torch.int32), scaling, len_offset=0)
    assert excess_err(actual, ref) <= 0


@pytest.mark.parametrize("kw", [
    dict(dtype=torch.float16, num_kv_heads=2, num_kv_groups=4, head_dim=64, block_size=16, seq_len=128),
    dict(dtype=torch.float16, num_kv_heads=2, num_kv_groups=4, head_dim=64, block_size=16, seq_len=768),
    dict(dtype=torch.float32, num_kv_heads=2, num_kv_groups=2, head_dim=32, block_size=4, seq_len=7),
    dict(dtype=torch.float32, num_kv_heads=4, num_kv_groups=4, head_dim=64, block_size=16, seq_len=100),
    dict(dtype=torch.bfloat16, num_kv_heads=8, num_kv_groups=4, head_dim=128, block_size=16, seq_len=4000),
])
def test_reference_parity_suite_on_gpu(kw):
    _run_parity(**kw)


def test_batched_ragged_reference_test():
    """tests/test_paged_attention_kernel_parity.py:127-185 through the batched entry."""
    dtype, num_kv_heads, num_kv_groups, head_dim, block_size = torch.float16, 2, 4, 64, 16
    batch_size, seq_lens = 4, [7, 15, 31, 63]
    num_blocks = math.ceil(max(seq_lens) / block_size) + 2
    pool = GpuKVBlockPool(num_blocks=num_blocks * batch_size, block_size_tokens=block_size, num_layers=1,
                          num_kv_heads=num_kv_heads, head_dim=head_dim, dtype=dtype, device=DEV)
    torch.manual_seed(99)
    scaling = head_dim ** -0.5
    num_heads = num_kv_heads * num_kv_groups
    block_tables = torch.zeros(batch_size, num_blocks, device=DEV, dtype=torch.int32)
    rows = []
    for b in range(batch_size):
        ids = list(range(b * num_blocks, (b + 1) * num_blocks))
        sl = seq_lens[b]
        nlog = math.ceil(sl / block_size)
        block_tables[b, :nlog] = torch.tensor(ids[:nlog], device=DEV, dtype=torch.int32)
        k = torch.randn(1, num_kv_heads, sl, head_dim, device=DEV, dtype=dtype)
        v = torch.randn(1, num_kv_heads, sl, head_dim, device=DEV, dtype=dtype)
        pool.write_tokens(0, ids, 0, k, v)
        rows.append((ids, sl))
    query = torch.randn(batch_size, num_heads, 1, head_dim, device=DEV, dtype=dtype)
    meta = ra.PagedDecodeBatchMetadata(pool=pool, layer_idx=0, block_tables=block_tables,
                                       seq_lens=torch.tensor(seq_lens, device=DEV, dtype=torch.int32))
    actual = ra.paged_attention_decode_batched(query, meta, num_kv_groups, scaling)
    for b, (ids, sl) in enumerate(rows):
        nlog = math.ceil(sl / block_size)
        keys, values = pool.gather_layer(0, ids[:nlog], sl)
        expected = ra.reference_sdpa_attention(query[b:b + 1], keys, values, scaling, num_kv_groups)
        assert (expected - actual[b:b + 1]).abs().max().item() < 1e-2


def test_q_len_other_than_one_rejected_like_the_reference():
    pool = GpuKVBlockPool(num_blocks=4, block_size_tokens=16, num_layers=1, num_kv_heads=2, head_dim=64,
                          dtype=torch.float16, device=DEV)
    q = torch.zeros(1, 8, 2, 64, device=DEV, dtype=torch.float16)
    meta = ra.PagedDecodeBatchMetadata(pool, 0, torch.zeros(1, 2, dtype=torch.int32, device=DEV),
                                       torch.tensor([5], dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError, match="q_len=1"):
        ra.paged_attention_decode_batched(q, meta, 4, 0.125)
    with pytest.raises(ValueError, match="seq_len must be positive"):
        ra.paged_attention_decode(q[:, :, :1], pool, 0, [0], 0, 4, 0.125)


def test_hook_and_batched_cache_flow():
    """What BlockPagedBatchLayer.update + the attention hook do per layer
    (paged_kv_cache.py:136-166, block_paged_attention.py:35-48)."""
    B, Hkv, G, D, bs, layers = 5, 8, 4, 128, 16, 2
    g = torch.Generator().manual_seed(0)
    ctx = torch.tensor([3, 16, 100, 250, 31])
    max_blocks = 20
    pool = GpuKVBlockPool(num_blocks=B * max_blocks, block_size_tokens=bs, num_layers=layers,
                          num_kv_heads=Hkv, head_dim=D, dtype=torch.bfloat16, device=DEV)
    pool.reserve()
    pool._k_pool.copy_((torch.randn(pool._k_pool.shape, generator=g) * 0.5).to(torch.bfloat16))
    pool._v_pool.copy_((torch.randn(pool._v_pool.shape, generator=g) * 0.5).to(torch.bfloat16))
    tables = torch.randperm(B * max_blocks, generator=g).reshape(B, max_blocks).to(torch.int32).to(DEV)
    seq_lens = ctx.to(torch.int32).to(DEV)

    class Attn:
        num_key_value_groups = G
        training = False

    for layer in range(layers):
        k_new = (torch.randn(B, Hkv, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
        v_new = (torch.randn(B, Hkv, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
        q = (torch.randn(B, Hkv * G, 1, D, generator=g) * 0.5).to(torch.bfloat16).to(DEV)
        pool.write_tokens_batch(layer, tables, seq_lens, k_new, v_new)
        meta = ra.PagedDecodeBatchMetadata(pool=pool, layer_idx=layer, block_tables=tables, seq_lens=seq_lens + 1)
        token = ra.set_paged_decode_batch_metadata(meta)
        out, weights = block_paged_attention_forward(Attn(), q, k_new, v_new, None, D ** -0.5)
        ra.reset_paged_decode_batch_metadata(token)
        assert weights is None and out.shape == (B, 1, Hkv * G, D)
        ref = oracle.paged_decode(q.cpu(), pool.k_layer_view(layer).cpu(), pool.v_layer_view(layer).cpu(),
                                  tables.cpu(), seq_lens.cpu() + 1, D ** -0.5, len_offset=0)
        assert excess_err(out.transpose(1, 2), ref) <= 0
    assert pool.allocated_block_count() > 0


def test_triton_available_and_warmup():
    assert ra.triton_available()
    pool = GpuKVBlockPool(num_blocks=4, block_size_tokens=16, num_layers=1, num_kv_heads=2, head_dim=128,
                          dtype=torch.bfloat16, device=DEV)
    ra.warmup_paged_attention_kernel(pool, num_heads=8, num_kv_groups=4, head_dim=128, block_ids=[0, 1])


def test_batched_speculative_verify_through_the_pool():
    """k = 4 draft tokens per sequence appended with write_tokens_batch (as the
    batched cache update does), then verified in one batched call: causal over
    the drafts, against the oracle."""
    dtype, Hkv, G, D, bs, k = torch.bfloat16, 8, 4, 128, 16, 4
    cached = [5, 60, 333, 1000, 16]
    B = len(cached)
    nmax = math.ceil((max(cached) + k) / bs)
    pool = GpuKVBlockPool(num_blocks=B * nmax + 1, block_size_tokens=bs, num_layers=2, num_kv_heads=Hkv,
                          head_dim=D, dtype=dtype, device=DEV)
    g = torch.Generator(device="cpu").manual_seed(7)
    perm = torch.randperm(B * nmax + 1, generator=g)[: B * nmax].view(B, nmax).to(torch.int32)
    tables = perm.to(DEV)
    for b, c in enumerate(cached):  # the cached context of each row, layer 1
        kk = torch.randn(1, Hkv, c, D, generator=g).to(dtype).to(DEV)
        vv = torch.randn(1, Hkv, c, D, generator=g).to(dtype).to(DEV)
        pool.write_tokens(1, perm[b].tolist(), 0, kk, vv)
    new_k = torch.randn(B, Hkv, k, D, generator=g).to(dtype).to(DEV)
    new_v = torch.randn(B, Hkv, k, D, generator=g).to(dtype).to(DEV)
    pool.write_tokens_batch(1, tables, torch.tensor(cached, device=DEV), new_k, new_v)
    query = torch.randn(B, Hkv * G, k, D, generator=g).to(dtype).to(DEV)
    seq_lens = torch.tensor(cached, dtype=torch.int32, device=DEV) + k
    meta = ra.PagedDecodeBatchMetadata(pool=pool, layer_idx=1, block_tables=tables, seq_lens=seq_lens)
    out = ra.paged_attention_verify_batched(query, meta, G, D ** -0.5)
    assert out.shape == (B, Hkv * G, k, D)
    ref = oracle.paged_decode(query.cpu(), pool.k_layer_view(1).cpu(), pool.v_layer_view(1).cpu(), perm,
                              seq_lens.cpu(), D ** -0.5, len_offset=0)
    assert excess_err(out, ref) <= 0
    with pytest.raises(ValueError, match="num_heads"):
        ra.paged_attention_verify_batched(query, meta, G + 1, D ** -0.5)
