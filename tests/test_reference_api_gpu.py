"""The reference-API shim on the GPU: the reference's own parity tests replayed
through reference_api over a layered test pool whose append is
kv_block_pool.write_tokens_batch_into.  (The reference's own cache, hook and
graph manager on top of the kernels are in test_reference_runtime_gpu.py.)"""

from __future__ import annotations

import math

import pytest
import torch

from _pool import LayeredKV
from _util import excess_err
from llm_serving_runtime_b200 import reference_api as ra
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _write_seq(pool, layer, block_ids, k, v):
    """One sequence's tokens 0..n-1 through its blocks (the reference's write_tokens)."""
    pool.write_tokens_batch(layer, torch.tensor([block_ids]), torch.tensor([0]), k, v)


def _gather(pool, layer, block_ids, seq_len):
    """Dense [1, kv_heads, seq_len, dim] K/V of one sequence (the reference's gather_layer)."""
    n = math.ceil(seq_len / pool.block_size_tokens)
    ids = torch.tensor(block_ids[:n], device=pool.device)
    k = pool.k_layer_view(layer)[ids].permute(1, 0, 2, 3)
    v = pool.v_layer_view(layer)[ids].permute(1, 0, 2, 3)
    H, D = k.shape[0], k.shape[-1]
    return k.reshape(H, -1, D)[:, :seq_len].unsqueeze(0), v.reshape(H, -1, D)[:, :seq_len].unsqueeze(0)


def _run_parity(*, dtype, num_kv_heads, num_kv_groups, head_dim, block_size, seq_len):
    """tests/test_paged_attention_kernel_parity.py:19-79 with the CUDA branch."""
    num_heads = num_kv_heads * num_kv_groups
    num_blocks = math.ceil(seq_len / block_size) + 1
    pool = LayeredKV(num_blocks, 1, num_kv_heads, block_size, head_dim, dtype, DEV)
    block_ids = list(range(num_blocks))
    torch.manual_seed(42)
    k = torch.randn(1, num_kv_heads, seq_len, head_dim, device=DEV, dtype=dtype)
    v = torch.randn(1, num_kv_heads, seq_len, head_dim, device=DEV, dtype=dtype)
    _write_seq(pool, 0, block_ids, k, v)
    query = torch.randn(1, num_heads, 1, head_dim, device=DEV, dtype=dtype)
    scaling = head_dim ** -0.5
    keys, values = _gather(pool, 0, block_ids, seq_len)
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
    pool = LayeredKV(num_blocks * batch_size, 1, num_kv_heads, block_size, head_dim, dtype, DEV)
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
        _write_seq(pool, 0, ids, k, v)
        rows.append((ids, sl))
    query = torch.randn(batch_size, num_heads, 1, head_dim, device=DEV, dtype=dtype)
    meta = ra.PagedDecodeBatchMetadata(pool=pool, layer_idx=0, block_tables=block_tables,
                                       seq_lens=torch.tensor(seq_lens, device=DEV, dtype=torch.int32))
    actual = ra.paged_attention_decode_batched(query, meta, num_kv_groups, scaling)
    for b, (ids, sl) in enumerate(rows):
        nlog = math.ceil(sl / block_size)
        keys, values = _gather(pool, 0, ids[:nlog], sl)
        expected = ra.reference_sdpa_attention(query[b:b + 1], keys, values, scaling, num_kv_groups)
        assert (expected - actual[b:b + 1]).abs().max().item() < 1e-2


def test_q_len_other_than_one_rejected_like_the_reference():
    pool = LayeredKV(4, 1, 2, 16, 64, torch.float16, DEV)
    q = torch.zeros(1, 8, 2, 64, device=DEV, dtype=torch.float16)
    meta = ra.PagedDecodeBatchMetadata(pool, 0, torch.zeros(1, 2, dtype=torch.int32, device=DEV),
                                       torch.tensor([5], dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError, match="q_len=1"):
        ra.paged_attention_decode_batched(q, meta, 4, 0.125)
    with pytest.raises(ValueError, match="seq_len must be positive"):
        ra.paged_attention_decode(q[:, :, :1], pool, 0, [0], 0, 4, 0.125)


def test_triton_available_and_warmup():
    assert ra.triton_available()
    pool = LayeredKV(4, 1, 2, 16, 128, torch.bfloat16, DEV)
    ra.warmup_paged_attention_kernel(pool, num_heads=8, num_kv_groups=4, head_dim=128, block_ids=[0, 1])


def test_batched_speculative_verify_through_the_pool():
    """k = 4 draft tokens per sequence appended with write_tokens_batch (as the
    batched cache update does), then verified in one batched call: causal over
    the drafts, against the oracle."""
    dtype, Hkv, G, D, bs, k = torch.bfloat16, 8, 4, 128, 16, 4
    cached = [5, 60, 333, 1000, 16]
    B = len(cached)
    nmax = math.ceil((max(cached) + k) / bs)
    pool = LayeredKV(B * nmax + 1, 2, Hkv, bs, D, dtype, DEV)
    g = torch.Generator(device="cpu").manual_seed(7)
    perm = torch.randperm(B * nmax + 1, generator=g)[: B * nmax].view(B, nmax).to(torch.int32)
    tables = perm.to(DEV)
    for b, c in enumerate(cached):  # the cached context of each row, layer 1
        kk = torch.randn(1, Hkv, c, D, generator=g).to(dtype).to(DEV)
        vv = torch.randn(1, Hkv, c, D, generator=g).to(dtype).to(DEV)
        _write_seq(pool, 1, perm[b].tolist(), kk, vv)
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
