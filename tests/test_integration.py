"""integration.install() on the reference runtime itself: every patch point is
replaced by this package's function and uninstall() restores the originals.
Needs the reference checkout (LLM_SERVING_RUNTIME_ROOT) and its imports; no GPU."""

from __future__ import annotations

import importlib
import sys

import pytest

from conftest import reference_root


@pytest.fixture
def reference_modules():
    root = reference_root()
    if root is None:
        pytest.skip("reference checkout not available (set LLM_SERVING_RUNTIME_ROOT)")
    sys.path.insert(0, str(root))
    try:
        mods = {name: importlib.import_module(name) for name in (
            "runtime.phase2.paged_attention_triton", "runtime.phase2.block_paged_attention",
            "runtime.phase2.paged_kv_kernel", "runtime.phase2.paged_kv_cache")}
    except ImportError as exc:
        sys.path.remove(str(root))
        pytest.skip(f"reference modules do not import here: {exc}")
    yield mods
    sys.path.remove(str(root))


def _current(point):
    from llm_serving_runtime_b200 import integration

    owner, attr = integration._resolve(importlib.import_module(point[0]), point[1])
    return getattr(owner, attr)


def test_install_patches_every_point_and_uninstall_restores(reference_modules):
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from llm_serving_runtime_b200 import integration, reference_api

    pat = reference_modules["runtime.phase2.paged_attention_triton"]
    bpa = reference_modules["runtime.phase2.block_paged_attention"]
    pool_cls = reference_modules["runtime.phase2.paged_kv_kernel"].GpuKVBlockPool
    points = integration.PATCH_POINTS + integration.MULTI_QUERY_PATCH_POINTS
    before = [_current(p) for p in points]
    # the worker registers the reference's hook under this name (worker_server.py:274-280)
    ALL_ATTENTION_FUNCTIONS.register("block_paged", bpa.block_paged_attention_forward)
    patched = integration.install()
    try:
        assert len(patched) == len(points) + 1
        assert all(_current(p) is not b for p, b in zip(points, before))
        assert pat._paged_attention_decode_batched_triton.b200_impl is \
            reference_api._paged_attention_decode_batched_triton
        assert pat.paged_attention_decode_batched.b200_impl is reference_api.paged_attention_decode_batched
        assert pat.paged_attention_decode.b200_impl is reference_api.paged_attention_decode
        assert pat.triton_available is reference_api.triton_available
        assert bpa.paged_attention_decode_batched.b200_impl is reference_api.paged_attention_decode_batched
        assert bpa.block_paged_attention_forward.b200_impl is True
        assert ALL_ATTENTION_FUNCTIONS["block_paged"] is bpa.block_paged_attention_forward
        # the reference's own metadata type flows through the shim unchanged
        assert pat.PagedDecodeBatchMetadata.__name__ == reference_api.PagedDecodeBatchMetadata.__name__
        integration.install()  # idempotent: the originals stay saved once
    finally:
        integration.uninstall()
    after = [_current(p) for p in points]
    assert all(a is b for a, b in zip(before, after))
    assert ALL_ATTENTION_FUNCTIONS["block_paged"] is bpa.block_paged_attention_forward
    assert integration.install(multi_query=False) and _current(integration.MULTI_QUERY_PATCH_POINTS[0]) is before[
        len(integration.PATCH_POINTS)]
    integration.uninstall()


def test_multi_query_mask_check():
    """The hook runs the paged kernels only for masks that mean plain causal
    attention over each row's own length; anything else goes the reference's way."""
    import torch

    from llm_serving_runtime_b200.integration import MultiQueryMetadata, _mask_is_plain_causal

    class Causal:
        is_causal = True

    lens = torch.tensor([5, 9], dtype=torch.int32)
    meta = MultiQueryMetadata(pool=None, layer_idx=0, block_tables=torch.zeros(2, 1, dtype=torch.int32),
                              seq_lens=lens, q_len=3)
    cols = torch.arange(12)
    last = lens[:, None].long() - 3 + torch.arange(3)[None, :]
    allowed = (cols[None, None, :] <= last[:, :, None])[:, None]  # [B, 1, q, cols]
    minf = torch.finfo(torch.float32).min
    additive = torch.zeros(allowed.shape).masked_fill(~allowed, minf)
    assert _mask_is_plain_causal(meta, None, Causal())
    assert _mask_is_plain_causal(meta, allowed, Causal())
    assert _mask_is_plain_causal(meta, additive, Causal())
    padded = additive.clone()
    padded[0, :, :, 0] = minf  # a left pad in row 0
    assert not _mask_is_plain_causal(meta, padded, Causal())
    full = torch.zeros_like(additive)  # no causal limit at all
    assert not _mask_is_plain_causal(meta, full, Causal())

    class Bidirectional:
        is_causal = False

    assert not _mask_is_plain_causal(meta, None, Bidirectional())


def test_cpu_inputs_keep_the_reference_cpu_path(reference_modules):
    """After install(), CPU tensors still run the reference's own code (its
    unit tests on CPU-only hosts keep working); CUDA tensors go to the kernels."""
    import torch

    from llm_serving_runtime_b200 import integration

    pat = reference_modules["runtime.phase2.paged_attention_triton"]
    kvk = reference_modules["runtime.phase2.paged_kv_kernel"]
    torch.manual_seed(0)
    pool = kvk.GpuKVBlockPool(num_blocks=8, block_size_tokens=4, num_layers=1, num_kv_heads=2, head_dim=8,
                              dtype=torch.float32, device="cpu")
    k = torch.randn(1, 2, 10, 8)
    v = torch.randn(1, 2, 10, 8)
    q = torch.randn(1, 4, 1, 8)
    ids = [0, 1, 2]
    expected_pool = None
    integration.install()
    try:
        tables = torch.tensor([[3, 4, 5]], dtype=torch.int32)
        pool.write_tokens_batch(0, tables, torch.tensor([0]), k, v)  # the reference's own append (CPU pool)
        expected_pool = pool.k_layer_view(0)[3].clone()
        pool.write_tokens(0, ids, 0, k, v)
        out = pat.paged_attention_decode(q, pool, 0, ids, 10, 2, 8 ** -0.5)
    finally:
        integration.uninstall()
    ref = pat.paged_attention_decode(q, pool, 0, ids, 10, 2, 8 ** -0.5)
    assert torch.equal(out, ref)
    assert torch.equal(expected_pool, k[0, :, 0:4].to(expected_pool.dtype))
