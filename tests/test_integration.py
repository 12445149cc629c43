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
            "runtime.phase2.paged_kv_kernel")}
    except ImportError as exc:
        sys.path.remove(str(root))
        pytest.skip(f"reference modules do not import here: {exc}")
    yield mods
    sys.path.remove(str(root))


def test_install_patches_every_point_and_uninstall_restores(reference_modules):
    from llm_serving_runtime_b200 import integration, reference_api

    pat = reference_modules["runtime.phase2.paged_attention_triton"]
    bpa = reference_modules["runtime.phase2.block_paged_attention"]
    pool_cls = reference_modules["runtime.phase2.paged_kv_kernel"].GpuKVBlockPool
    before = (pat._paged_attention_decode_batched_triton, pat.paged_attention_decode_batched,
              pat.paged_attention_decode, pat.triton_available, bpa.paged_attention_decode_batched,
              pool_cls.write_tokens_batch)
    patched = integration.install()
    try:
        assert len(patched) == len(integration.PATCH_POINTS)
        assert pat._paged_attention_decode_batched_triton.b200_impl is \
            reference_api._paged_attention_decode_batched_triton
        assert pat.paged_attention_decode_batched.b200_impl is reference_api.paged_attention_decode_batched
        assert pat.paged_attention_decode.b200_impl is reference_api.paged_attention_decode
        assert pat.triton_available is reference_api.triton_available
        assert bpa.paged_attention_decode_batched.b200_impl is reference_api.paged_attention_decode_batched
        assert pool_cls.write_tokens_batch is not before[-1]
        # the reference's own metadata type flows through the shim unchanged
        assert pat.PagedDecodeBatchMetadata.__name__ == reference_api.PagedDecodeBatchMetadata.__name__
        integration.install()  # idempotent: the originals stay saved once
    finally:
        integration.uninstall()
    after = (pat._paged_attention_decode_batched_triton, pat.paged_attention_decode_batched,
             pat.paged_attention_decode, pat.triton_available, bpa.paged_attention_decode_batched,
             pool_cls.write_tokens_batch)
    assert all(a is b for a, b in zip(before, after))


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
