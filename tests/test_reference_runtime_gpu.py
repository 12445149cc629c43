"""The drop-in on the B200 through the reference's own code.

``integration.install()`` patches the reference runtime (imported from the
checkout, or from the unmodified copy in baseline/_ref), then the reference's
own classes run on top of the sm_100a kernels:

* ``BlockPagedBatchLayer.update`` (paged_kv_cache.py:121-170) for several
  layers and decode steps, each followed by the reference's attention hook
  (block_paged_attention.py:35-48) — outputs against the oracle, the pool
  against the oracle's append, bit for bit;
* its graph-safe branch (paged_kv_cache.py:130-145) captured once in a CUDA
  graph and replayed for later steps;
* a multi-token step (batched prefill, then a 4-token verify) through the same
  update and hook, which now runs the causal multi-query kernels over the paged
  KV instead of gathering;
* ``BlockPagedLayer`` (batch 1) prefill and decode;
* ``CudaGraphDecodeManager.try_decode`` (cuda_graph_decode.py:136-245) driving
  a small random-init Llama through capture and replay, against the manager's
  own eager step on a twin pool.
"""

from __future__ import annotations

import importlib
import sys
from types import SimpleNamespace

import pytest
import torch

from _util import excess_err, max_err
from conftest import reference_root
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
BF16 = torch.bfloat16


def _import_reference(root):
    sys.path.insert(0, str(root))
    names = ("paged_attention_triton", "paged_kv_kernel", "paged_kv_cache", "block_paged_attention",
             "cuda_graph_decode")
    return SimpleNamespace(**{n: importlib.import_module(f"runtime.phase2.{n}") for n in names})


@pytest.fixture(scope="module")
def ref():
    root = reference_root()
    if root is None:
        pytest.skip("reference runtime not importable (no checkout and no baseline/_ref copy)")
    from llm_serving_runtime_b200 import integration

    mods = _import_reference(root)
    integration.install()
    yield mods
    integration.uninstall()
    sys.path.remove(str(root))


def _config(layers, heads, kv_heads, head_dim, vocab=256):
    from transformers import LlamaConfig

    cfg = LlamaConfig(hidden_size=heads * head_dim, intermediate_size=2 * heads * head_dim,
                      num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                      head_dim=head_dim, vocab_size=vocab, max_position_embeddings=8192)
    cfg._attn_implementation = "block_paged"
    return cfg


class _Attn:
    def __init__(self, groups):
        self.num_key_value_groups = groups
        self.training = False
        self.is_causal = True


def _rand(shape, g, scale=0.5):
    return (torch.randn(shape, generator=g) * scale).to(BF16)


def _batch_cache(ref, cfg, pool, lens, max_blocks, g):
    """A BlockPagedBatchCache over rows with ``lens`` tokens cached, written into
    the pool through the reference's own write_tokens (patched append)."""
    B = len(lens)
    # the reference's pool grows on first touch (reallocating); grow it whole up
    # front so the snapshots the checks take keep one shape
    pool._grow_pools(pool.shape.num_blocks)
    ids = torch.randperm(pool.shape.num_blocks, generator=g)[: B * max_blocks].view(B, max_blocks)
    Hkv, D = pool.shape.num_kv_heads, pool.shape.head_dim
    for b, n in enumerate(lens):
        for layer in range(pool.shape.num_layers):
            k, v = _rand((1, Hkv, n, D), g), _rand((1, Hkv, n, D), g)
            pool.write_tokens(layer, ids[b].tolist(), 0, k.to(DEV), v.to(DEV))
    cache = ref.paged_kv_cache.BlockPagedBatchCache(
        cfg, pool, block_tables=ids.to(torch.int32), seq_lens=torch.tensor(lens, dtype=torch.int32),
        block_ids_rows=ids.tolist())
    return cache, ids.to(torch.int32)


def _step_and_check(ref, cache, pool, layer, q, k_new, v_new, tables, G, D):
    """One layer of one step: the reference's update + hook, checked against
    the oracle's append and attention."""
    before_k = pool.k_layer_view(layer).cpu().unsqueeze(1)
    before_v = pool.v_layer_view(layer).cpu().unsqueeze(1)
    start = cache.layers[layer]._row_seq_lens.cpu().clone()
    k_out, v_out = cache.layers[layer].update(k_new, v_new)
    if q.shape[2] > 1:  # a multi-token step attends the paged cache instead of a gather
        from llm_serving_runtime_b200.integration import MultiQueryMetadata

        meta = ref.paged_attention_triton.get_paged_decode_batch_metadata()
        assert isinstance(meta, MultiQueryMetadata) and meta.q_len == q.shape[2]
        assert k_out is k_new and v_out is v_new
    out, weights = ref.block_paged_attention.block_paged_attention_forward(_Attn(G), q, k_out, v_out, None,
                                                                           D ** -0.5)
    torch.cuda.synchronize()
    q_len = q.shape[2]
    oracle.write_tokens_batch(before_k, before_v, 0, tables, start, k_new.cpu(), v_new.cpu())
    assert torch.equal(pool.k_layer_view(layer).cpu().view(torch.int16), before_k[:, 0].view(torch.int16))
    assert torch.equal(pool.v_layer_view(layer).cpu().view(torch.int16), before_v[:, 0].view(torch.int16))
    assert weights is None and out.shape == (q.shape[0], q_len, q.shape[1], D)
    expected = oracle.paged_decode(q.cpu(), before_k[:, 0], before_v[:, 0], tables, start.to(torch.int32), D ** -0.5,
                                   len_offset=q_len)
    assert excess_err(out.transpose(1, 2), expected) <= 0, f"max abs err {max_err(out.transpose(1, 2), expected)}"


def test_batch_cache_decode_steps_through_the_reference_hook(ref):
    B, Hkv, G, D, layers = 5, 8, 4, 128, 2
    g = torch.Generator().manual_seed(11)
    lens, max_blocks = [3, 16, 100, 250, 31], 20
    pool = ref.paged_kv_kernel.GpuKVBlockPool(num_blocks=B * max_blocks + 8, block_size_tokens=16,
                                              num_layers=layers, num_kv_heads=Hkv, head_dim=D, dtype=BF16,
                                              device=DEV)
    cache, tables = _batch_cache(ref, _config(layers, Hkv * G, Hkv, D), pool, lens, max_blocks, g)
    for _step in range(3):
        for layer in range(layers):
            q = _rand((B, Hkv * G, 1, D), g).to(DEV)
            k_new, v_new = _rand((B, Hkv, 1, D), g).to(DEV), _rand((B, Hkv, 1, D), g).to(DEV)
            _step_and_check(ref, cache, pool, layer, q, k_new, v_new, tables, G, D)
    assert cache.seq_lens.cpu().tolist() == [n + 3 for n in lens]


def test_multi_token_steps_run_the_paged_kernels(ref):
    """Batched prefill of 64 new tokens per row over cached contexts, then a
    4-token verify: the update publishes multi-query metadata instead of
    gathering, and the hook attends causally over the paged KV."""
    B, Hkv, G, D, layers = 6, 8, 4, 128, 2
    g = torch.Generator().manual_seed(12)
    lens, max_blocks = [0, 5, 77, 300, 16, 1000], 70
    pool = ref.paged_kv_kernel.GpuKVBlockPool(num_blocks=B * max_blocks + 8, block_size_tokens=16,
                                              num_layers=layers, num_kv_heads=Hkv, head_dim=D, dtype=BF16,
                                              device=DEV)
    cache, tables = _batch_cache(ref, _config(layers, Hkv * G, Hkv, D), pool, lens, max_blocks, g)
    for q_len in (64, 4):
        for layer in range(layers):
            q = _rand((B, Hkv * G, q_len, D), g).to(DEV)
            k_new, v_new = _rand((B, Hkv, q_len, D), g).to(DEV), _rand((B, Hkv, q_len, D), g).to(DEV)
            _step_and_check(ref, cache, pool, layer, q, k_new, v_new, tables, G, D)
    assert cache.seq_lens.cpu().tolist() == [n + 68 for n in lens]


def test_padded_multi_token_mask_keeps_the_reference_eager_path(ref):
    """A mask with a pad inside a row is not the plain causal pattern: the hook
    gathers and runs the reference's eager attention, as the reference does."""
    B, Hkv, G, D = 2, 2, 4, 64
    g = torch.Generator().manual_seed(13)
    pool = ref.paged_kv_kernel.GpuKVBlockPool(num_blocks=16, block_size_tokens=16, num_layers=1,
                                              num_kv_heads=Hkv, head_dim=D, dtype=BF16, device=DEV)
    cache, tables = _batch_cache(ref, _config(1, Hkv * G, Hkv, D), pool, [10, 10], 4, g)
    q_len = 3
    q = _rand((B, Hkv * G, q_len, D), g).to(DEV)
    k_new, v_new = _rand((B, Hkv, q_len, D), g).to(DEV), _rand((B, Hkv, q_len, D), g).to(DEV)
    k_out, v_out = cache.layers[0].update(k_new, v_new)
    cols = torch.arange(13, device=DEV)
    allowed = (cols[None, :] <= (10 + torch.arange(q_len, device=DEV))[:, None])[None, None].expand(B, 1, q_len, 13)
    mask = torch.zeros(B, 1, q_len, 13, device=DEV, dtype=BF16).masked_fill(~allowed, torch.finfo(BF16).min)
    mask[1, :, :, 2] = torch.finfo(BF16).min  # row 1 does not attend position 2
    out, weights = ref.block_paged_attention.block_paged_attention_forward(_Attn(G), q, k_out, v_out, mask,
                                                                           D ** -0.5)
    assert weights is not None  # the reference's eager branch returns its weights
    keys, values = pool.gather_layer_batch(0, cache.block_tables, cache.seq_lens)
    kk = keys.repeat_interleave(G, dim=1).float()
    vv = values.repeat_interleave(G, dim=1).float()
    s = (q.float() @ kk.transpose(2, 3)) * D ** -0.5 + mask.float()
    expected = (torch.softmax(s, dim=-1).to(BF16).float() @ vv).transpose(1, 2)
    assert (out.float() - expected).abs().max().item() < 2e-2


def test_graph_safe_branch_captured_and_replayed(ref):
    """The graph-safe update (reused start-position buffer, in-place lengths)
    plus the hook, captured once and replayed for two more steps."""
    B, Hkv, G, D, layers = 4, 8, 4, 128, 2
    g = torch.Generator().manual_seed(14)
    lens, max_blocks = [7, 64, 200, 33], 16
    pool = ref.paged_kv_kernel.GpuKVBlockPool(num_blocks=B * max_blocks + 4, block_size_tokens=16,
                                              num_layers=layers, num_kv_heads=Hkv, head_dim=D, dtype=BF16,
                                              device=DEV)
    cfg = _config(layers, Hkv * G, Hkv, D)
    cache, tables = _batch_cache(ref, cfg, pool, lens, max_blocks, g)
    cache._graph_safe = True
    statics = [(torch.zeros(B, Hkv * G, 1, D, dtype=BF16, device=DEV),
                torch.zeros(B, Hkv, 1, D, dtype=BF16, device=DEV),
                torch.zeros(B, Hkv, 1, D, dtype=BF16, device=DEV)) for _ in range(layers)]
    outs = [None] * layers

    def step():
        for layer, (q, k, v) in enumerate(statics):
            ko, vo = cache.layers[layer].update(k, v)
            outs[layer], _ = ref.block_paged_attention.block_paged_attention_forward(_Attn(G), q, ko, vo, None,
                                                                                     D ** -0.5)

    def fill():
        for q, k, v in statics:
            q.copy_(_rand(q.shape, g))
            k.copy_(_rand(k.shape, g))
            v.copy_(_rand(v.shape, g))

    fill()
    step()  # eager: sizes the workspace and the start-position buffer
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for replay in range(2):
        fill()
        before = [(pool.k_layer_view(l).cpu().unsqueeze(1), pool.v_layer_view(l).cpu().unsqueeze(1))
                  for l in range(layers)]
        start = cache.seq_lens.cpu().clone()
        graph.replay()
        torch.cuda.synchronize()
        for layer, (q, k, v) in enumerate(statics):
            kb, vb = before[layer]
            oracle.write_tokens_batch(kb, vb, 0, tables, start, k.cpu(), v.cpu())
            assert torch.equal(pool.k_layer_view(layer).cpu().view(torch.int16), kb[:, 0].view(torch.int16))
            expected = oracle.paged_decode(q.cpu(), kb[:, 0], vb[:, 0], tables, start.to(torch.int32), D ** -0.5)
            assert excess_err(outs[layer].transpose(1, 2), expected) <= 0
        assert cache.seq_lens.cpu().tolist() == [n + 2 + replay for n in lens]
    del graph


def test_single_sequence_layer_prefill_and_decode(ref):
    """BlockPagedLayer (batch 1): a 40-token prefill and two decode steps."""
    Hkv, G, D, layers = 8, 4, 128, 1
    g = torch.Generator().manual_seed(15)
    pool = ref.paged_kv_kernel.GpuKVBlockPool(num_blocks=16, block_size_tokens=16, num_layers=layers,
                                              num_kv_heads=Hkv, head_dim=D, dtype=BF16, device=DEV)
    pool._grow_pools(pool.shape.num_blocks)
    cache = ref.paged_kv_cache.BlockPagedCache(_config(layers, Hkv * G, Hkv, D), pool)
    ids = [9, 3, 12, 0, 5]
    cache.set_block_ids(ids)
    table = torch.tensor([ids], dtype=torch.int32)
    seen = 0
    for q_len in (40, 1, 1):
        q = _rand((1, Hkv * G, q_len, D), g).to(DEV)
        k_new, v_new = _rand((1, Hkv, q_len, D), g).to(DEV), _rand((1, Hkv, q_len, D), g).to(DEV)
        before_k = pool.k_layer_view(0).cpu().unsqueeze(1)
        before_v = pool.v_layer_view(0).cpu().unsqueeze(1)
        ko, vo = cache.layers[0].update(k_new, v_new)
        out, _ = ref.block_paged_attention.block_paged_attention_forward(_Attn(G), q, ko, vo, None, D ** -0.5)
        torch.cuda.synchronize()
        oracle.write_tokens_batch(before_k, before_v, 0, table, torch.tensor([seen]), k_new.cpu(), v_new.cpu())
        expected = oracle.paged_decode(q.cpu(), before_k[:, 0], before_v[:, 0], table,
                                       torch.tensor([seen], dtype=torch.int32), D ** -0.5)
        assert excess_err(out.transpose(1, 2), expected) <= 0
        seen += q_len
    assert cache.get_seq_length() == seen


def _graph_manager_run(root: str) -> dict:
    """The reference's CudaGraphDecodeManager over a small random Llama: three
    requests prefilled one at a time (as the worker does, through the
    multi-query path), bound to a persistent batch, then decode steps through
    try_decode; each step is also run as the manager's own eager step on a
    twin pool."""
    import os

    os.environ["PHASE2_CUDA_GRAPH"] = "1"
    os.environ["PHASE2_CUDA_GRAPH_TRY_HF"] = "1"
    from transformers import LlamaForCausalLM
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    from llm_serving_runtime_b200 import integration

    mods = _import_reference(root)
    ALL_ATTENTION_FUNCTIONS.register("block_paged", mods.block_paged_attention.block_paged_attention_forward)
    integration.install()
    torch.manual_seed(0)
    cfg = _config(2, 16, 4, 128, vocab=512)
    llama = LlamaForCausalLM(cfg).to(device=DEV, dtype=BF16).eval()

    class PositionsFromCachePosition(torch.nn.Module):
        """The manager hands the model each row's position as cache_position
        (cuda_graph_decode.py:119, :180-186).  transformers 5.5's Llama ignores
        it and derives position ids from the cache-level get_seq_length(),
        whose .item() (paged_kv_cache.py:407) invalidates any capture; this
        wrapper passes the manager's positions as position ids instead."""

        def __init__(self, inner):
            super().__init__()
            self.inner = inner

        def forward(self, input_ids, past_key_values, cache_position=None, use_cache=True):
            return self.inner(input_ids=input_ids, past_key_values=past_key_values,
                              position_ids=cache_position.view(-1, 1), use_cache=use_cache)

    model = PositionsFromCachePosition(llama)
    prompts = [torch.randint(0, 512, (1, n)) for n in (23, 57, 130)]

    def setup():
        pool = mods.paged_kv_kernel.GpuKVBlockPool(num_blocks=64, block_size_tokens=16, num_layers=2,
                                                   num_kv_heads=4, head_dim=128, dtype=BF16, device=DEV)
        pool._grow_pools(64)
        persistent = mods.paged_kv_cache.BlockPagedBatchCache.empty(cfg, pool, max_batch_size=3, max_blocks=16)
        states = []
        with torch.no_grad():
            for i, ids in enumerate(prompts):
                cache = mods.paged_kv_cache.BlockPagedCache(cfg, pool)
                cache.set_block_ids(list(range(16 * i + 1, 16 * i + 13)))
                llama(input_ids=ids.to(DEV), past_key_values=cache, use_cache=True)
                state = SimpleNamespace(req=SimpleNamespace(request_id=f"r{i}"), past_key_values=cache)
                persistent.bind_cache(f"r{i}", cache)
                states.append(state)
        manager = mods.cuda_graph_decode.CudaGraphDecodeManager(model=model, device=DEV)
        return pool, persistent, states, manager

    pool_g, pers_g, states_g, mgr = setup()
    pool_e, pers_e, states_e, twin = setup()
    diffs, replays = [], []
    for step in range(7):
        ids = torch.randint(0, 512, (3, 1), device=DEV)
        with torch.no_grad():
            logits = mgr.try_decode(persistent=pers_g, decode_states=states_g, input_ids=ids)
        if logits is None:
            return {"error": f"try_decode fell back to eager: {mgr.disable_reason}"}
        bucket = next(iter(mgr.buckets.values()))
        captured_now = bucket.graph is not None and bucket.replays == 1
        if captured_now:
            # the capture call returns the captured (not yet run) step's outputs
            # and leaves the lengths where they were (cuda_graph_decode.py:199-229)
            replays.append(0)
            continue
        slots = [pers_e._request_to_slot[s.req.request_id] for s in states_e]
        tb = twin._ensure_bucket(3, max(len(pers_e.block_ids_rows[s]) for s in slots), pers_e)
        twin._copy_rows_into_bucket(tb, pers_e, slots, ids)
        with torch.no_grad():
            eager = twin._forward(tb).logits[:, -1, :]
        twin._write_back(pers_e, tb, slots, states_e)
        torch.cuda.synchronize()
        diffs.append((logits.float() - eager.float()).abs().max().item() / eager.float().abs().max().item())
        replays.append(bucket.replays)
    same_pool = torch.equal(pool_g._k_pool.view(torch.int16), pool_e._k_pool.view(torch.int16))
    return {"diffs": diffs, "replays": replays, "disabled": mgr.disabled, "same_pool": same_pool,
            "seq_lens": pers_g.seq_lens.cpu().tolist(), "twin_seq_lens": pers_e.seq_lens.cpu().tolist()}


def _graph_manager_child(rank, root, queue):
    try:
        queue.put(_graph_manager_run(root))
    except Exception as exc:  # noqa: BLE001 - reported to the parent test
        queue.put({"error": f"{type(exc).__name__}: {exc}"})


def test_cuda_graph_decode_manager_capture_and_replay():
    """Runs in a child process: a failed HF capture can leave the CUDA context
    unusable for the rest of the process (cuda_graph_decode.py:150-151)."""
    import torch.multiprocessing as mp

    root = reference_root()
    if root is None:
        pytest.skip("reference runtime not importable (no checkout and no baseline/_ref copy)")
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    proc = ctx.Process(target=_graph_manager_child, args=(0, str(root), queue))
    proc.start()
    proc.join(timeout=600)
    assert proc.exitcode == 0, f"child exited with {proc.exitcode}"
    res = queue.get(timeout=10)
    assert "error" not in res, res["error"]
    assert not res["disabled"]
    assert res["replays"][-1] >= 3, res
    assert res["seq_lens"] == res["twin_seq_lens"]
    assert res["same_pool"], "graph replays wrote different K/V than the eager steps"
    assert max(res["diffs"]) <= 1e-2, res["diffs"]  # relative to the largest logit
