"""KV append on the GPU: bit-exact against the reference's write_tokens_batch
(golden vectors) and the oracle's slot-mapping scatter."""

from __future__ import annotations

import pytest
import torch

from _pool import LayeredKV
from conftest import load_golden
from llm_serving_runtime_b200 import kv_append, read_device_errors
from llm_serving_runtime_b200.workloads import make_workload
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _bits(t):
    return t.cpu().contiguous().view(torch.int16 if t.element_size() == 2 else torch.int32)


@pytest.mark.parametrize("case", ["append_fp16", "append_bf16"])
@pytest.mark.parametrize("pos_dtype", [torch.int64, torch.int32])
def test_write_tokens_batch_matches_reference_bits(case, pos_dtype):
    data, meta = load_golden(case)
    layer = meta["layer_idx"]
    kp = data["k_pool_before"].to(DEV)
    vp = data["v_pool_before"].to(DEV)
    kv_append(data["key_states"].to(DEV), data["value_states"].to(DEV), kp[:, layer], vp[:, layer],
              block_tables=data["block_tables"].to(DEV), positions=data["start_positions"].to(pos_dtype).to(DEV),
              validate=True)
    assert torch.equal(_bits(kp), _bits(data["k_pool_after"]))
    assert torch.equal(_bits(vp), _bits(data["v_pool_after"]))


@pytest.mark.parametrize("case", ["append_fp16", "append_bf16"])
def test_pool_write_tokens_batch_into_matches_reference_bits(case):
    """kv_block_pool.write_tokens_batch_into on a 5-D layered pool, against the
    reference's own write_tokens_batch outputs; the reference's underrun error."""
    data, meta = load_golden(case)
    kp0 = data["k_pool_before"]
    nb, L, Hkv, bs, D = kp0.shape
    pool = LayeredKV(nb, L, Hkv, bs, D, kp0.dtype, DEV)
    pool.k.copy_(kp0.to(DEV))
    pool.v.copy_(data["v_pool_before"].to(DEV))
    pool.write_tokens_batch(meta["layer_idx"], data["block_tables"], data["start_positions"],
                            data["key_states"].to(DEV), data["value_states"].to(DEV))
    assert torch.equal(_bits(pool.k), _bits(data["k_pool_after"]))
    assert torch.equal(_bits(pool.v), _bits(data["v_pool_after"]))
    with pytest.raises(IndexError, match="underrun"):
        pool.write_tokens_batch(0, data["block_tables"], torch.tensor([2, 7, 14]),
                                data["key_states"].to(DEV), data["value_states"].to(DEV))


def test_roundtrip_reference_test():
    # tests/test_paged_kv_kernel.py:11-28 on a GPU pool: write two tokens of a
    # single sequence through blocks [0, 1], read them back through the table
    data, _ = load_golden("roundtrip_fp32")
    pool = LayeredKV(4, 1, 2, 2, 4, torch.float32, DEV)
    pool.write_tokens_batch(0, torch.tensor([[0, 1]]), torch.tensor([0]), data["key_states"].to(DEV),
                            data["value_states"].to(DEV))
    keys = pool.k_layer_view(0)[:2].permute(1, 0, 2, 3).reshape(2, 4, 4)[:, :2].unsqueeze(0)
    values = pool.v_layer_view(0)[:2].permute(1, 0, 2, 3).reshape(2, 4, 4)[:, :2].unsqueeze(0)
    assert keys.shape == (1, 2, 2, 4)
    assert torch.equal(keys.cpu(), data["keys"]) and torch.equal(values.cpu(), data["values"])


@pytest.mark.parametrize("name", ["cfg1-fp32-small", "cfg2-qwen2-0.5b", "cfg4-prefix-verify"])
def test_slot_mapping_append_bit_exact_vs_oracle(name):
    w = make_workload(name, device="cpu")
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    oracle.kv_append(w.new_key, w.new_value, kc, vc, w.slot_mapping)
    wd = w.to(DEV)
    kv_append(wd.new_key, wd.new_value, wd.key_cache, wd.value_cache, wd.slot_mapping, validate=True)
    assert torch.equal(_bits(wd.key_cache), _bits(kc))
    assert torch.equal(_bits(wd.value_cache), _bits(vc))


def test_derived_slots_equal_explicit_slots():
    w = make_workload("cfg4-prefix-verify", device=DEV)
    k1, v1 = w.key_cache.clone(), w.value_cache.clone()
    k2, v2 = w.key_cache.clone(), w.value_cache.clone()
    kv_append(w.new_key, w.new_value, k1, v1, w.slot_mapping)
    kv_append(w.new_key, w.new_value, k2, v2, block_tables=w.block_tables, positions=w.context_lens)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)


def test_padding_slots_are_skipped_and_bad_slots_flagged():
    w = make_workload("cfg2-qwen2-0.5b", device=DEV)
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    slots = w.slot_mapping.clone()
    slots[3] = -1
    kv_append(w.new_key, w.new_value, kc, vc, slots, validate=True)
    # row 3's slot untouched
    s = int(w.slot_mapping[3])
    bs = kc.shape[2]
    assert torch.equal(kc[s // bs, :, s % bs], w.key_cache[s // bs, :, s % bs])
    assert not torch.equal(kc[s // bs, :, s % bs], w.new_key[3, :, 0])
    read_device_errors(DEV)
    slots[5] = kc.shape[0] * bs + 3  # outside the pool: skipped and flagged
    with pytest.raises(IndexError, match="slot"):
        kv_append(w.new_key, w.new_value, kc, vc, slots, validate=True)


def test_non_contiguous_new_rows():
    # HF gives key_states as [B, q, H, D] transposed to [B, H, q, D].
    w = make_workload("cfg4-prefix-verify", device=DEV)
    k_hf = w.new_key.transpose(1, 2).contiguous().transpose(1, 2)
    v_hf = w.new_value.transpose(1, 2).contiguous().transpose(1, 2)
    k1, v1 = w.key_cache.clone(), w.value_cache.clone()
    kv_append(k_hf, v_hf, k1, v1, w.slot_mapping)
    k2, v2 = w.key_cache.clone(), w.value_cache.clone()
    kv_append(w.new_key, w.new_value, k2, v2, w.slot_mapping)
    assert torch.equal(k1, k2) and torch.equal(v1, v2)


@pytest.mark.parametrize("bs,D,dtype", [(4, 64, torch.float32), (8, 128, torch.bfloat16), (32, 96, torch.float16),
                                        (64, 128, torch.bfloat16), (128, 64, torch.float16),
                                        (256, 128, torch.bfloat16)])
def test_append_bit_exact_across_block_sizes(bs, D, dtype):
    """Both forms of the append (explicit slots; block tables + positions) at
    every block size the decode kernels take, against the oracle's scatter."""
    g = torch.Generator().manual_seed(bs * 7 + D)
    B, Hkv, q_len, nb = 5, 4, 3, 16
    kc = torch.randn(nb, Hkv, bs, D, generator=g).to(dtype)
    vc = torch.randn(nb, Hkv, bs, D, generator=g).to(dtype)
    nk = torch.randn(B, Hkv, q_len, D, generator=g).to(dtype)
    nv = torch.randn(B, Hkv, q_len, D, generator=g).to(dtype)
    slots = torch.randperm(nb * bs, generator=g)[:B * q_len].to(torch.int64)
    kc_d, vc_d = kc.to(DEV), vc.to(DEV)
    kv_append(nk.to(DEV), nv.to(DEV), kc_d, vc_d, slots.to(DEV), validate=True)
    ref_k, ref_v = kc.clone(), vc.clone()
    oracle.kv_append(nk, nv, ref_k, ref_v, slots)
    assert torch.equal(_bits(kc_d), _bits(ref_k)) and torch.equal(_bits(vc_d), _bits(ref_v))

    # rows own 3 blocks each; a write may cross a block boundary
    tables = torch.randperm(nb, generator=g)[:B * 3].reshape(B, 3).to(torch.int32)
    starts = torch.randint(0, 3 * bs - q_len + 1, (B,), generator=g).to(torch.int64)
    kv_append(nk.to(DEV), nv.to(DEV), kc_d, vc_d, block_tables=tables.to(DEV), positions=starts.to(DEV),
              validate=True)
    derived = oracle.slot_mapping_from_tables(tables, starts, q_len, bs)
    oracle.kv_append(nk, nv, ref_k, ref_v, derived)
    assert torch.equal(_bits(kc_d), _bits(ref_k)) and torch.equal(_bits(vc_d), _bits(ref_v))


def _random_append(seed):
    import random

    from test_decode_gpu import _synthetic

    rnd = random.Random(seed)
    dtype = rnd.choice([torch.bfloat16, torch.float16, torch.float32])
    D = rnd.choice([rnd.randint(1, 160), 64, 128])
    bs = rnd.choice([4, 8, 16, 16, 32, 64, 128, 256])
    Hkv = rnd.randint(1, 8)
    q_len = rnd.choice([1, 1, 2, 4, 8, 16])
    B = rnd.randint(1, 30)
    lens = [rnd.choice([0, rnd.randint(0, 3 * bs), rnd.randint(0, 2000)]) for _ in range(B)]
    _, kc, vc, bt, cl = _synthetic(B, Hkv, Hkv, D, bs, dtype, lens, q_len, seed=5000 + seed)
    g = torch.Generator().manual_seed(6000 + seed)
    nk = torch.randn(B, Hkv, q_len, D, generator=g).to(dtype)
    nv = torch.randn(B, Hkv, q_len, D, generator=g).to(dtype)
    pos = cl.long()[:, None] + torch.arange(q_len)[None, :]
    phys = torch.gather(bt.long(), 1, pos // bs)
    slots = (phys * bs + pos % bs).reshape(-1)
    pad = torch.rand(slots.shape, generator=g) < 0.1
    return kc, vc, bt, cl, nk, nv, slots, torch.where(pad, torch.full_like(slots, -1), slots)


@pytest.mark.parametrize("seed", range(40))
def test_random_appends_bit_exact(seed):
    """Seeded random appends (dtype, head_dim 1..160, block size, KV heads,
    tokens per sequence, lengths; a tenth of the slots padding) through a slot
    mapping and through block tables + positions, bit for bit against the
    oracle's scatter."""
    kc, vc, bt, cl, nk, nv, slots, padded = _random_append(seed)
    for how in ("slots", "tables"):
        kd, vd = kc.to(DEV), vc.to(DEV)
        kr, vr = kc.clone(), vc.clone()
        if how == "slots":
            kv_append(nk.to(DEV), nv.to(DEV), kd, vd, padded.to(DEV), validate=True)
            oracle.kv_append(nk, nv, kr, vr, padded)
        else:
            kv_append(nk.to(DEV), nv.to(DEV), kd, vd, block_tables=bt.to(DEV), positions=cl.to(DEV), validate=True)
            oracle.kv_append(nk, nv, kr, vr, slots)
        assert torch.equal(_bits(kd), _bits(kr)), f"seed {seed} ({how}): key cache differs"
        assert torch.equal(_bits(vd), _bits(vr)), f"seed {seed} ({how}): value cache differs"
