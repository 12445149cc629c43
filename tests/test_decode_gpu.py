"""Parity of the sm_100a decode kernels with the reference (golden vectors) and
with the oracle, through the C ABI (ctypes -> libpa_b200.so).

Tolerance (north star): max-abs error <= 2e-3 for fp16/bf16 and <= 1e-5 for
fp32, against the fp32 oracle rounded to the output dtype.
"""

from __future__ import annotations

import math

import pytest
import torch

from _util import TOL, excess_err, max_err, oracle_rows, split_row_pieces
from conftest import decode_cases, load_golden
from llm_serving_runtime_b200 import kv_append, paged_attention_decode, read_device_errors
from llm_serving_runtime_b200.workloads import make_workload
from oracle import oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _run_golden(case):
    data, meta = load_golden(case)
    include = meta["lens_include_query"]
    lens = data["seq_lens"] if include else data["context_lens"]
    out = paged_attention_decode(
        data["query"].to(DEV), data["key_cache"].to(DEV), data["value_cache"].to(DEV),
        data["block_tables"].to(DEV), lens.to(DEV), meta["scale"], context_lens_include_new=include,
        validate=True,
    )
    return data, meta, out


@pytest.mark.parametrize("case", [c for c in decode_cases() if c != "cfg1_fp32"])
def test_golden_decode(case):
    data, meta, out = _run_golden(case)
    expected = data.get("expected_torch", data.get("expected_eager"))
    # expected is the reference's fp32 result rounded to the dtype
    assert excess_err(out, expected) <= 0, f"{case}: max abs err {max_err(out, expected)}"


def test_golden_reference_own_tolerance_vs_sdpa():
    # the reference's parity bar, tests/test_paged_attention_kernel_parity.py:79
    for case in ("fp32_short", "fp32_longer", "fp16_128", "fp16_long_split"):
        data, meta, out = _run_golden(case)
        err = (out.float().cpu() - data["expected_sdpa"].float()).abs().max().item()
        assert err < 1e-2, (case, err)


def test_config1_append_and_decode_bit_exact_append():
    import hashlib

    data, meta = load_golden("cfg1_fp32")
    w = make_workload("cfg1-fp32-small", device="cpu").to(DEV)
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    out = paged_attention_decode(w.query, kc, vc, w.block_tables, w.context_lens, w.scale,
                                 w.slot_mapping, w.new_key, w.new_value, validate=True)
    sha = lambda t: hashlib.sha256(t.cpu().contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()
    assert sha(kc) == meta["k_cache_after_sha256"]
    assert sha(vc) == meta["v_cache_after_sha256"]
    assert max_err(out, data["expected_torch"]) <= TOL[torch.float32]


def _config_parity(name, rows=None):
    w = make_workload(name, device=DEV)
    out = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens,
                                 w.scale, w.slot_mapping, w.new_key, w.new_value, validate=True)
    torch.cuda.synchronize()
    rows = list(range(w.batch)) if rows is None else rows(w)
    ref = oracle_rows(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                      w.q_len, rows)
    err = max_err(out[rows], ref)
    assert err <= TOL[w.spec.dtype], f"{name}: max abs err {err} over {len(rows)} rows"
    return w, out


def test_config2_qwen2_full_batch():
    _config_parity("cfg2-qwen2-0.5b")


def test_config3_llama3_8b_full_batch():
    # all 256 rows; nearly every one is cut by a warp-slice boundary of the
    # stream-K split and merged from up to 3 pieces
    _config_parity("cfg3-llama3-8b")


def test_config4_prefix_shared_verify_q4_full_batch():
    _config_parity("cfg4-prefix-verify")


def test_config5_llama3_70b_full_batch():
    # all 512 rows; the stream-K split cuts most of them into several pieces
    w, out = _config_parity("cfg5-llama3-70b")
    s = w.spec
    pieces = split_row_pieces(w.context_lens, s.q_len, s.num_q_heads // s.num_kv_heads, s.num_kv_heads)
    assert sum(k > 1 for k in pieces.values()) >= 64
    del w, out
    torch.cuda.empty_cache()


def _append_touched_blocks_bit_exact(name):
    """The step's append at full size, checked bit for bit on every block the
    step's slots touch (a compact CPU copy through the oracle's scatter), and
    every other block unchanged."""
    w = make_workload(name, device=DEV)
    bs = w.key_cache.shape[2]
    slots = w.slot_mapping.cpu()
    blocks = torch.unique(slots // bs)
    index = torch.full((w.key_cache.shape[0],), -1, dtype=torch.int64)
    index[blocks] = torch.arange(blocks.numel())
    compact_slots = index[slots // bs] * bs + slots % bs
    kc_ref, vc_ref = w.key_cache[blocks.to(DEV)].cpu(), w.value_cache[blocks.to(DEV)].cpu()
    oracle.kv_append(w.new_key.cpu(), w.new_value.cpu(), kc_ref, vc_ref, compact_slots)
    k_before, v_before = w.key_cache.clone(), w.value_cache.clone()
    kv_append(w.new_key, w.new_value, w.key_cache, w.value_cache, w.slot_mapping, validate=True)
    torch.cuda.synchronize()
    bits = lambda t: t.contiguous().view(torch.int16)
    assert torch.equal(bits(w.key_cache[blocks.to(DEV)].cpu()), bits(kc_ref))
    assert torch.equal(bits(w.value_cache[blocks.to(DEV)].cpu()), bits(vc_ref))
    # the rest of the pool: equal once the touched blocks are carried over
    k_before[blocks.to(DEV)] = w.key_cache[blocks.to(DEV)]
    v_before[blocks.to(DEV)] = w.value_cache[blocks.to(DEV)]
    assert torch.equal(bits(w.key_cache), bits(k_before))
    assert torch.equal(bits(w.value_cache), bits(v_before))
    del w, k_before, v_before
    torch.cuda.empty_cache()


@pytest.mark.parametrize("name", ["cfg3-llama3-8b", "cfg5-llama3-70b"])
def test_append_at_full_size_bit_exact(name):
    _append_touched_blocks_bit_exact(name)


def _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len=1, seed=0, pool_extra=5, scale_v=0.5):
    g = torch.Generator().manual_seed(seed)
    lens = torch.as_tensor(lens, dtype=torch.int64)
    att = lens + q_len
    nblk = (att + bs - 1) // bs
    maxb = max(1, int(nblk.max()))
    nb = int(nblk.sum()) + pool_extra
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(B, maxb, dtype=torch.int32)
    c = 0
    for i in range(B):
        n = int(nblk[i])
        bt[i, :n] = perm[c:c + n].to(torch.int32)
        c += n
    kc = (torch.randn(nb, Hkv, bs, D, generator=g) * scale_v).to(dtype)
    vc = (torch.randn(nb, Hkv, bs, D, generator=g) * scale_v).to(dtype)
    q = (torch.randn(B, Hq, q_len, D, generator=g) * scale_v).to(dtype)
    return q, kc, vc, bt, lens.to(torch.int32)


EDGE = [
    # (B, Hq, Hkv, D, bs, dtype, lens, q_len)
    (6, 8, 2, 128, 16, torch.bfloat16, [0, 14, 15, 16, 31, 32], 1),
    (5, 32, 8, 128, 16, torch.bfloat16, [1, 100, 4095, 8191, 3], 1),
    (4, 14, 2, 64, 16, torch.float16, [127, 128, 129, 2047], 1),
    (3, 8, 8, 128, 16, torch.bfloat16, [5, 77, 300], 1),          # G = 1 (MHA)
    (3, 16, 1, 64, 16, torch.float16, [40, 41, 500], 1),          # G = 16 (one full m-tile)
    (3, 64, 8, 128, 16, torch.bfloat16, [2048, 3000, 9], 1),      # G = 8
    (4, 32, 8, 128, 16, torch.bfloat16, [0, 12, 13, 1000], 4),    # q_len 4, causal
    (3, 64, 8, 128, 16, torch.bfloat16, [20, 33, 700], 4),        # G*q = 32: two row groups
    (3, 14, 2, 64, 16, torch.float16, [1, 2, 300], 2),            # G*q = 14
    (4, 8, 2, 128, 8, torch.bfloat16, [0, 7, 8, 250], 1),         # block size 8
    (4, 8, 2, 64, 32, torch.float16, [0, 31, 32, 1000], 1),       # block size 32
    (3, 8, 2, 128, 64, torch.bfloat16, [63, 64, 513], 2),         # block size 64
    (3, 8, 2, 128, 128, torch.bfloat16, [127, 128, 1000], 1),    # block size 128
    (3, 32, 8, 128, 256, torch.float16, [255, 256, 2000], 2),     # block size 256
    (4, 8, 2, 64, 4, torch.float32, [0, 3, 4, 77], 1),            # fp32, block size 4
    (3, 8, 2, 64, 128, torch.float32, [100, 128, 700], 1),       # fp32, block size 128
    (3, 8, 2, 128, 16, torch.float32, [10, 31, 300], 4),          # fp32, causal
    (2, 4, 2, 32, 16, torch.float32, [5, 64], 1),                 # fp32, head_dim 32
]


@pytest.mark.parametrize("B,Hq,Hkv,D,bs,dtype,lens,q_len", EDGE)
def test_edge_shapes_vs_oracle(B, Hq, Hkv, D, bs, dtype, lens, q_len):
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len, seed=B * 7 + D)
    scale = D ** -0.5
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), scale, validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, scale)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


HEAD_DIMS = [
    # head_dim the reference's kernels serve (any size, padded to a power of
    # two) but the tiles do not match: the 16-bit kernels pad to 64 / 128 and
    # the fp32 kernel to 32 / 64 / 128 (B, Hq, Hkv, D, bs, dtype, lens, q_len)
    (4, 32, 8, 80, 16, torch.bfloat16, [1, 100, 1000, 3000], 1),
    (4, 14, 2, 96, 16, torch.float16, [7, 64, 500, 2047], 1),
    (3, 16, 4, 112, 8, torch.bfloat16, [15, 300, 999], 4),
    (3, 8, 2, 32, 16, torch.bfloat16, [3, 200, 1500], 1),
    (3, 8, 2, 40, 32, torch.float16, [33, 64, 700], 2),
    (3, 8, 8, 48, 16, torch.bfloat16, [0, 17, 640], 1),
    (3, 8, 2, 80, 16, torch.float32, [5, 100, 900], 1),
    (3, 8, 2, 100, 16, torch.float32, [1, 63, 400], 2),
    (2, 4, 2, 24, 4, torch.float32, [7, 30], 1),
    (2, 2, 2, 1, 4, torch.float32, [3, 12], 1),     # a one-dimensional head
]


@pytest.mark.parametrize("B,Hq,Hkv,D,bs,dtype,lens,q_len", HEAD_DIMS)
def test_other_head_dims_vs_oracle(B, Hq, Hkv, D, bs, dtype, lens, q_len):
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len, seed=B * 11 + D)
    nk, nv = torch.randn(B, Hkv, q_len, D).to(dtype), torch.randn(B, Hkv, q_len, D).to(dtype)
    kcd, vcd = kc.to(DEV), vc.to(DEV)
    out = paged_attention_decode(q.to(DEV), kcd, vcd, bt.to(DEV), cl.to(DEV), D ** -0.5, None, nk.to(DEV),
                                 nv.to(DEV), validate=True)
    kc2, vc2 = kc.clone(), vc.clone()
    oracle.write_tokens_batch(kc2.unsqueeze(1), vc2.unsqueeze(1), 0, bt, cl.long(), nk, nv)
    assert torch.equal(kcd.cpu(), kc2) and torch.equal(vcd.cpu(), vc2)  # the append, bit for bit
    ref = oracle.paged_decode(q, kc2, vc2, bt, cl, D ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_unserved_head_dims_are_value_errors():
    for D, dtype in ((136, torch.bfloat16), (256, torch.float16), (20, torch.bfloat16), (160, torch.float32)):
        q, kc, vc, bt, cl = _synthetic(1, 2, 2, D, 16, dtype, [5], seed=3)
        with pytest.raises(ValueError, match="head_dim"):
            paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 0.1)


def test_one_long_sequence_split_over_the_whole_grid():
    # B = 1, 64k tokens: every warp of the grid takes a slice of the one row,
    # so the log-sum-exp merge combines hundreds of partials.
    q, kc, vc, bt, cl = _synthetic(1, 32, 8, 128, 16, torch.bfloat16, [65535], seed=3)
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 128 ** -0.5,
                                 validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, 128 ** -0.5)
    assert max_err(out, ref) <= TOL[torch.bfloat16]


def test_many_short_sequences_and_large_batch():
    lens = torch.randint(0, 64, (3000,), generator=torch.Generator().manual_seed(1)).tolist()
    q, kc, vc, bt, cl = _synthetic(3000, 8, 2, 128, 16, torch.bfloat16, lens, seed=4)
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 128 ** -0.5,
                                 validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, 128 ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_batch_beyond_the_shared_memory_tables_is_split():
    # 9000 sequences at head_dim 128: more than the decode kernel's per-sequence
    # shared-memory tables hold (about 8.3 k), so the call attends the batch in
    # halves; the append covers every row in one launch first.
    B = 9000
    lens = torch.randint(0, 40, (B,), generator=torch.Generator().manual_seed(12)).tolist()
    q, kc, vc, bt, cl = _synthetic(B, 8, 2, 128, 16, torch.bfloat16, lens, seed=13)
    nk = (torch.randn(B, 2, 1, 128, generator=torch.Generator().manual_seed(14)) * 0.5).to(torch.bfloat16)
    nv = (torch.randn(B, 2, 1, 128, generator=torch.Generator().manual_seed(15)) * 0.5).to(torch.bfloat16)
    kcd, vcd = kc.to(DEV), vc.to(DEV)
    out = paged_attention_decode(q.to(DEV), kcd, vcd, bt.to(DEV), cl.to(DEV), 128 ** -0.5, None, nk.to(DEV),
                                 nv.to(DEV), validate=True)
    oracle.write_tokens_batch(kc.unsqueeze(1), vc.unsqueeze(1), 0, bt, cl.long(), nk, nv)
    assert torch.equal(kcd.cpu(), kc) and torch.equal(vcd.cpu(), vc)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, 128 ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_strided_pool_layer_view_and_transposed_query():
    # GpuKVBlockPool layout [num_blocks, layers, Hkv, bs, D]; layer 1 of 3; query
    # as HF produces it ([B, q, H, D] transposed to [B, H, q, D]).
    B, Hq, Hkv, D, bs = 4, 32, 8, 128, 16
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, torch.bfloat16, [17, 250, 16, 1], q_len=2, seed=9)
    nb = kc.shape[0]
    kpool = torch.randn(nb, 3, Hkv, bs, D).to(torch.bfloat16)
    vpool = torch.randn(nb, 3, Hkv, bs, D).to(torch.bfloat16)
    kpool[:, 1] = kc
    vpool[:, 1] = vc
    kpool, vpool = kpool.to(DEV), vpool.to(DEV)
    q_hf = q.transpose(1, 2).contiguous().to(DEV).transpose(1, 2)
    assert not q_hf.is_contiguous()
    out = paged_attention_decode(q_hf, kpool[:, 1], vpool[:, 1], bt.to(DEV), cl.to(DEV), D ** -0.5,
                                 validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_non_finite_values_past_the_sequence_end_do_not_leak():
    # Slots past L in the last block hold NaN/Inf (an uninitialised pool): the
    # output must not see them (the reference masks its loads, :208-226).
    B, Hq, Hkv, D, bs = 3, 8, 2, 128, 16
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, torch.bfloat16, [4, 20, 33], seed=5)
    kc_d, vc_d = kc.to(DEV), vc.to(DEV)
    for b in range(B):
        L = int(cl[b]) + 1
        last = int(bt[b, (L - 1) // bs])
        off = L % bs
        if off:
            kc_d[last, :, off:] = float("nan")
            vc_d[last, :, off:] = float("inf")
    out = paged_attention_decode(q.to(DEV), kc_d, vc_d, bt.to(DEV), cl.to(DEV), D ** -0.5, validate=True)
    assert torch.isfinite(out.float()).all()
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5)
    assert excess_err(out, ref) <= 0


def test_deterministic_bitwise():
    q, kc, vc, bt, cl = _synthetic(64, 32, 8, 128, 16, torch.bfloat16,
                                   torch.randint(1, 3000, (64,), generator=torch.Generator().manual_seed(2)).tolist())
    args = [t.to(DEV) for t in (q, kc, vc, bt, cl)]
    a = paged_attention_decode(*args, 128 ** -0.5)
    b = paged_attention_decode(*args, 128 ** -0.5)
    assert torch.equal(a, b)


def test_rows_with_nothing_to_attend_are_zero():
    q, kc, vc, bt, cl = _synthetic(3, 8, 2, 128, 16, torch.bfloat16, [0, 40, 0], seed=6)
    # context_lens_include_new=True with 0 -> nothing to attend
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV),
                                 torch.tensor([0, 41, 0], dtype=torch.int32, device=DEV), 128 ** -0.5,
                                 context_lens_include_new=True)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    ref = oracle.paged_decode(q, kc, vc, bt, cl, 128 ** -0.5)
    assert excess_err(out[1:2], ref[1:2]) <= 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_out_of_range_block_id_is_flagged_not_faulted(dtype):
    q, kc, vc, bt, cl = _synthetic(2, 8, 2, 64, 16, dtype, [40, 40], seed=8)
    read_device_errors(DEV)  # clear
    bt[1, 1] = kc.shape[0] + 5  # outside the pool: TMA zero-fills / the fp32 kernel skips
    with pytest.raises(IndexError, match="out of range"):
        paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 0.125, validate=True)
    assert read_device_errors(DEV) == 0  # cleared by the failing call


def test_table_underrun_is_flagged():
    q, kc, vc, bt, cl = _synthetic(2, 8, 2, 64, 16, torch.float16, [40, 40], seed=8)
    cl[0] = 10_000  # needs far more blocks than the table holds
    with pytest.raises(IndexError, match="underrun"):
        paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), 0.125, validate=True)


def test_shape_errors_are_value_errors():
    q, kc, vc, bt, cl = _synthetic(2, 8, 2, 64, 16, torch.float16, [4, 4], seed=1)
    q, kc, vc, bt, cl = (t.to(DEV) for t in (q, kc, vc, bt, cl))
    with pytest.raises(ValueError, match="batch size must match"):
        paged_attention_decode(q, kc, vc, bt[:1], cl, 0.125)
    with pytest.raises(ValueError):
        paged_attention_decode(q.float(), kc, vc, bt, cl, 0.125)
    with pytest.raises(ValueError, match="multiple"):
        paged_attention_decode(q[:, :7], kc, vc, bt, cl, 0.125)  # 7 query heads over 2 kv heads
    with pytest.raises(ValueError):
        paged_attention_decode(q, kc, vc[:, :1], bt, cl, 0.125)


def test_cuda_graph_capture_and_replay():
    w = make_workload("cfg2-qwen2-0.5b", device=DEV)
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    out = torch.empty_like(w.query)
    static_q = w.query.clone()
    args = (static_q, kc, vc, w.block_tables, w.context_lens, w.scale, w.slot_mapping, w.new_key, w.new_value)
    paged_attention_decode(*args, out=out)  # eager call sizes the workspace
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        paged_attention_decode(*args, out=out)
    new_q = torch.randn_like(w.query.float()).to(w.query.dtype)
    static_q.copy_(new_q)
    g.replay()
    torch.cuda.synchronize()
    eager = paged_attention_decode(new_q, kc, vc, w.block_tables, w.context_lens, w.scale)
    assert torch.equal(out, eager)
