"""The CPU oracle against the golden vectors recorded from the reference itself.

Pins ``oracle/`` before it is trusted as the checker of the CUDA kernels:
decode outputs must match the reference's own CPU decode
(_paged_attention_decode_torch) and eager causal path, and the append
restatements must reproduce write_tokens_batch bit for bit.
"""

from __future__ import annotations

import hashlib

import pytest
import torch

from conftest import decode_cases, golden_manifest, load_golden
from oracle import oracle

# fp32 outputs: the oracle sums in a different order than torch's einsum.
F32_TOL = 2e-6


def _lens_and_offset(data, meta):
    if meta["lens_include_query"]:
        return data["seq_lens"], 0
    return data["context_lens"], meta["q_len"]


@pytest.mark.parametrize("case", decode_cases())
def test_oracle_matches_reference_decode(case):
    if case == "cfg1_fp32":
        pytest.skip("covered by test_oracle_config1")
    data, meta = load_golden(case)
    lens, off = _lens_and_offset(data, meta)
    out = oracle.paged_decode(data["query"], data["key_cache"], data["value_cache"], data["block_tables"],
                              lens, meta["scale"], len_offset=off)
    expected = data.get("expected_torch", data.get("expected_eager"))
    got = out.to(expected.dtype)
    if expected.dtype == torch.float32:
        err = (got - expected).abs().max().item()
        assert err <= F32_TOL, f"{case}: max abs err {err}"
    else:
        # Both sides computed in fp32 and rounded to the query dtype: equal up to
        # one rounding step of the output dtype.
        diff = (got.float() - expected.float()).abs()
        ulp = torch.finfo(expected.dtype).eps * expected.float().abs().clamp_min(2.0 ** -14)
        assert bool((diff <= ulp).all()), f"{case}: max diff {diff.max().item()}"


def test_oracle_matches_reference_sdpa_on_its_own_tests():
    # tests/test_paged_attention_kernel_parity.py:79 — max_abs < 1e-2 vs SDPA
    for case in ("fp32_short", "fp32_longer", "fp16_128", "fp16_long_split"):
        data, meta = load_golden(case)
        out = oracle.paged_decode(data["query"], data["key_cache"], data["value_cache"], data["block_tables"],
                                  data["seq_lens"], meta["scale"], len_offset=0)
        err = (out.to(data["expected_sdpa"].dtype).float() - data["expected_sdpa"].float()).abs().max().item()
        assert err < 1e-2, (case, err)


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def test_oracle_config1():
    from llm_serving_runtime_b200.workloads import make_workload

    data, meta = load_golden("cfg1_fp32")
    w = make_workload(meta["workload"], device="cpu")
    for k, h in meta["input_sha256"].items():
        assert _sha(getattr(w, k)) == h, f"regenerated input {k} differs from the fixture's"
    kc, vc = w.key_cache.clone(), w.value_cache.clone()
    oracle.kv_append(w.new_key, w.new_value, kc, vc, w.slot_mapping)
    assert _sha(kc) == meta["k_cache_after_sha256"]
    assert _sha(vc) == meta["v_cache_after_sha256"]
    out = oracle.paged_decode(w.query, kc, vc, w.block_tables, w.context_lens, w.scale)
    err = (out - data["expected_torch"]).abs().max().item()
    assert err <= F32_TOL, err


@pytest.mark.parametrize("case", ["append_fp16", "append_bf16"])
def test_oracle_write_tokens_batch_bit_exact(case):
    data, meta = load_golden(case)
    kp, vp = data["k_pool_before"].clone(), data["v_pool_before"].clone()
    oracle.write_tokens_batch(kp, vp, meta["layer_idx"], data["block_tables"], data["start_positions"],
                              data["key_states"], data["value_states"])
    assert torch.equal(kp.view(torch.int16), data["k_pool_after"].view(torch.int16))
    assert torch.equal(vp.view(torch.int16), data["v_pool_after"].view(torch.int16))


@pytest.mark.parametrize("case", ["append_fp16", "append_bf16"])
def test_oracle_slot_mapping_append_equals_write_tokens_batch(case):
    data, meta = load_golden(case)
    layer = meta["layer_idx"]
    kp, vp = data["k_pool_before"].clone(), data["v_pool_before"].clone()
    q_len = data["key_states"].shape[2]
    bs = kp.shape[3]
    slots = oracle.slot_mapping_from_tables(data["block_tables"], data["start_positions"], q_len, bs)
    kview, vview = kp[:, layer], vp[:, layer]
    oracle.kv_append(data["key_states"], data["value_states"], kview, vview, slots)
    assert torch.equal(kp.view(torch.int16), data["k_pool_after"].view(torch.int16))
    assert torch.equal(vp.view(torch.int16), data["v_pool_after"].view(torch.int16))


def test_oracle_roundtrip():
    data, _ = load_golden("roundtrip_fp32")
    kp = torch.zeros_like(data["k_pool_after"])
    vp = torch.zeros_like(data["v_pool_after"])
    oracle.write_tokens_batch(kp, vp, 0, torch.tensor([[0, 1]], dtype=torch.int32), torch.tensor([0]),
                              data["key_states"], data["value_states"])
    assert torch.equal(kp, data["k_pool_after"]) and torch.equal(vp, data["v_pool_after"])


def test_oracle_underrun_raises():
    data, meta = load_golden("append_fp16")
    kp, vp = data["k_pool_before"].clone(), data["v_pool_before"].clone()
    with pytest.raises(IndexError):
        oracle.write_tokens_batch(kp, vp, 0, data["block_tables"], torch.tensor([2, 7, 14]),
                                  data["key_states"], data["value_states"])


def test_oracle_bad_block_id_raises():
    data, meta = load_golden("fp16_ragged")
    bt = data["block_tables"].clone()
    bt[1, 0] = 10_000
    with pytest.raises(IndexError):
        oracle.paged_decode(data["query"], data["key_cache"], data["value_cache"], bt, data["seq_lens"],
                            meta["scale"], len_offset=0)


def test_manifest_lists_every_fixture():
    names = {k for k in golden_manifest() if not k.startswith("_")}
    from conftest import GOLDEN

    assert names == {p.stem for p in GOLDEN.glob("*.npz")}
