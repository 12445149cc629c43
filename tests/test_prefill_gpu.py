"""Multi-query attention over paged KV (chunked prefill / long speculative
verify): q_len new tokens per sequence, causal over them, on top of the cached
context — the same op as decode.  Checked against the oracle, which restates
the reference's eager masked attention (block_paged_attention.py:50-59)."""

from __future__ import annotations

import pytest
import torch

from _util import excess_err, max_err
from llm_serving_runtime_b200 import paged_attention_decode
from llm_serving_runtime_b200.workloads import make_workload
from oracle import oracle
from test_decode_gpu import _synthetic

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

CASES = [
    # (B, Hq, Hkv, D, bs, dtype, context_lens, q_len)
    (3, 32, 8, 128, 16, torch.bfloat16, [0, 100, 1000], 64),
    (2, 32, 8, 128, 16, torch.bfloat16, [0, 0], 512),        # pure prefill, nothing cached
    (3, 14, 2, 64, 16, torch.float16, [5, 300, 2000], 128),
    (2, 64, 8, 128, 16, torch.bfloat16, [17, 700], 33),       # G = 8, ragged chunk
    (2, 28, 4, 128, 16, torch.bfloat16, [3, 64], 16),          # G = 7
    (2, 8, 8, 64, 32, torch.float16, [40, 1], 100),            # MHA, block size 32
    (2, 8, 2, 128, 8, torch.bfloat16, [9, 250], 40),           # block size 8
    (2, 8, 2, 64, 16, torch.float32, [30, 200], 48),           # fp32 path
    # enough 128-row tiles (>= one per SM) to take the multi-query kernel:
    (10, 32, 8, 128, 16, torch.bfloat16, [0, 50, 300, 1000, 17, 0, 2000, 64, 5, 700], 256),
    (12, 14, 2, 64, 16, torch.float16, [1, 2, 3, 900, 100, 0, 33, 64, 65, 500, 8, 1200], 640),
    (6, 32, 8, 128, 8, torch.bfloat16, [3, 40, 0, 600, 129, 255], 200),   # block size 8
    (8, 64, 8, 128, 32, torch.bfloat16, [16, 0, 400, 31, 1000, 7, 65, 300], 96),  # G = 8, bs 32
    # head_dim 80 / 96 (padded to 128 tiles), on the multi-query kernels
    (10, 32, 8, 80, 16, torch.bfloat16, [0, 50, 300, 1000, 17, 0, 2000, 64, 5, 700], 256),
    (12, 14, 2, 96, 16, torch.float16, [1, 2, 3, 900, 100, 0, 33, 64, 65, 500, 8, 1200], 640),
    # 64- and 128-token blocks on the tcgen05 multi-query kernel
    (10, 32, 8, 128, 64, torch.bfloat16, [0, 50, 300, 1000, 17, 0, 2000, 64, 5, 700], 256),
    (10, 32, 8, 128, 128, torch.float16, [0, 50, 300, 1000, 17, 0, 2000, 64, 5, 700], 256),
    # long cached contexts: a 256-token chunk over up to 16k cached tokens
    (4, 32, 8, 128, 16, torch.bfloat16, [16000, 5, 9000, 12000], 256),
]


@pytest.mark.parametrize("B,Hq,Hkv,D,bs,dtype,lens,q_len", CASES)
def test_multi_query_chunks_vs_oracle(B, Hq, Hkv, D, bs, dtype, lens, q_len):
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len, seed=q_len + D)
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), D ** -0.5,
                                 validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


@pytest.mark.parametrize("D", [128, 64])
def test_bf16_values_far_beyond_fp16_range(D):
    """bf16 caches holding values fp16 cannot (up to 3e5, and 65280 / 65536
    at the edge of fp16's range) on the tcgen05 multi-query kernel: P is split
    into two bf16 parts, so the products keep ~16 bits of it at any scale."""
    B, Hq, Hkv, bs, q_len = 10, 32, 8, 16, 256
    lens = [0, 50, 300, 1000, 17, 0, 2000, 64, 5, 700]
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, torch.bfloat16, lens, q_len, seed=77 + D)
    v = vc.float()
    v[::3, :, 5, 7] = 3.0e5
    v[1::7, :, 2, 1] = -65536.0
    v[2::5, :, 9, 3] = 65280.0
    v[4::9, :, 11, 0] = -65280.0
    vc = v.to(torch.bfloat16)
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), D ** -0.5,
                                 validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_prefill_workload_with_append_sampled_rows():
    from _util import oracle_rows

    w = make_workload("prefill-llama3-8b", device=DEV)
    out = paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale,
                                 w.slot_mapping, w.new_key, w.new_value, validate=True)
    rows = [0, 5, 11]
    ref = oracle_rows(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale, w.q_len, rows)
    assert excess_err(out[rows], ref) <= 0, f"max abs err {max_err(out[rows], ref)}"


@pytest.mark.parametrize("B,Hq,Hkv,D,bs,dtype,lens,q_len", CASES[8:12])
def test_mma_multi_query_kernel_on_unaligned_output(B, Hq, Hkv, D, bs, dtype, lens, q_len):
    """Output rows that are 4- but not 16-byte aligned take the mma.sync
    multi-query kernel (the tcgen05 one stores whole 16-byte pieces); same
    results."""
    from llm_serving_runtime_b200 import _lib

    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len, seed=q_len + D + 1)
    buf = torch.full((B * Hq * q_len * D + 2,), float("nan"), dtype=dtype, device=DEV)
    out = buf[2:].view(B, Hq, q_len, D)
    paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), D ** -0.5, out=out,
                           validate=True)
    assert _lib.last_kernel() == "pa::prefill_mma_kernel"
    ref = oracle.paged_decode(q, kc, vc, bt, cl, D ** -0.5)
    assert excess_err(out, ref) <= 0, f"max abs err {max_err(out, ref)}"


def test_sm_pair_kernel_passes_the_same_cases():
    """The SM-pair tcgen05 kernel (cta_group::2, opt-in: PA_B200_MULTIQUERY=umma2)
    on this file's cases, in a child process (the library reads the policy
    once): every head_dim-128 case with 16-token or larger blocks takes it."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent
    env = dict(os.environ, PA_B200_MULTIQUERY="umma2")
    probe = ("import sys, torch; sys.path[:0] = ['.', 'tests']\n"
             "from llm_serving_runtime_b200 import paged_attention_decode, _lib\n"
             "from llm_serving_runtime_b200.workloads import make_workload\n"
             "w = make_workload('prefill-llama3-8b', device='cuda')\n"
             "paged_attention_decode(w.query, w.key_cache, w.value_cache, w.block_tables, w.context_lens, w.scale)\n"
             "torch.cuda.synchronize(); print(_lib.last_kernel())\n")
    kernel = subprocess.run([sys.executable, "-c", probe], cwd=here.parent, env=env, capture_output=True, text=True,
                            timeout=600)
    assert kernel.returncode == 0, kernel.stderr[-2000:]
    assert kernel.stdout.strip().endswith("pa::prefill_umma2_kernel")
    run = subprocess.run([sys.executable, "-m", "pytest", str(here / "test_prefill_gpu.py"), "-q", "-x",
                          "-p", "no:cacheprovider", "-k", "multi_query_chunks or prefill_workload"],
                         cwd=here.parent, env=env, capture_output=True, text=True, timeout=1200)
    assert run.returncode == 0, run.stdout[-3000:]


def _random_multi_query(seed):
    import random

    rnd = random.Random(seed)
    dtype = rnd.choice([torch.bfloat16, torch.float16])
    D = rnd.choice([64, 128, 128, 80, 96])
    bs = rnd.choice([8, 16, 16, 32, 64, 128])
    Hkv = rnd.choice([4, 8, 8])
    G = rnd.choice([4, 7, 8])
    q_len = rnd.choice([64, 128, 160, 256])
    B = rnd.randint(3, 10)
    lens = [rnd.choice([0, rnd.randint(1, 64), rnd.randint(0, 1200)]) for _ in range(B)]
    return B, G * Hkv, Hkv, D, bs, dtype, lens, q_len


@pytest.mark.parametrize("seed", range(20))
def test_random_multi_query_vs_oracle(seed):
    """Seeded random chunked-prefill shapes, most of them with enough 128-row
    tiles for the tcgen05 multi-query kernel, against the oracle on three rows
    (the first, the last and the longest)."""
    from _util import oracle_rows

    B, Hq, Hkv, D, bs, dtype, lens, q_len = _random_multi_query(seed)
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len, seed=3000 + seed)
    q, kc, vc, bt, cl = q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV)
    out = paged_attention_decode(q, kc, vc, bt, cl, D ** -0.5, validate=True)
    rows = sorted({0, B - 1, max(range(B), key=lambda b: lens[b])})
    ref = oracle_rows(q, kc, vc, bt, cl, D ** -0.5, q_len, rows)
    assert excess_err(out[rows], ref) <= 0, f"seed {seed}: max abs err {max_err(out[rows], ref)}"
