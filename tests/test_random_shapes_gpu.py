"""Seeded random decode shapes against the oracle: dtype, head_dim, block size,
query heads per KV head, query tokens per sequence and ragged lengths drawn
together, so that combinations the hand-picked cases leave out get run too.
Every draw is fixed by its seed; the kernels reached are the split-K decode
kernels (fp16 / bf16 and fp32) and, for wide enough q_len * G, the
multi-query kernels."""

from __future__ import annotations

import random

import pytest
import torch

from _util import excess_err, max_err
from llm_serving_runtime_b200 import paged_attention_decode
from oracle import oracle
from test_decode_gpu import _synthetic

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

N_CASES = 100


def _draw(seed: int):
    rnd = random.Random(seed)
    dtype = rnd.choice([torch.bfloat16, torch.bfloat16, torch.float16, torch.float32])
    if dtype == torch.float32:
        D = rnd.choice([rnd.randint(1, 128), 32, 64, 128])
        bs = rnd.choice([4, 8, 16, 32, 64, 128])
    else:
        D = rnd.choice([8 * rnd.randint(1, 16), 64, 128, 128])
        bs = rnd.choice([8, 16, 16, 32, 64, 128, 256])
    Hkv = rnd.choice([1, 2, 4, 8])
    G = rnd.choice([1, 2, 4, 4, 7, 8, 16])
    q_len = rnd.choice([1, 1, 1, 2, 4, 8])
    B = rnd.randint(1, 40)
    lens = []
    for _ in range(B):
        kind = rnd.random()
        if kind < 0.1:
            lens.append(0)
        elif kind < 0.3:  # on or next to a block boundary
            lens.append(max(0, bs * rnd.randint(1, 40) + rnd.choice([-1, 0, 1])))
        else:
            lens.append(rnd.randint(1, 3000))
    return B, G * Hkv, Hkv, D, bs, dtype, lens, q_len


@pytest.mark.parametrize("seed", range(N_CASES))
def test_random_shape_vs_oracle(seed):
    B, Hq, Hkv, D, bs, dtype, lens, q_len = _draw(seed)
    q, kc, vc, bt, cl = _synthetic(B, Hq, Hkv, D, bs, dtype, lens, q_len, seed=1000 + seed)
    scale = max(D, 1) ** -0.5
    out = paged_attention_decode(q.to(DEV), kc.to(DEV), vc.to(DEV), bt.to(DEV), cl.to(DEV), scale, validate=True)
    ref = oracle.paged_decode(q, kc, vc, bt, cl, scale)
    shape = f"B={B} Hq={Hq} Hkv={Hkv} D={D} bs={bs} {dtype} q_len={q_len}"
    assert excess_err(out, ref) <= 0, f"{shape}: max abs err {max_err(out, ref)}"
