"""The integer bookkeeping the decode kernel's stream-K split relies on.

The kernel (llm_serving_runtime_b200/csrc/pa_decode_mma.cu) cuts one flat list
of (sequence, row, 16-token unit) into equal contiguous warp slices and merges
rows cut by a slice boundary through per-warp partial slots and arrival
counters.  This test replays that arithmetic in Python over random ragged
batches and checks the invariants the kernel needs:
  * every split row receives exactly the number of pieces the merger expects
    (npieces = warp_of(last unit) - warp_of(first unit) + 1);
  * no two pieces share a partial slot (2*warp + first/last);
  * the counter index (the warp holding the row's last unit) is unique per split row,
    so the counter region does not depend on the batch.
"""

from __future__ import annotations

import random

import pytest


def _warp_of(x, nw, W):
    return ((x + 1) * nw - 1) // W


def simulate(ns, rows_per_b, nw_total, min_units=8):
    B = len(ns)
    P = [0]
    for n in ns:
        P.append(P[-1] + n)
    W = rows_per_b * P[B]
    if W == 0:
        return []
    nw = min(nw_total, max(1, (W + min_units - 1) // min_units))
    counters, slots, owners, problems = {}, {}, {}, []
    for gw in range(nw):
        ws, we = W * gw // nw, W * (gw + 1) // nw
        if ws >= we:
            continue
        lo, hi = 0, B - 1
        while lo < hi:
            mid = (lo + hi + 1) >> 1
            if rows_per_b * P[mid] <= ws:
                lo = mid
            else:
                hi = mid - 1
        b = lo
        n = P[b + 1] - P[b]
        off = ws - rows_per_b * P[b]
        r, u = off // n, off % n
        cf = ws
        first = from_start = False
        while cf < we:
            if u == 0 or cf == ws:
                first, from_start = cf == ws, u == 0
            row_end = u + 1 == n
            if (row_end or cf + 1 == we) and not (row_end and from_start):
                si = 2 * gw + (0 if first else 1)
                if si in slots:
                    problems.append(("slot reused", si))
                slots[si] = (b, r)
                counters[(b, r)] = counters.get((b, r), 0) + 1
                row_start = cf - u
                owner = _warp_of(row_start + n - 1, nw, W)
                if owners.setdefault(owner, (b, r)) != (b, r):
                    problems.append(("counter shared", owner))
            u += 1
            if u == n:
                u, r = 0, r + 1
                if r == rows_per_b:
                    r, b = 0, b + 1
                    while b < B and P[b + 1] == P[b]:
                        b += 1
                    if b < B:
                        n = P[b + 1] - P[b]
            cf += 1
    for (b, r), c in counters.items():
        n = P[b + 1] - P[b]
        rs = rows_per_b * P[b] + r * n
        expected = _warp_of(rs + n - 1, nw, W) - _warp_of(rs, nw, W) + 1
        if c != expected:
            problems.append(("piece count", (b, r), c, expected))
    return problems


@pytest.mark.parametrize("seed", range(6))
def test_split_bookkeeping_invariants(seed):
    rng = random.Random(seed)
    for _ in range(300):
        B = rng.randint(1, 60)
        ns = [rng.choice([0, 1, 2, 5, 30, 68, 200]) if rng.random() < 0.5 else rng.randint(0, 300)
              for _ in range(B)]
        rows = rng.choice([1, 2, 8, 16, 32])
        assert simulate(ns, rows, rng.choice([8, 64, 1184])) == []


def test_one_row_over_every_warp():
    assert simulate([4096], 8, 1184) == []
