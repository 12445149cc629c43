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


def simulate(row_units, min_units=8, nw_total=1184):
    """row_units: units of each row in flat order (0 = a row with nothing to
    attend, skipped).  Replays the kernel's slicing, piece and merge logic."""
    rows = [n for n in row_units]
    starts = []
    acc = 0
    for n in rows:
        starts.append(acc)
        acc += n
    W = acc
    if W == 0:
        return []
    nw = min(nw_total, max(1, (W + min_units - 1) // min_units))
    counters, slots, owners, problems = {}, {}, {}, []
    for gw in range(nw):
        ws, we = W * gw // nw, W * (gw + 1) // nw
        if ws >= we:
            continue
        # locate: the row holding flat index ws (rows with 0 units are skipped)
        r = max(i for i in range(len(rows)) if rows[i] > 0 and starts[i] <= ws)
        u = ws - starts[r]
        cf = ws
        first = from_start = False
        while cf < we:
            n = rows[r]
            if u == 0 or cf == ws:
                first, from_start = cf == ws, u == 0
            row_end = u + 1 == n
            if (row_end or cf + 1 == we) and not (row_end and from_start):
                si = 2 * gw + (0 if first else 1)
                if si in slots:
                    problems.append(("slot reused", si))
                slots[si] = r
                counters[r] = counters.get(r, 0) + 1
                owner = _warp_of(cf - u + n - 1, nw, W)
                if owners.setdefault(owner, r) != r:
                    problems.append(("counter shared", owner))
            u += 1
            if u == n:  # advance to the next row with units
                u = 0
                r += 1
                while r < len(rows) and rows[r] == 0:
                    r += 1
            cf += 1
    for r, c in counters.items():
        n, rs = rows[r], starts[r]
        expected = _warp_of(rs + n - 1, nw, W) - _warp_of(rs, nw, W) + 1
        if c != expected:
            problems.append(("piece count", r, c, expected))
    return problems


def _decode_rows(rng, B, Hkv, groups):
    """Row units in the kernel's flat order for random attended lengths."""
    out = []
    for _ in range(B):
        L = rng.choice([0, 1, 15, 16, 17]) if rng.random() < 0.3 else rng.randint(0, 5000)
        q_len = rng.choice([1, 4, 64])
        for _h in range(Hkv):
            for mg in range(groups):
                t_max = min(q_len - 1, mg * (16 // 4) + 3)  # G = 4: 4 tokens per 16-row group
                lim = L - q_len + t_max
                out.append(0 if lim < 0 else (lim + 16) // 16)
    return out


@pytest.mark.parametrize("seed", range(6))
def test_split_bookkeeping_invariants(seed):
    rng = random.Random(seed)
    for _ in range(150):
        rows = _decode_rows(rng, rng.randint(1, 24), rng.choice([1, 2, 8]), rng.choice([1, 2, 4]))
        assert simulate(rows, nw_total=rng.choice([8, 64, 1184])) == []


def test_ragged_rows_with_empty_ones():
    rng = random.Random(99)
    for _ in range(200):
        rows = [0 if rng.random() < 0.3 else rng.randint(1, 300) for _ in range(rng.randint(1, 80))]
        assert simulate(rows, nw_total=rng.choice([8, 64, 1184])) == []


def test_one_row_over_every_warp():
    assert simulate([4096 // 16 * 16]) == []
