"""The integer bookkeeping the decode kernel's stream-K split relies on.

The kernel (llm_serving_runtime_b200/csrc/pa_decode_mma.cu) cuts one flat list
of (sequence, row, 16-token unit) into contiguous warp slices of equal cost --
a row costs its units plus ROW_COST for its start and end, unit u of a row
whose cost starts at rc sitting at cost position rc + ROW_COST + u -- and
merges rows cut by a slice boundary through per-warp partial slots and arrival
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


def _header_constant(name: str) -> int:
    import re
    from pathlib import Path

    text = (Path(__file__).resolve().parent.parent / "llm_serving_runtime_b200" / "csrc" / "pa_internal.h").read_text()
    return int(re.search(rf"constexpr int {name} = (\d+);", text).group(1))


# The row costs the kernel uses (plain decode and the cascade's suffix pass).
ROW_COST = _header_constant("kRowCostUnitsPlain")
ROW_COST_CASCADE = _header_constant("kRowCostUnitsCascade")


def _warp_of(x, nw, C):
    """The warp whose cost share [C*g//nw, C*(g+1)//nw) holds cost position x."""
    return ((x + 1) * nw - 1) // C


def simulate(row_units, min_units=8, nw_total=1184, row_cost=ROW_COST):
    """row_units: units of each row in flat order (0 = a row with nothing to
    attend, skipped).  Replays the kernel's slicing, piece and merge logic."""
    rows = [n for n in row_units]
    starts, cstarts = [], []  # flat unit start and cost start of each row
    acc = cacc = 0
    for n in rows:
        starts.append(acc)
        cstarts.append(cacc)
        acc += n
        cacc += n + (row_cost if n > 0 else 0)
    W, C = acc, cacc
    if W == 0:
        return []
    nw = min(nw_total, max(1, (C + min_units - 1) // min_units))

    def unit_at_cost(x):  # first flat unit whose cost position is >= x
        if x >= C:
            return W
        for r, n in enumerate(rows):
            if n > 0 and x < cstarts[r] + row_cost + n:
                return starts[r] + max(0, x - cstarts[r] - row_cost)
        return W

    counters, slots, owners, problems = {}, {}, {}, []
    for gw in range(nw):
        ws, we = unit_at_cost(C * gw // nw), unit_at_cost(C * (gw + 1) // nw)
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
                owner = _warp_of(cstarts[r] + row_cost + n - 1, nw, C)
                if owners.setdefault(owner, r) != r:
                    problems.append(("counter shared", owner))
                # the merger's choice of the first piece's slot
                g1 = _warp_of(cstarts[r] + row_cost, nw, C)
                if row_end and counters[r] == owner - g1 + 1:
                    g1_first = unit_at_cost(C * g1 // nw) == starts[r]
                    want = 2 * g1 + (0 if g1_first else 1)
                    if slots.get(want) != r:
                        problems.append(("first slot", r, want))
            u += 1
            if u == n:  # advance to the next row with units
                u = 0
                r += 1
                while r < len(rows) and rows[r] == 0:
                    r += 1
            cf += 1
    for r, c in counters.items():
        n = rows[r]
        expected = _warp_of(cstarts[r] + row_cost + n - 1, nw, C) - _warp_of(cstarts[r] + row_cost, nw, C) + 1
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
@pytest.mark.parametrize("row_cost", [ROW_COST, ROW_COST_CASCADE, 0, 5])
def test_split_bookkeeping_invariants(seed, row_cost):
    rng = random.Random(seed)
    for _ in range(150):
        rows = _decode_rows(rng, rng.randint(1, 24), rng.choice([1, 2, 8]), rng.choice([1, 2, 4]))
        assert simulate(rows, nw_total=rng.choice([8, 64, 1184]), row_cost=row_cost) == []


def test_ragged_rows_with_empty_ones():
    rng = random.Random(99)
    for _ in range(200):
        rows = [0 if rng.random() < 0.3 else rng.randint(1, 300) for _ in range(rng.randint(1, 80))]
        assert simulate(rows, nw_total=rng.choice([8, 64, 1184])) == []


def test_one_row_over_every_warp():
    assert simulate([4096 // 16 * 16]) == []
