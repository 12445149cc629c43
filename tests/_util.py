"""Helpers shared by the GPU parity tests: run the oracle on a subset of rows."""

from __future__ import annotations

import torch

from oracle import oracle

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-3}


def compact_rows(query, key_cache, value_cache, block_tables, context_lens, q_len, rows):
    """CPU copies of just what ``rows`` attend: their query rows, their blocks
    gathered into a small pool, and block tables renumbered into it."""
    rows_t = torch.as_tensor(rows, dtype=torch.long, device=block_tables.device)
    bs = key_cache.shape[2]
    lens = context_lens[rows_t].to(torch.int64) + q_len
    nblk = (lens + bs - 1) // bs
    maxb = int(nblk.max().item())
    tables = block_tables[rows_t, :maxb].to(torch.int64)
    ids = []
    new_tables = torch.zeros(len(rows), maxb, dtype=torch.int32)
    cursor = 0
    for i in range(len(rows)):
        n = int(nblk[i])
        ids.append(tables[i, :n])
        new_tables[i, :n] = torch.arange(cursor, cursor + n, dtype=torch.int32)
        cursor += n
    ids = torch.cat(ids)
    kc = key_cache[ids].cpu()
    vc = value_cache[ids].cpu()
    return query[rows_t].cpu(), kc, vc, new_tables, context_lens[rows_t].cpu()


def oracle_rows(query, key_cache, value_cache, block_tables, context_lens, scale, q_len, rows):
    q, kc, vc, bt, cl = compact_rows(query, key_cache, value_cache, block_tables, context_lens, q_len, rows)
    return oracle.paged_decode(q, kc, vc, bt, cl, scale, len_offset=q_len)


def max_err(out: torch.Tensor, ref_f32: torch.Tensor) -> float:
    """Max abs difference with the fp32 oracle rounded to the output dtype (the
    reference rounds its fp32 result the same way, paged_attention_triton.py:703)."""
    return (out.float().cpu() - ref_f32.to(out.dtype).float().cpu()).abs().max().item()


def ulp(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Spacing of ``dtype`` values at |x| (one rounding step of the output)."""
    a = x.abs().float().clamp_min(torch.finfo(dtype).tiny)
    return torch.exp2(torch.floor(torch.log2(a))) * torch.finfo(dtype).eps


def excess_err(out: torch.Tensor, ref_f32: torch.Tensor) -> float:
    """How far the output is beyond the bar.

    Both sides round an fp32 value to the output dtype, so where one rounding
    step of the dtype is itself coarser than the north-star tolerance (bf16
    outputs of magnitude >= 0.5, whose step is 2^-8 = 3.9e-3) a one-step
    disagreement is the finest resolvable answer.  The bar per element is
    max(TOL[dtype], one step of the dtype at the reference value).
    Returns max(err - bar); <= 0 means within the bar.
    """
    o = out.float().cpu()
    r = ref_f32.float().cpu()
    rr = r.to(out.dtype).float()
    err = (o - rr).abs()
    bar = torch.full_like(err, TOL[out.dtype])
    if out.dtype != torch.float32:
        bar = torch.maximum(bar, ulp(rr, out.dtype) * 1.0001)
    return (err - bar).max().item()


def split_row_pieces(context_lens, q_len: int, G: int, Hkv: int, *, nw_total: int = 148 * 8,
                     row_cost: int = 1, min_units: int = 8) -> dict[int, int]:
    """Pieces the decode kernel's stream-K split cuts each sequence's rows into.

    Replays the cost split of csrc/pa_decode_mma.cu: the flat order is sequence,
    kv head, 16-row group; a row (b, h, mg) holds the 16-token units its last
    query row attends and costs them plus ``row_cost`` (kRowCostUnitsPlain);
    warp w owns the cost positions [C*w/nw, C*(w+1)/nw).  Returns, per sequence
    b, the largest number of warps any of its rows spans (1 = never cut).
    """
    lens = [int(x) + q_len for x in torch.as_tensor(context_lens).cpu().tolist()]
    GQ = G * q_len
    NMG = (GQ + 15) // 16
    rows = []  # (b, cost of unit 0, units)
    cost = 0
    for b, L in enumerate(lens):
        for _h in range(Hkv):
            for mg in range(NMG):
                last_row = min(16 * mg + 15, GQ - 1)
                lim = L - q_len + last_row // G
                n = 0 if lim < 0 else (lim + 16) // 16
                if n > 0:
                    rows.append((b, cost + row_cost, n))
                    cost += n + row_cost
    C = cost
    if C == 0:
        return {}
    nw = min(nw_total, max(1, (C + min_units - 1) // min_units))

    def warp_at(x):
        return ((x + 1) * nw - 1) // C

    pieces: dict[int, int] = {}
    for b, c0, n in rows:
        k = warp_at(c0 + n - 1) - warp_at(c0) + 1
        pieces[b] = max(pieces.get(b, 1), k)
    return pieces
