"""Seeded synthetic decode workloads (the five configurations of the benchmark).

Each generator returns a ``DecodeWorkload``: a paged KV cache with random
block placement, block tables, pre-append context lengths, the step's query
and new K/V rows, and the slot mapping of the new rows.  Lengths, tables and
slots come from a CPU ``torch.Generator`` (identical on every machine); the
bulk tensors are drawn on the target device from a device generator seeded the
same way.  The reference publishes no dataset for this path, so these seeded
inputs stand in for real traffic with the shapes and distributions of
BASELINE.json's configs.

Lengths follow the convention of the decode op: ``context_lens[b]`` counts the
tokens cached before the step; the step appends ``q_len`` tokens at positions
``context_lens[b] .. context_lens[b] + q_len - 1``; the attended length is
``L_b = context_lens[b] + q_len``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

__all__ = [
    "DecodeWorkload",
    "WorkloadSpec",
    "SPECS",
    "make_workload",
    "sample_lengths",
    "algorithmic_bytes",
    "attention_flops",
    "lpt_partition",
]


@dataclass(frozen=True)
class WorkloadSpec:
    name: str
    batch: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    dtype: torch.dtype
    q_len: int
    length_dist: str            # "uniform" | "loguniform" | "prefix"
    length_lo: int
    length_hi: int
    value_scale: float
    pool_slack: float = 0.0     # extra pool blocks as a fraction of the blocks in use
    prefix_groups: int = 0      # "prefix": sequences per group share prefix_tokens
    prefix_tokens: int = 0
    fixed_pool_blocks: int = 0  # config 1: a 160-block pool handed out in chunks
    seed: int = 1000


SPECS: dict[str, WorkloadSpec] = {
    # CPU-runnable, fp32
    "cfg1-fp32-small": WorkloadSpec("cfg1-fp32-small", 4, 8, 2, 64, 16, torch.float32, 1,
                                    "uniform", 1, 512, 1.0, fixed_pool_blocks=160, seed=1001),
    # Qwen2-0.5B shape, fp16
    "cfg2-qwen2-0.5b": WorkloadSpec("cfg2-qwen2-0.5b", 64, 14, 2, 64, 16, torch.float16, 1,
                                    "uniform", 128, 2048, 1.0, pool_slack=0.1, seed=1002),
    # Llama-3-8B shape, bf16 (the headline)
    "cfg3-llama3-8b": WorkloadSpec("cfg3-llama3-8b", 256, 32, 8, 128, 16, torch.bfloat16, 1,
                                   "loguniform", 256, 8192, 0.5, pool_slack=0.0, seed=1003),
    # prefix-shared speculative verify, q_len 4
    "cfg4-prefix-verify": WorkloadSpec("cfg4-prefix-verify", 512, 32, 8, 128, 16, torch.bfloat16, 4,
                                       "prefix", 16, 1024, 0.5, prefix_groups=16, prefix_tokens=1024,
                                       seed=1004),
    # Llama-3-70B shape, bf16
    "cfg5-llama3-70b": WorkloadSpec("cfg5-llama3-70b", 512, 64, 8, 128, 16, torch.bfloat16, 1,
                                    "uniform", 2048, 16384, 0.5, pool_slack=0.0, seed=1005),
    # chunked prefill over paged KV (next to the path): 512 new tokens per
    # sequence on top of 0..4096 cached ones, Llama-3-8B heads
    "prefill-llama3-8b": WorkloadSpec("prefill-llama3-8b", 16, 32, 8, 128, 16, torch.bfloat16, 512,
                                      "uniform", 0, 4096, 0.5, seed=1006),
}


@dataclass
class DecodeWorkload:
    spec: WorkloadSpec
    query: torch.Tensor          # [B, Hq, q_len, D]
    key_cache: torch.Tensor      # [num_blocks, Hkv, bs, D]
    value_cache: torch.Tensor
    block_tables: torch.Tensor   # int32 [B, max_blocks]
    context_lens: torch.Tensor   # int32 [B], tokens cached before the step
    new_key: torch.Tensor        # [B, Hkv, q_len, D]
    new_value: torch.Tensor
    slot_mapping: torch.Tensor   # int64 [B * q_len]
    scale: float
    rows: list[int]              # global row ids held by this workload
    unique_blocks: int           # distinct physical blocks referenced
    extra: dict = field(default_factory=dict)

    @property
    def q_len(self) -> int:
        return self.query.shape[2]

    @property
    def batch(self) -> int:
        return self.query.shape[0]

    def attended_lengths(self) -> torch.Tensor:
        return self.context_lens.to(torch.int64).cpu() + self.q_len

    def shared_prefixes(self):
        """The workload's prefix groups (``PrefixGroups``) on its device, or None."""
        spec = self.spec
        if not spec.prefix_groups:
            return None
        from .prefix_sharing import PrefixGroups

        per_group = spec.batch // spec.prefix_groups
        members: dict[int, list[int]] = {}
        for i, r in enumerate(self.rows):
            members.setdefault(r // per_group, []).append(i)
        groups = [members[k] for k in sorted(members)]
        return PrefixGroups.from_members(groups, [spec.prefix_tokens] * len(groups), self.batch,
                                         self.query.device)

    def to(self, device: str | torch.device) -> "DecodeWorkload":
        """Copy every tensor to ``device`` (bit-identical inputs on CPU and GPU)."""
        names = ("query", "key_cache", "value_cache", "block_tables", "context_lens",
                 "new_key", "new_value", "slot_mapping")
        moved = {k: getattr(self, k).to(device) for k in names}
        return DecodeWorkload(spec=self.spec, scale=self.scale, rows=list(self.rows),
                              unique_blocks=self.unique_blocks, extra=dict(self.extra), **moved)


def sample_lengths(spec: WorkloadSpec, batch: int | None = None) -> torch.Tensor:
    """Pre-append context lengths (int64 [B]) drawn from the spec's distribution."""
    B = spec.batch if batch is None else batch
    g = torch.Generator().manual_seed(spec.seed)
    if spec.length_dist == "uniform":
        return torch.randint(spec.length_lo, spec.length_hi + 1, (B,), generator=g, dtype=torch.int64)
    if spec.length_dist == "loguniform":
        u = torch.rand(B, generator=g, dtype=torch.float64)
        lo, hi = math.log(spec.length_lo), math.log(spec.length_hi)
        return torch.exp(lo + u * (hi - lo)).floor().to(torch.int64).clamp(spec.length_lo, spec.length_hi)
    if spec.length_dist == "prefix":
        suffix = torch.randint(spec.length_lo, spec.length_hi + 1, (B,), generator=g, dtype=torch.int64)
        return suffix + spec.prefix_tokens
    raise ValueError(spec.length_dist)


def lpt_partition(weights: list[int] | torch.Tensor, n_parts: int,
                  groups: list[list[int]] | None = None) -> list[list[int]]:
    """Greedy longest-processing-time partition of items (or groups of items)
    into ``n_parts`` bins of near-equal total weight.  Returns item ids per bin,
    each sorted ascending."""
    w = [int(x) for x in (weights.tolist() if isinstance(weights, torch.Tensor) else weights)]
    units = groups if groups is not None else [[i] for i in range(len(w))]
    order = sorted(range(len(units)), key=lambda u: -sum(w[i] for i in units[u]))
    loads = [0] * n_parts
    bins: list[list[int]] = [[] for _ in range(n_parts)]
    for u in order:
        k = min(range(n_parts), key=lambda j: (loads[j], j))
        bins[k].extend(units[u])
        loads[k] += sum(w[i] for i in units[u])
    return [sorted(b) for b in bins]


def _randn(shape, gen, device, dtype, scale):
    t = torch.randn(shape, generator=gen, device=device, dtype=torch.float32)
    if scale != 1.0:
        t.mul_(scale)
    return t.to(dtype)


def make_workload(
    spec: WorkloadSpec | str,
    *,
    device: str | torch.device = "cpu",
    rows: list[int] | None = None,
    global_batch: int | None = None,
    kv_heads: tuple[int, int] | None = None,
    seed_offset: int = 0,
) -> DecodeWorkload:
    """Build the workload (or the shard holding global ``rows``).

    ``global_batch`` overrides the spec's batch before sharding (weak-scaling
    runs draw N x batch rows and give each rank its LPT share).  ``kv_heads``
    = (first, count) keeps only those KV heads and their query heads (KV-head
    sharding).  The pool holds exactly the blocks the chosen rows use (+ slack).
    """
    if isinstance(spec, str):
        spec = SPECS[spec]
    device = torch.device(device)
    GB = spec.batch if global_batch is None else global_batch
    lens_all = sample_lengths(spec, GB)
    rows = list(range(GB)) if rows is None else list(rows)
    B = len(rows)
    lens = lens_all[rows]
    q = spec.q_len
    bs = spec.block_size
    G = spec.num_q_heads // spec.num_kv_heads
    h0, Hkv = (0, spec.num_kv_heads) if kv_heads is None else kv_heads
    Hq = Hkv * G
    D = spec.head_dim
    attended = lens + q
    nblk = (attended + bs - 1) // bs
    max_blocks = int(nblk.max().item())
    g = torch.Generator().manual_seed(spec.seed + 7919 * seed_offset + 1)

    tables = torch.zeros(B, max_blocks, dtype=torch.int64)
    if spec.length_dist == "prefix":
        # Sequences in one group share their first prefix_tokens // bs blocks.
        per_group = spec.batch // spec.prefix_groups
        pblk = spec.prefix_tokens // bs
        groups_here = sorted({r // per_group for r in rows})
        private = int((nblk - pblk).sum().item())
        total = len(groups_here) * pblk + private
        perm = torch.randperm(total, generator=g)
        cursor = 0
        prefix_ids = {}
        for grp in groups_here:
            prefix_ids[grp] = perm[cursor:cursor + pblk]
            cursor += pblk
        for i, r in enumerate(rows):
            tables[i, :pblk] = prefix_ids[r // per_group]
            n_priv = int(nblk[i]) - pblk
            tables[i, pblk:pblk + n_priv] = perm[cursor:cursor + n_priv]
            cursor += n_priv
        num_blocks = total
        unique = total
    elif spec.fixed_pool_blocks:
        num_blocks = spec.fixed_pool_blocks
        need = int(nblk.sum().item())
        if need > num_blocks:
            raise ValueError("fixed pool too small for the sampled lengths")
        perm = torch.randperm(num_blocks, generator=g)
        cursor = 0
        for i in range(B):
            n = int(nblk[i])
            tables[i, :n] = perm[cursor:cursor + n]
            cursor += n
        unique = need
    else:
        used = int(nblk.sum().item())
        num_blocks = int(math.ceil(used * (1.0 + spec.pool_slack)))
        perm = torch.randperm(num_blocks, generator=g)[:used]
        cursor = 0
        for i in range(B):
            n = int(nblk[i])
            tables[i, :n] = perm[cursor:cursor + n]
            cursor += n
        unique = used

    positions = lens[:, None] + torch.arange(q)[None, :]
    phys = torch.gather(tables, 1, positions // bs)
    slots = (phys * bs + positions % bs).reshape(-1)

    dgen = torch.Generator(device=device).manual_seed(spec.seed * 31 + seed_offset)
    dt = spec.dtype
    key_cache = _randn((num_blocks, Hkv, bs, D), dgen, device, dt, spec.value_scale)
    value_cache = _randn((num_blocks, Hkv, bs, D), dgen, device, dt, spec.value_scale)
    query = _randn((B, Hq, q, D), dgen, device, dt, spec.value_scale)
    new_key = _randn((B, Hkv, q, D), dgen, device, dt, spec.value_scale)
    new_value = _randn((B, Hkv, q, D), dgen, device, dt, spec.value_scale)
    return DecodeWorkload(
        spec=spec,
        query=query,
        key_cache=key_cache,
        value_cache=value_cache,
        block_tables=tables.to(torch.int32).to(device),
        context_lens=lens.to(torch.int32).to(device),
        new_key=new_key,
        new_value=new_value,
        slot_mapping=slots.to(device),
        scale=1.0 / math.sqrt(D),
        rows=rows,
        unique_blocks=unique,
        extra={"kv_heads": (h0, Hkv)},
    )


def attention_flops(w: DecodeWorkload) -> int:
    """Multiply-add FLOPs of QK^T and PV over the attended (causal) positions:
    4 * D * sum over query rows of the positions each attends."""
    B, Hq, q, D = w.query.shape
    L = w.attended_lengths()
    t = torch.arange(q)
    per_row = (L[:, None] - q + t[None, :] + 1).clamp_min(0)  # positions row (b, t) attends
    return int(4 * D * Hq * per_row.sum().item())


def algorithmic_bytes(w: DecodeWorkload, *, include_append: bool = True, unique: bool = False) -> int:
    """Minimum HBM bytes of one append + decode call.

    sum_b L_b*2*Hkv*D*e (KV read) + 2*B*q*Hq*D*e (Q read, O write)
    + sum_b ceil(L_b/bs)*4 + 4*B (tables, lengths)
    [+ 4*B*q*Hkv*D*e (new K/V read + cache write) + 8*B*q (slot mapping)].
    With ``unique`` a block shared by several sequences counts once.
    """
    e = w.query.element_size()
    B, Hq, q, D = w.query.shape
    Hkv, bs = w.key_cache.shape[1], w.key_cache.shape[2]
    L = w.attended_lengths()
    nblk = (L + bs - 1) // bs
    if unique:
        kv = w.unique_blocks * bs * 2 * Hkv * D * e
        # the last block of each row is only partly used; keep the token-exact
        # figure for private tails by subtracting the unused slots
        kv -= int((nblk * bs - L).sum().item()) * 2 * Hkv * D * e
    else:
        kv = int(L.sum().item()) * 2 * Hkv * D * e
    total = kv + 2 * B * q * Hq * D * e + int(nblk.sum().item()) * 4 + 4 * B
    if include_append:
        total += 4 * B * q * Hkv * D * e + 8 * B * q
    return int(total)
