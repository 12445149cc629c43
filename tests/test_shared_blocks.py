"""Zero-copy prefix sharing on the host: ``BlockRefAllocator`` (no GPU).

The allocator must answer exactly as the reference's PagedKVAllocator on the
recorded trace (tests/golden/allocator_trace.json, made by
make_allocator_trace.py from the reference itself) and pass the reference's
own allocator tests (tests/test_kv_allocator.py:14-70); the sharing tests
check that a prefix snapshot and a hit copy nothing, that copy-on-write copies
exactly the shared block a write touches, and that every block comes back.
"""

from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

import pytest
import torch

from llm_serving_runtime_b200.prefix_sharing import find_shared_prefixes
from llm_serving_runtime_b200.shared_blocks import BlockRefAllocator

from conftest import reference_root

GOLDEN = Path(__file__).resolve().parent / "golden"


def _trace_module():
    spec = importlib.util.spec_from_file_location("make_allocator_trace", GOLDEN / "make_allocator_trace.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_replays_the_reference_allocator_trace():
    trace = json.loads((GOLDEN / "allocator_trace.json").read_text())
    replay = _trace_module().replay
    assert len(trace["cases"]) == 3
    for case in trace["cases"]:
        alloc = BlockRefAllocator(case["total_blocks"], case["block_size_tokens"], case["bytes_per_token"])
        results = replay(alloc, case["ops"])
        for i, (got, want) in enumerate(zip(results, case["results"])):
            assert got == want, f"seed {case['seed']} call {i} {case['ops'][i]}: {got} != {want}"
        stats = alloc.stats()
        for key, want in case["stats"].items():
            assert stats[key] == pytest.approx(want), key


# ---- the reference's own allocator tests (tests/test_kv_allocator.py:14-70) ----

def test_capacity_exhaustion_and_reuse_after_free():
    alloc = BlockRefAllocator(total_blocks=4, block_size_tokens=8)
    assert alloc.allocate_for_tokens("req-a", 8) is not None
    assert alloc.allocate_for_tokens("req-b", 16) is not None
    assert alloc.allocate_for_tokens("req-c", 8) is not None
    assert alloc.allocate_for_tokens("req-d", 8) is None
    assert alloc.stats()["free_blocks"] == 0
    assert alloc.stats()["active_allocations"] == 3
    alloc.free_request("req-b")
    reused = alloc.allocate_for_tokens("req-d", 8)
    assert reused is not None and reused.request_id == "req-d"
    assert alloc.stats()["free_blocks"] == 1
    assert alloc.stats()["active_allocations"] == 3


def test_fragmentation_metrics_reflect_free_and_active_mix():
    alloc = BlockRefAllocator(total_blocks=6, block_size_tokens=4)
    alloc.allocate_for_tokens("req-a", 8)
    alloc.allocate_for_tokens("req-b", 4)
    before = alloc.stats()
    assert (before["used_blocks"], before["free_blocks"], before["active_allocations"]) == (3, 3, 2)
    assert before["fragmentation_ratio"] > 0.0
    alloc.free_request("req-a")
    after = alloc.stats()
    assert (after["used_blocks"], after["free_blocks"], after["active_allocations"]) == (1, 5, 1)
    assert after["fragmentation_ratio"] < before["fragmentation_ratio"]
    alloc.free_request("req-b")
    final = alloc.stats()
    assert (final["free_blocks"], final["active_allocations"], final["fragmentation_ratio"]) == (6, 0, 0.0)


def test_duplicate_allocation_returns_existing_allocation():
    alloc = BlockRefAllocator(total_blocks=2, block_size_tokens=4)
    first = alloc.allocate_for_tokens("req-a", 6)
    second = alloc.allocate_for_tokens("req-a", 2)
    assert first is second
    assert first.requested_tokens == 6
    assert alloc.stats()["active_allocations"] == 1


# ---- zero-copy sharing ----

def _insert_every_depth(alloc, block_ids, n_full):
    """What PrefixBlockCache.insert does with ``snapshot_blocks``: one entry per
    full-block depth (prefix_cache.py:214-246)."""
    return [alloc.snapshot_blocks(block_ids[:d]) for d in range(1, n_full + 1)]


def test_snapshot_and_hit_copy_nothing_and_every_block_comes_back():
    alloc = BlockRefAllocator(total_blocks=32, block_size_tokens=4)
    a = alloc.allocate_for_tokens("a", 12 + 2)  # a 12-token prompt (3 full blocks) + 2 new
    own = list(a.block_ids)
    free_before = alloc.stats()["free_blocks"]
    entries = _insert_every_depth(alloc, own, 3)
    assert alloc.stats()["free_blocks"] == free_before  # the snapshots took no block
    assert entries[-1] == own[:3]
    assert [alloc.ref_count(b) for b in own] == [4, 3, 2, 1]

    alloc.free_request("a")  # the cache keeps the prompt blocks alive
    assert [alloc.ref_count(b) for b in own] == [3, 2, 1, 0]
    assert alloc.stats()["free_blocks"] == free_before + 1

    hits = [alloc.allocate_for_tokens(f"r{i}", 12 + 8, borrowed_block_ids=entries[-1]) for i in range(3)]
    for h in hits:
        assert h.block_ids[:3] == own[:3]
        assert len(h.block_ids) == 5
    assert [alloc.ref_count(b) for b in own[:3]] == [6, 5, 4]
    assert alloc.stats()["borrowed_blocks_total"] == 9
    assert alloc.stats()["shared_blocks"] == 3

    for h in hits:
        alloc.free_request(h.request_id)
    for e in entries:
        alloc.release_blocks(e)
    s = alloc.stats()
    assert s["free_blocks"] == 32 and s["used_blocks"] == 0 and s["shared_blocks"] == 0
    assert s["cow_copies_total"] == 0


def test_copy_on_write_copies_only_the_shared_block_written():
    alloc = BlockRefAllocator(total_blocks=16, block_size_tokens=4)
    a = alloc.allocate_for_tokens("a", 8)
    entry = alloc.snapshot_blocks(a.block_ids[:2])
    alloc.free_request("a")
    b = alloc.allocate_for_tokens("b", 16, borrowed_block_ids=entry)
    copies = []

    def copy_blocks(src, dst):
        copies.append((list(src), list(dst)))

    # a rewrite of the last cached prompt token (position 7, block 1)
    pairs = alloc.make_writable("b", 7, 1, copy_blocks)
    assert len(pairs) == 1 and pairs[0][0] == entry[1]
    assert copies == [([entry[1]], [pairs[0][1]])]
    assert b.block_ids[1] == pairs[0][1] and b.block_ids[0] == entry[0]
    assert alloc.ref_count(entry[1]) == 1 and alloc.ref_count(pairs[0][1]) == 1
    # the block is private now, and the decode positions past the prefix are too
    assert alloc.make_writable("b", 7, 1, copy_blocks) == []
    assert alloc.make_writable("b", 8, 8, copy_blocks) == []
    # a write that spans the still-shared block 0 and block 1 copies block 0 only
    pairs = alloc.make_writable("b", 3, 2, copy_blocks)
    assert [p[0] for p in pairs] == [entry[0]]
    assert alloc.stats()["cow_copies_total"] == 2
    alloc.free_request("b")
    alloc.release_blocks(entry)
    assert alloc.stats()["free_blocks"] == 16


def test_copy_on_write_moves_the_pool_contents():
    torch.manual_seed(0)
    k_pool = torch.randn(12, 2, 2, 4, 8)  # [blocks, layers, kv heads, block size, head dim]
    v_pool = torch.randn(12, 2, 2, 4, 8)

    def copy_blocks(src_ids, dst_ids):
        for s, d in zip(src_ids, dst_ids):
            k_pool[d] = k_pool[s]
            v_pool[d] = v_pool[s]

    k_before, v_before = k_pool.clone(), v_pool.clone()
    alloc = BlockRefAllocator(total_blocks=12, block_size_tokens=4)
    a = alloc.allocate_for_tokens("a", 8)
    entry = alloc.snapshot_blocks(a.block_ids)
    b = alloc.allocate_for_tokens("b", 12, borrowed_block_ids=entry)
    (old, new), = alloc.make_writable("b", 6, 1, copy_blocks)
    assert torch.equal(k_pool[new], k_before[old]) and torch.equal(v_pool[new], v_before[old])
    assert torch.equal(k_pool[old], k_before[old])  # the shared original is untouched
    assert b.block_ids[1] == new


def test_copy_on_write_failures_change_nothing():
    alloc = BlockRefAllocator(total_blocks=3, block_size_tokens=4)
    a = alloc.allocate_for_tokens("a", 8)
    entry = alloc.snapshot_blocks(a.block_ids)
    b = alloc.allocate_for_tokens("b", 12, borrowed_block_ids=entry)  # takes the last free block
    table = list(b.block_ids)
    assert alloc.make_writable("b", 0, 8, lambda s, d: None) is None  # no free block for the copies
    assert b.block_ids == table and alloc.stats()["allocation_failures_total"] == 1

    alloc.free_request("a")
    alloc.free_request("b")
    alloc.release_blocks(entry)
    alloc = BlockRefAllocator(total_blocks=6, block_size_tokens=4)
    a = alloc.allocate_for_tokens("a", 4)
    entry = alloc.snapshot_blocks(a.block_ids)
    alloc.allocate_for_tokens("b", 8, borrowed_block_ids=entry)
    free_before = list(alloc._free)

    def broken_copy(src, dst):
        raise RuntimeError("copy failed")

    with pytest.raises(RuntimeError):
        alloc.make_writable("b", 0, 1, broken_copy)
    assert alloc._free == free_before  # the copies' blocks went back in their old order


def test_argument_errors():
    alloc = BlockRefAllocator(total_blocks=8, block_size_tokens=4)
    with pytest.raises(ValueError):
        alloc.allocate_for_tokens("x", 4, borrowed_block_ids=[3])  # nobody holds block 3
    with pytest.raises(IndexError):
        alloc.retain_blocks([8])
    alloc.allocate_for_tokens("a", 8)
    with pytest.raises(IndexError):
        alloc.make_writable("a", 6, 3, lambda s, d: None)  # runs past the 2-block table
    with pytest.raises(KeyError):
        alloc.make_writable("nobody", 0, 1, lambda s, d: None)
    assert alloc.make_writable("a", 0, 0, lambda s, d: None) == []
    with pytest.raises(ValueError):
        BlockRefAllocator(total_blocks=0, block_size_tokens=4)


def test_borrowers_form_one_cascade_group():
    """Rows that borrowed one entry share leading block ids, which is what the
    cascade decode's group finder keys on."""
    bs = 4
    alloc = BlockRefAllocator(total_blocks=64, block_size_tokens=bs)
    a = alloc.allocate_for_tokens("a", 16)
    entry = alloc.snapshot_blocks(a.block_ids[:3])
    alloc.free_request("a")
    rows = [alloc.allocate_for_tokens(f"r{i}", 12 + 4 * (i + 1), borrowed_block_ids=entry) for i in range(4)]
    lone = alloc.allocate_for_tokens("lone", 20)
    allocs = rows + [lone]
    width = max(len(x.block_ids) for x in allocs)
    tables = torch.tensor([x.block_ids + [0] * (width - len(x.block_ids)) for x in allocs], dtype=torch.int32)
    cached = torch.tensor([12 + 2 * i for i in range(4)] + [17], dtype=torch.int32)
    groups = find_shared_prefixes(tables, cached, block_size=bs, min_shared_tokens=8)
    assert groups.num_groups == 1
    assert groups.member_seqs.tolist() == [0, 1, 2, 3]
    assert groups.prefix_lens.tolist() == [12]
    assert groups.seq_group.tolist() == [0, 0, 0, 0, -1]


@pytest.fixture
def reference_prefix_cache():
    root = reference_root()
    if root is None:
        pytest.skip("reference checkout not available (set LLM_SERVING_RUNTIME_ROOT)")
    sys.path.insert(0, str(root))
    try:
        from runtime.phase2.prefix_cache import PrefixBlockCache
    except ImportError as exc:
        pytest.skip(f"reference prefix cache does not import here: {exc}")
    finally:
        sys.path.remove(str(root))
    return PrefixBlockCache


def test_reference_prefix_cache_on_zero_copy_snapshots(reference_prefix_cache):
    """The reference's radix cache, unchanged, with ``snapshot_blocks`` as its
    snapshot callback.  Its eviction is not exercised: ``_evict_if_needed``
    pops the entry and ``_remove_entry`` then deletes it again, a KeyError
    (prefix_cache.py:264-285); the entries' blocks are released by hand here,
    as its ``on_release_blocks`` callback would."""
    alloc = BlockRefAllocator(total_blocks=40, block_size_tokens=4)
    cache = reference_prefix_cache(block_size_tokens=4, max_entries=64)
    prompts = [list(range(100 * i, 100 * i + 12)) for i in range(3)]
    for i, p in enumerate(prompts):
        a = alloc.allocate_for_tokens(f"w{i}", len(p) + 1)
        used = alloc.stats()["used_blocks"]
        leaf = cache.insert(p, a.block_ids, {"backend": "paged", "seq_len": len(p)},
                            snapshot_blocks=alloc.snapshot_blocks)
        assert leaf is not None and leaf.block_ids == a.block_ids[:3]
        assert alloc.stats()["used_blocks"] == used  # no copy, no new block
        alloc.free_request(f"w{i}")
    assert alloc.stats()["used_blocks"] == 9  # three prompts of three full blocks, held by the cache
    hit = cache.lookup(prompts[2][:8] + [7, 7, 7, 7])
    assert hit.hit and hit.matched_tokens == 8
    b = alloc.allocate_for_tokens("b", 20, borrowed_block_ids=hit.entry.block_ids)
    assert b.block_ids[:2] == hit.entry.block_ids
    entries = list(cache._entries.values())
    assert len(entries) == 9
    for e in entries:
        alloc.release_blocks(e.block_ids)
    assert alloc.stats()["used_blocks"] == len(b.block_ids)  # the borrower keeps its prefix alive
    alloc.free_request("b")
    assert alloc.stats()["free_blocks"] == 40


def test_reference_counts_stay_consistent_under_random_sharing():
    """Seeded random mix of allocations, growth, snapshots, borrowing,
    copy-on-write, releases and frees.  After every call each block's count
    equals the holders that name it, and a block is free exactly when nobody
    holds it; at the end every block comes back."""
    import random

    rng = random.Random(2024)
    bs, total = 4, 64
    alloc = BlockRefAllocator(total_blocks=total, block_size_tokens=bs)
    entries: list[list[int]] = []
    live: list[str] = []
    n_req = 0

    def check():
        holders: dict[int, int] = {}
        for rid in live:
            for b in alloc.get_request_allocation(rid).block_ids:
                holders[b] = holders.get(b, 0) + 1
        for e in entries:
            for b in e:
                holders[b] = holders.get(b, 0) + 1
        for b in range(total):
            assert alloc.ref_count(b) == holders.get(b, 0), b
            assert (b in alloc._free_set) == (b not in holders), b
        assert len(alloc._free) == len(alloc._free_set) == total - len(holders)

    for _ in range(3000):
        r = rng.random()
        if r < 0.25 or not live:
            borrowed = rng.choice(entries) if entries and rng.random() < 0.6 else None
            a = alloc.allocate_for_tokens(f"q{n_req}", rng.randint(1, 10 * bs), borrowed_block_ids=borrowed)
            if a is not None:
                live.append(a.request_id)
            n_req += 1
        elif r < 0.35:
            alloc.allocate_for_tokens(rng.choice(live), rng.randint(1, 14 * bs))
        elif r < 0.5:
            a = alloc.get_request_allocation(rng.choice(live))
            n = rng.randint(1, len(a.block_ids))
            entries.append(alloc.snapshot_blocks(a.block_ids[:n]))
        elif r < 0.65:
            a = alloc.get_request_allocation(rng.choice(live))
            cap = len(a.block_ids) * bs
            start = rng.randrange(cap)
            alloc.make_writable(a.request_id, start, rng.randint(1, cap - start), lambda s, d: None)
        elif r < 0.8 and entries:
            alloc.release_blocks(entries.pop(rng.randrange(len(entries))))
        else:
            alloc.free_request(live.pop(rng.randrange(len(live))), reason="cancel")
        check()
    s = alloc.stats()
    assert s["cow_copies_total"] > 0 and s["borrowed_blocks_total"] > 0 and s["snapshot_blocks_total"] > 0
    for rid in live:
        alloc.free_request(rid)
    for e in entries:
        alloc.release_blocks(e)
    live.clear()
    entries.clear()
    check()
    assert alloc.stats()["free_blocks"] == total
