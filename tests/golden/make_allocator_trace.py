"""Record the reference allocator's answers to a seeded sequence of calls.

Run where the reference runtime is importable:

    python tests/golden/make_allocator_trace.py --reference /path/to/llm-serving-runtime

It drives runtime.phase2.kv_allocator.PagedKVAllocator (kv_allocator.py:14-172)
through request allocations, growth, duplicate calls, frees with every reason,
detached (prefix snapshot) blocks, borrowing of those blocks by later requests
and their release, and writes each call with its result and the final
statistics to allocator_trace.json.  These are the calls on which the
reference's reference counts and ``BlockRefAllocator``'s agree (a request's own
blocks are never retained by a snapshot here), so the replay must match it
call for call.  The GPU box never runs this script.
"""

from __future__ import annotations

import argparse
import json
import random
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def make_ops(seed: int, n_ops: int, total_blocks: int, block_size: int) -> list[dict]:
    rng = random.Random(seed)
    ops: list[dict] = []
    live: list[str] = []
    next_req = 0
    for _ in range(n_ops):
        r = rng.random()
        if r < 0.3 or not live:
            ops.append({"op": "allocate", "request_id": f"req-{next_req}",
                        "tokens": rng.randint(1, 6 * block_size), "borrow": rng.random() < 0.3})
            live.append(f"req-{next_req}")
            next_req += 1
        elif r < 0.4:
            rid = rng.choice(live)
            ops.append({"op": "allocate", "request_id": rid, "tokens": rng.randint(1, 10 * block_size),
                        "borrow": False})
        elif r < 0.7:
            rid = live.pop(rng.randrange(len(live)))
            ops.append({"op": "free", "request_id": rid,
                        "reason": rng.choice(["complete", "cancel", "timeout", "error"])})
        elif r < 0.85:
            ops.append({"op": "detach", "n": rng.randint(0, 4)})
        else:
            ops.append({"op": "release_detached"})
    return ops


def replay(alloc, ops: list[dict]) -> list:
    """Run ``ops`` on ``alloc``; the same driver replays them in the test."""
    results = []
    snapshots: list[list[int]] = []
    for op in ops:
        kind = op["op"]
        if kind == "allocate":
            borrowed = snapshots[-1] if (op["borrow"] and snapshots) else None
            a = alloc.allocate_for_tokens(op["request_id"], op["tokens"], borrowed_block_ids=borrowed)
            results.append(None if a is None else list(a.block_ids))
        elif kind == "free":
            results.append(alloc.free_request(op["request_id"], reason=op["reason"]))
        elif kind == "detach":
            ids = alloc.allocate_detached_blocks(op["n"])
            if ids:
                snapshots.append(list(ids))
            results.append(ids)
        else:
            if snapshots:
                ids = snapshots.pop(0)
                alloc.release_blocks(ids)
                results.append(ids)
            else:
                results.append(None)
    return results


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from runtime.phase2.kv_allocator import PagedKVAllocator

    cases = []
    for seed, total, bs, n in ((1, 48, 4, 400), (2, 160, 16, 600), (3, 8, 8, 200)):
        ops = make_ops(seed, n, total, bs)
        alloc = PagedKVAllocator(total_blocks=total, block_size_tokens=bs, bytes_per_token=3)
        results = replay(alloc, ops)
        cases.append({"seed": seed, "total_blocks": total, "block_size_tokens": bs, "bytes_per_token": 3,
                      "ops": ops, "results": results, "stats": alloc.stats()})
    out = {"source": "runtime/phase2/kv_allocator.py:14-172 PagedKVAllocator",
           "generator": "tests/golden/make_allocator_trace.py", "cases": cases}
    (HERE / "allocator_trace.json").write_text(json.dumps(out, separators=(",", ":")) + "\n")
    print("wrote", HERE / "allocator_trace.json")


if __name__ == "__main__":
    main()
