"""Zero-copy prefix sharing: physical KV blocks held by reference count.

The reference copies blocks on every prefix-cache event:

- an insert snapshots the leading blocks of the inserting request into freshly
  allocated detached blocks, once per cached depth
  (runtime/phase2/prefix_cache.py:200-246 with the snapshot callback of
  worker_server.py:1264-1273);
- a paged hit allocates fresh blocks for the new request and copies the cached
  ones into them (``GpuKVBlockPool.copy_blocks``, worker_server.py:1436-1448).

``BlockRefAllocator`` keeps the reference allocator's interface and behaviour
(runtime/phase2/kv_allocator.py:14-172: first fit from a LIFO free list, the
same ids in the same order, ``None`` on exhaustion, the same statistics) but
counts EVERY holder of a block (the request that owns it, each prefix-cache
entry, each borrowing request), so a block goes back to the free list exactly
when its last holder lets go.  On top of that:

- ``snapshot_blocks(src)`` is the insert callback without a copy: the cache
  entry retains the request's own blocks;
- ``allocate_for_tokens(..., borrowed_block_ids=entry.block_ids)`` on a hit puts
  the cached blocks at the head of the new request's block table;
- ``make_writable(request_id, start_pos, n_tokens, copy_blocks)`` is the
  copy-on-write guard to call before a KV append: a block the write would touch
  that other holders still read is replaced by a private copy.  On the
  reference's hit path no write lands there (cached prefixes are whole blocks,
  prefix_cache.py:165, and the exact-logits rerun appends after the hydrated
  prefix, worker_server.py:1447-1455), so it copies nothing; it keeps a caller
  that rewrites a cached position (e.g. the last prompt token) from changing
  what the other holders read.

Rows that borrowed the same blocks then carry identical leading block ids,
which is what ``find_shared_prefixes`` groups for the cascade decode.  The
reference's allocator does not count a request's own blocks
(kv_allocator.py:96-110, :116-123), so retaining them in a snapshot and then
freeing the request would put them back on the free list while the cache still
reads them; that is why this is a separate allocator rather than a wrapper.

Host bookkeeping only (no device work besides the ``copy_blocks`` callback).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

__all__ = ["Allocation", "BlockRefAllocator"]


@dataclass
class Allocation:
    """A request's block table (kv_allocator.py:7-11)."""

    request_id: str
    block_ids: list[int]
    requested_tokens: int


class BlockRefAllocator:
    """Paged KV block allocator whose blocks are held by reference count.

    Not thread-safe, like the reference's: the worker calls it from its one
    scheduler thread (worker_server.py:1298).  ``make_writable``'s copy runs on
    the caller's current CUDA stream before the append that follows it there.
    """

    def __init__(self, total_blocks: int, block_size_tokens: int, bytes_per_token: int = 1) -> None:
        if total_blocks <= 0:
            raise ValueError("total_blocks must be > 0")
        if block_size_tokens <= 0:
            raise ValueError("block_size_tokens must be > 0")
        if bytes_per_token <= 0:
            raise ValueError("bytes_per_token must be > 0")
        self.total_blocks = total_blocks
        self.block_size_tokens = block_size_tokens
        self.bytes_per_token = bytes_per_token
        self.block_size_bytes = block_size_tokens * bytes_per_token
        # LIFO free list (popped from the end) plus its membership set.
        self._free: list[int] = list(range(total_blocks))
        self._free_set: set[int] = set(self._free)
        self._refs: dict[int, int] = {}
        self._owned: dict[str, Allocation] = {}
        self._allocations_total = 0
        self._allocation_failures_total = 0
        self._frees_total = 0
        self._frees_cancel_total = 0
        self._frees_timeout_total = 0
        self._frees_error_total = 0
        self._peak_used_blocks = 0
        self._peak_active_allocations = 0
        self._borrowed_blocks_total = 0
        self._snapshot_blocks_total = 0
        self._cow_copies_total = 0

    # ---- reference counts ----
    def ref_count(self, block_id: int) -> int:
        """Holders of a block: 0 when it is free."""
        return self._refs.get(int(block_id), 0)

    def is_shared(self, block_id: int) -> bool:
        return self.ref_count(block_id) > 1

    def _check_id(self, block_id: int) -> int:
        b = int(block_id)
        if not 0 <= b < self.total_blocks:
            raise IndexError(f"block id {b} outside the pool of {self.total_blocks} blocks")
        return b

    def _take_free(self, n: int) -> list[int]:
        ids = [self._free.pop() for _ in range(n)]
        for b in ids:
            self._free_set.discard(b)
            self._refs[b] = 1
        return ids

    def _drop_ref(self, block_id: int) -> None:
        refs = self._refs.get(block_id, 0)
        if refs <= 1:
            self._refs.pop(block_id, None)
            if block_id not in self._free_set:
                self._free.append(block_id)
                self._free_set.add(block_id)
        else:
            self._refs[block_id] = refs - 1

    def retain_blocks(self, block_ids: list[int]) -> None:
        """One more holder for each block (a free block leaves the free list)."""
        for raw in block_ids:
            b = self._check_id(raw)
            self._refs[b] = self._refs.get(b, 0) + 1
            if b in self._free_set:
                self._free_set.discard(b)
                self._free.remove(b)
        self._update_peaks()

    def release_blocks(self, block_ids: list[int]) -> None:
        """One holder fewer for each block; a block nobody holds is freed."""
        for raw in block_ids:
            self._drop_ref(self._check_id(raw))

    def allocate_detached_blocks(self, n_blocks: int) -> list[int] | None:
        """Blocks held by their caller's reference only, not by a request."""
        if n_blocks <= 0:
            return []
        if n_blocks > len(self._free):
            self._allocation_failures_total += 1
            return None
        ids = self._take_free(n_blocks)
        self._allocations_total += 1
        self._update_peaks()
        return ids

    def snapshot_blocks(self, src_block_ids: list[int]) -> list[int]:
        """Prefix-cache insert callback without a copy: the entry holds ``src``."""
        self.retain_blocks(src_block_ids)
        self._snapshot_blocks_total += len(src_block_ids)
        return list(src_block_ids)

    # ---- requests ----
    def allocate_for_tokens(
        self,
        request_id: str,
        token_capacity: int,
        *,
        borrowed_block_ids: list[int] | None = None,
    ) -> Allocation | None:
        """Blocks for ``token_capacity`` tokens; ``borrowed_block_ids`` (a
        prefix-cache hit) head the table and gain this request as a holder."""
        needed = max(1, math.ceil(token_capacity / self.block_size_tokens))
        existing = self._owned.get(request_id)
        if existing is not None:
            extra = needed - len(existing.block_ids)
            if extra <= 0:
                return existing
            if extra > len(self._free):
                self._allocation_failures_total += 1
                return None
            existing.block_ids.extend(self._take_free(extra))
            existing.requested_tokens = max(existing.requested_tokens, token_capacity)
            self._allocations_total += 1
            self._update_peaks()
            return existing
        borrowed = [self._check_id(b) for b in (borrowed_block_ids or [])][:needed]
        for b in borrowed:
            if self._refs.get(b, 0) == 0:
                raise ValueError(f"borrowed block {b} is not held by anyone")
        extra = needed - len(borrowed)
        if extra > len(self._free):
            self._allocation_failures_total += 1
            return None
        for b in borrowed:
            self._refs[b] += 1
        alloc = Allocation(request_id=request_id, block_ids=borrowed + self._take_free(extra),
                           requested_tokens=token_capacity)
        self._owned[request_id] = alloc
        self._borrowed_blocks_total += len(borrowed)
        self._allocations_total += 1
        self._update_peaks()
        return alloc

    def free_request(self, request_id: str, reason: str = "complete") -> bool:
        alloc = self._owned.pop(request_id, None)
        if alloc is None:
            return False
        for b in alloc.block_ids:
            self._drop_ref(b)
        self._frees_total += 1
        if reason == "cancel":
            self._frees_cancel_total += 1
        elif reason == "timeout":
            self._frees_timeout_total += 1
        elif reason == "error":
            self._frees_error_total += 1
        return True

    def get_request_allocation(self, request_id: str) -> Allocation | None:
        return self._owned.get(request_id)

    def make_writable(self, request_id: str, start_pos: int, n_tokens: int,
                      copy_blocks: Callable[[list[int], list[int]], None]) -> list[tuple[int, int]] | None:
        """Copy-on-write before writing tokens [start_pos, start_pos + n_tokens).

        Every block of the request's table that the write touches and that
        another holder still reads is replaced by a fresh private block, after
        ``copy_blocks(src_ids, dst_ids)`` (e.g. ``GpuKVBlockPool.copy_blocks``)
        copied its contents.  Returns the (old, new) pairs, or ``None`` when the
        free list cannot supply the copies (nothing is changed then).  Raises
        KeyError for an unknown request and IndexError when the write runs past
        the table, as the append itself would (paged_kv_kernel.py:221-222).
        """
        alloc = self._owned.get(request_id)
        if alloc is None:
            raise KeyError(f"no allocation for request {request_id!r}")
        if n_tokens <= 0:
            return []
        if start_pos < 0:
            raise IndexError("negative write position")
        first = start_pos // self.block_size_tokens
        last = (start_pos + n_tokens - 1) // self.block_size_tokens
        if last >= len(alloc.block_ids):
            raise IndexError("block table underrun during write")
        logical = [j for j in range(first, last + 1) if self._refs.get(alloc.block_ids[j], 0) > 1]
        if not logical:
            return []
        if len(logical) > len(self._free):
            self._allocation_failures_total += 1
            return None
        old = [alloc.block_ids[j] for j in logical]
        new = self._take_free(len(logical))
        try:
            copy_blocks(old, new)
        except BaseException:
            for b in reversed(new):  # back onto the free list in their old order
                self._drop_ref(b)
            raise
        for j, b_old, b_new in zip(logical, old, new):
            alloc.block_ids[j] = b_new
            self._drop_ref(b_old)
        self._cow_copies_total += len(logical)
        self._update_peaks()
        return list(zip(old, new))

    # ---- statistics (kv_allocator.py:142-172, plus the sharing counters) ----
    def _update_peaks(self) -> None:
        used = self.total_blocks - len(self._free)
        self._peak_used_blocks = max(self._peak_used_blocks, used)
        self._peak_active_allocations = max(self._peak_active_allocations, len(self._owned))

    def stats(self) -> dict[str, float | int]:
        used = self.total_blocks - len(self._free)
        largest = max((len(a.block_ids) for a in self._owned.values()), default=0)
        free = len(self._free)
        frag = max(0.0, 1.0 - free / (free + largest)) if free > 0 and largest > 0 else 0.0
        return {
            "total_blocks": self.total_blocks,
            "free_blocks": free,
            "used_blocks": used,
            "used_pct": used / self.total_blocks * 100.0,
            "block_size_tokens": self.block_size_tokens,
            "bytes_per_token": self.bytes_per_token,
            "block_size_bytes": self.block_size_bytes,
            "total_kv_bytes": self.total_blocks * self.block_size_bytes,
            "free_kv_bytes": free * self.block_size_bytes,
            "used_kv_bytes": used * self.block_size_bytes,
            "active_allocations": len(self._owned),
            "peak_used_blocks": self._peak_used_blocks,
            "peak_kv_bytes": self._peak_used_blocks * self.block_size_bytes,
            "peak_active_allocations": self._peak_active_allocations,
            "allocations_total": self._allocations_total,
            "allocation_failures_total": self._allocation_failures_total,
            "frees_total": self._frees_total,
            "frees_cancel_total": self._frees_cancel_total,
            "frees_timeout_total": self._frees_timeout_total,
            "frees_error_total": self._frees_error_total,
            "fragmentation_ratio": frag,
            "shared_blocks": sum(1 for r in self._refs.values() if r > 1),
            "borrowed_blocks_total": self._borrowed_blocks_total,
            "snapshot_blocks_total": self._snapshot_blocks_total,
            "cow_copies_total": self._cow_copies_total,
        }
