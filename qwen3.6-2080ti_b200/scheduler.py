"""KV page bookkeeping for a shared page pool: block allocator, eviction and compaction planning.

The reference keeps one pool per request and per layer and never moves a page: its scheduler is a
request FIFO without block management (src/scheduler.py:61-276), pages are returned to a sorted free
list on release (src/decode_state.py:80-84) and the only page move is the whole-pool growth copy
(src/decode_state.py:58-69). With one shared pool per layer the host must own page placement, so this
module adds what a paged server needs around the kernels:

  BlockAllocator      sorted free list, lowest ids first (the reference pool's allocate/release
                      order, src/decode_state.py:72-84), over a fixed pool -- no growth copy;
  KVBlockManager      per-request page lists and lengths for one pool; appends allocate a page when a
                      request crosses a page boundary; finishing or evicting a request frees its pages;
                      produces the int32 block-table rows the kernels read;
  plan_compaction     (src, dst) page moves that pack the live pages into the lowest ids, with src and
                      dst disjoint, for pkv_copy_pages; the manager applies the id remap to its tables.

Everything here is host-side integer work on Python lists; the device side is kv_copy_pages and the
table upload. All pages of a request have the same id in every layer's pool, so one plan serves every
layer (pkv_copy_pages moves all layers in one launch).
"""

from __future__ import annotations

import bisect
from dataclasses import dataclass, field
from typing import Iterable, Sequence


class KVAllocationError(RuntimeError):
    """Raised when the pool has fewer free pages than a request needs."""


class BlockAllocator:
    """Free list over page ids [0, num_pages): allocate() hands out the lowest free ids."""

    def __init__(self, num_pages: int) -> None:
        if num_pages <= 0:
            raise ValueError("num_pages must be positive")
        self.num_pages = num_pages
        self._free: list[int] = list(range(num_pages))

    @property
    def free_blocks(self) -> list[int]:
        return list(self._free)

    @property
    def num_free(self) -> int:
        return len(self._free)

    @property
    def num_used(self) -> int:
        return self.num_pages - len(self._free)

    def allocate(self, count: int) -> list[int]:
        if count < 0:
            raise ValueError("count must be non-negative")
        if count > len(self._free):
            raise KVAllocationError(f"need {count} pages, {len(self._free)} of {self.num_pages} free")
        out = self._free[:count]
        del self._free[:count]
        return out

    def allocate_top(self, count: int) -> list[int]:
        """The highest free ids (a staging region at the top of the pool, e.g. for prefill writes that a
        later compaction moves down into holes)."""
        if count < 0:
            raise ValueError("count must be non-negative")
        if count > len(self._free):
            raise KVAllocationError(f"need {count} pages, {len(self._free)} of {self.num_pages} free")
        if count == 0:
            return []
        out = self._free[-count:]
        del self._free[-count:]
        return out

    def release(self, blocks: Iterable[int]) -> None:
        blocks = list(blocks)
        if not blocks:
            return
        for b in blocks:
            if not 0 <= b < self.num_pages:
                raise ValueError(f"page {b} outside the pool")
        merged = sorted(self._free + blocks)
        for a, b in zip(merged, merged[1:]):
            if a == b:
                raise ValueError(f"page {a} released twice")
        self._free = merged

    def take(self, blocks: Iterable[int]) -> None:
        """Marks specific free pages as used (the destinations of a compaction plan)."""
        for b in blocks:
            i = bisect.bisect_left(self._free, b)
            if i == len(self._free) or self._free[i] != b:
                raise ValueError(f"page {b} is not free")
            del self._free[i]


@dataclass
class RequestPages:
    pages: list[int] = field(default_factory=list)
    length: int = 0


def plan_compaction(live_pages: Iterable[int], free_pages: Sequence[int], max_moves: int | None = None
                    ) -> tuple[list[int], list[int]]:
    """Moves that pack live pages into the lowest ids.

    Every live page at or above the compacted boundary (the number of live pages) moves to the lowest
    free id below it, highest source first. Sources are live and destinations free, so the two lists
    are disjoint, which pkv_copy_pages requires. `max_moves` caps the plan (the highest pages move
    first, so a partial plan still lowers the high-water mark).
    """
    live = sorted(set(live_pages))
    boundary = len(live)
    sources = [p for p in reversed(live) if p >= boundary]
    holes = [p for p in free_pages if p < boundary]
    n = min(len(sources), len(holes))
    if max_moves is not None:
        n = min(n, max_moves)
    return sources[:n], sorted(holes)[:n]


class KVBlockManager:
    """Page lists of the requests that share one pool (per layer; every layer mirrors the same ids)."""

    def __init__(self, num_pages: int, block_size: int, max_blocks_per_request: int) -> None:
        if block_size <= 0 or max_blocks_per_request <= 0:
            raise ValueError("block_size and max_blocks_per_request must be positive")
        self.block_size = block_size
        self.max_blocks = max_blocks_per_request
        self.allocator = BlockAllocator(num_pages)
        self.requests: dict[str, RequestPages] = {}
        self.copies_planned = 0
        self.pages_released = 0

    # ---- request lifecycle ---------------------------------------------------------------------------
    def add_request(self, request_id: str, length: int, *, staging: bool = False) -> RequestPages:
        """Registers a request holding `length` tokens. `staging` places its pages at the top of the pool
        (highest free ids) for a later compaction to move down."""
        if request_id in self.requests:
            raise ValueError(f"duplicate request id {request_id}")
        if length < 0:
            raise ValueError("length must be non-negative")
        need = self._pages_for(length)
        if need > self.max_blocks:
            raise KVAllocationError(f"{request_id}: {length} tokens need {need} pages > {self.max_blocks}")
        pages = self.allocator.allocate_top(need)[::-1] if staging else self.allocator.allocate(need)
        entry = RequestPages(pages, length)
        self.requests[request_id] = entry
        return entry

    def slots(self, request_id: str, start: int, count: int) -> list[int]:
        """Slots of logical positions [start, start + count) of a request's existing pages."""
        pages = self.requests[request_id].pages
        bs = self.block_size
        return [pages[pos // bs] * bs + pos % bs for pos in range(start, start + count)]

    def slots_for_append(self, request_id: str, count: int) -> list[int]:
        """Slots of `count` new tokens of a request (allocating pages as it crosses page boundaries); the
        request's length advances. slot = page * block_size + offset, the positions the reference's
        append_blocks writes (src/decode_state.py:278-284)."""
        entry = self.requests[request_id]
        need = self._pages_for(entry.length + count)
        if need > self.max_blocks:
            raise KVAllocationError(f"{request_id}: table would exceed {self.max_blocks} pages")
        if need > len(entry.pages):
            entry.pages.extend(self.allocator.allocate(need - len(entry.pages)))
        out = self.slots(request_id, entry.length, count)
        entry.length += count
        return out

    def free_request(self, request_id: str) -> list[int]:
        """Returns a finished or evicted request's pages to the pool."""
        entry = self.requests.pop(request_id)
        self.allocator.release(entry.pages)
        self.pages_released += len(entry.pages)
        return entry.pages

    # ---- compaction --------------------------------------------------------------------------------------
    def live_pages(self) -> list[int]:
        return [p for entry in self.requests.values() for p in entry.pages]

    def high_water(self) -> int:
        """One past the highest page id in use (0 when empty)."""
        return max(self.live_pages(), default=-1) + 1

    def compact(self, max_moves: int | None = None) -> tuple[list[int], list[int]]:
        """Plans and applies a compaction: returns (src, dst) for pkv_copy_pages and rewrites the page
        lists. The caller must run the copy before the next kernel that reads the moved pages."""
        src, dst = plan_compaction(self.live_pages(), self.allocator.free_blocks, max_moves)
        if not src:
            return [], []
        remap = dict(zip(src, dst))
        for entry in self.requests.values():
            entry.pages = [remap.get(p, p) for p in entry.pages]
        self.allocator.take(dst)
        self.allocator.release(src)
        self.copies_planned += len(src)
        return src, dst

    # ---- tables ----------------------------------------------------------------------------------------------
    def block_table_rows(self, request_ids: Sequence[str]) -> list[list[int]]:
        """-1 padded rows of max_blocks entries, as the kernels read them (int32 on the device)."""
        rows = []
        for rid in request_ids:
            pages = self.requests[rid].pages
            rows.append(pages + [-1] * (self.max_blocks - len(pages)))
        return rows

    def lengths(self, request_ids: Sequence[str]) -> list[int]:
        return [self.requests[rid].length for rid in request_ids]

    def _pages_for(self, length: int) -> int:
        return (length + self.block_size - 1) // self.block_size


def shard_requests(lengths: Sequence[int], world_size: int) -> list[list[int]]:
    """Request indices per rank, balanced by total context (greedy: longest first onto the rank with the
    fewest tokens). Requests are independent, so this sharding needs no collective on the data path."""
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    loads = [0] * world_size
    out: list[list[int]] = [[] for _ in range(world_size)]
    for i in sorted(range(len(lengths)), key=lambda k: (-lengths[k], k)):
        r = min(range(world_size), key=lambda k: (loads[k], k))
        out[r].append(i)
        loads[r] += lengths[i]
    return [sorted(x) for x in out]
