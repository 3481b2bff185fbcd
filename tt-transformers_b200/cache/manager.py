"""The cache manager.

Layers that ask the same thing of the cache form a group: all keys (a paged request without
a window), a window of them (one with a window), or tensors of fixed size per request. A
request (parts.base.CacheRequest) says by itself which tensors it needs per page or per
live request, in which dtype, and how a mixer sees them; the manager knows no request kind
by name. Each paged group has its own page pool, its own device storage
{name: [units, pages + 1, *page shape]} and, per live request, its own list of pages (the
block table row). Pages are given back when the request ends, and, in a windowed group, as
soon as the window has passed them; given-back pages are handed out again first. Every
live request also owns a slot, which indexes the fixed-size state tensors {name: [units,
max_slots + 1, ...]} of the other groups (zeroed at admission; the last row belongs to no
request and takes what padded rows of a captured step write).

The reference keeps per-layer key and value tensors [num_blocks, kv_heads, block_size,
head_dim] and takes block tables from its caller
(src/tt_transformers/llm_runtime/paged_kv_cache.py:90-101,159-241); allocation, reuse and
release per request are this engine's own.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from ..parts.base import CacheRequest
from .pages import PagePool


class OutOfPages(RuntimeError):
    """A request needs more pages than its group's pool has free."""

    def __init__(self, request_id, group, needed, free):
        super().__init__(f"request {request_id!r} needs {needed} more pages in cache group {group}, {free} are free")
        self.request_id, self.group, self.needed, self.free = request_id, group, needed, free


class OutOfSlots(RuntimeError):
    """More requests are live than the engine has slots."""


@dataclass
class _Group:
    index: int
    request: CacheRequest
    units: List[int] = field(default_factory=list)     # layer-order entries that own a unit here
    pool: Optional[PagePool] = None                     # paged groups only
    storage: Optional[Dict[str, torch.Tensor]] = None   # name -> [units, pages + 1 | max_slots + 1, *shape]
    table: Optional[np.ndarray] = None    # int32 [max_slots, table_width]: the block table of every slot


@dataclass
class _Live:
    slot: int
    length: int = 0                                           # tokens whose keys are cached
    pages: Dict[int, List[int]] = field(default_factory=dict)  # group -> page of every page index (0: none)
    reserved_to: int = 0                                      # pages cover positions < reserved_to
    held_to: int = 0                                          # pages below this position stay even when unused (trim)


class CacheManager:
    ROLLBACK_SLACK = 1        # tokens by which a committed step may be taken back (the engine looks one step ahead)

    def __init__(self, cache_requests, page_size: int, num_pages: int, max_slots: int, max_seq_len: int,
                 device, dtype: torch.dtype, allocate_storage: bool = True):
        """cache_requests: per entry of the layer order a CacheRequest (PagedKV, SlotState or a kind of
        the caller's own), None, or the index of the entry whose unit it reads (as
        DecoderModel.cache_requests() gives). `dtype`: the compute dtype, for tensors whose request
        names none."""
        self.page_size, self.num_pages, self.max_slots = int(page_size), int(num_pages), int(max_slots)
        self.max_seq_len = int(max_seq_len)
        self.table_width = -(-self.max_seq_len // self.page_size)
        self.device, self.dtype = device, dtype
        self.groups: List[_Group] = []
        self._unit_of_entry: Dict[int, tuple] = {}             # entry -> (group index, unit index)
        by_request: Dict[object, _Group] = {}
        for entry, req in enumerate(cache_requests):
            if req is None or (isinstance(req, int) and not isinstance(req, bool)):
                continue
            several = isinstance(req, (tuple, list))         # a mixer made of mixers: a unit for each of them
            units = []
            for one in (req if several else (req,)):
                if not isinstance(one, CacheRequest):
                    raise TypeError(f"layer-order entry {entry}: {one!r} is no CacheRequest")
                if one not in by_request:
                    by_request[one] = _Group(index=len(self.groups), request=one)
                    self.groups.append(by_request[one])
                group = by_request[one]
                units.append((group.index, len(group.units)))
                group.units.append(entry)
            self._unit_of_entry[entry] = tuple(units) if several else units[0]
        for entry, req in enumerate(cache_requests):
            if isinstance(req, int) and not isinstance(req, bool):
                if req not in self._unit_of_entry:
                    raise ValueError(f"layer-order entry {entry} reads the cache of entry {req}, which has none")
                self._unit_of_entry[entry] = self._unit_of_entry[req]
        self.scratch_slot = self.max_slots                     # a state row that no request owns
        for g in self.groups:
            if g.request.paged:
                g.pool = PagePool(self.num_pages)
                g.table = np.zeros((self.max_slots, self.table_width), dtype=np.int32)
            if allocate_storage:
                rows = self.num_pages + 1 if g.request.paged else self.max_slots + 1
                g.storage = {name: torch.zeros(len(g.units), rows, *shape, dtype=dt or dtype, device=device)
                             for name, (shape, dt) in g.request.storage(self.page_size).items()}
        self._free_slots = list(range(self.max_slots - 1, -1, -1))
        self._live: Dict[object, _Live] = {}

    # ------------------------------------------------------------------ requests
    def is_live(self, request_id) -> bool:
        return request_id in self._live

    def live_requests(self):
        return list(self._live)

    def length(self, request_id) -> int:
        return self._live[request_id].length

    def slot(self, request_id) -> int:
        return self._live[request_id].slot

    @property
    def free_slots(self) -> int:
        return len(self._free_slots)

    def free_pages(self, group: int = None) -> int:
        """Free pages of one paged group, or the fewest over all paged groups."""
        pools = [g.pool for g in self.groups if g.pool is not None and (group is None or g.index == group)]
        return min((p.free_count for p in pools), default=1 << 30)

    def admit(self, request_id) -> int:
        """Give the request a slot (and zeroed fixed-size state). Raises OutOfSlots."""
        if request_id in self._live:
            raise ValueError(f"request {request_id!r} is live already")
        if not self._free_slots:
            raise OutOfSlots(f"all {self.max_slots} slots are taken; request {request_id!r} cannot be admitted")
        slot = self._free_slots.pop()
        live = _Live(slot=slot)
        for g in self.groups:
            if g.pool is not None:
                live.pages[g.index] = []
                g.table[slot, :] = 0
            elif g.storage is not None:
                for tensor in g.storage.values():
                    tensor[:, slot].zero_()
        self._live[request_id] = live
        return slot

    def room(self, request_id=None) -> int:
        """How many more tokens could be reserved right now: for a live request, beyond what
        it holds; for None, by a request that is not admitted yet."""
        P = self.page_size
        free = self.free_pages() * P
        if request_id is None:
            return free
        live = self._live[request_id]
        return free + (-(-live.reserved_to // P) * P - live.length)

    def pages_needed(self, request_id, new_length: int) -> int:
        """How many pages (in the most demanding group) reserve(new_length) would take."""
        live = self._live[request_id]
        have = -(-live.reserved_to // self.page_size)
        want = -(-new_length // self.page_size)
        return max(0, want - have)

    @staticmethod
    def bytes_per_page(cache_requests, page_size: int, dtype: torch.dtype) -> int:
        """Device bytes that one more page costs, over all paged groups (every group has the same number of pages)."""
        total, seen = 0, {}
        for entry in cache_requests:
            for req in (entry if isinstance(entry, (tuple, list)) else (entry,)):
                if isinstance(req, CacheRequest) and req.paged:
                    seen[req] = seen.get(req, 0) + 1
        for req, units in seen.items():
            for shape, dt in req.storage(page_size).values():
                count = 1
                for n in shape:
                    count *= n
                total += units * count * torch.empty(0, dtype=dt or dtype).element_size()
        return total

    def reserve(self, request_id, new_length: int, hold: bool = False) -> None:
        """Make sure pages cover positions below new_length, in every paged group, or take
        nothing and raise OutOfPages. hold: the pages stay with the request until it ends, also
        while it holds fewer tokens (an admission that reserves everything up front)."""
        live = self._live[request_id]
        if hold:
            self._reserve(live, request_id, new_length)
            live.held_to = max(live.held_to, new_length)
            return
        self._reserve(live, request_id, new_length)

    def _reserve(self, live, request_id, new_length: int) -> None:
        if new_length > self.max_seq_len:
            raise ValueError(f"request {request_id!r} would hold {new_length} tokens; the limit is {self.max_seq_len}")
        have = -(-live.reserved_to // self.page_size)
        want = -(-new_length // self.page_size)
        if want <= have:
            live.reserved_to = max(live.reserved_to, new_length)
            return
        need = want - have
        taken = []
        for g in self.groups:
            if g.pool is None:
                continue
            pages = g.pool.allocate(need)
            if pages is None:
                for gg, pp in taken:
                    gg.pool.free(pp)
                raise OutOfPages(request_id, g.index, need, g.pool.free_count)
            taken.append((g, pages))
        for g, pages in taken:
            live.pages[g.index].extend(pages)
            g.table[live.slot, have:want] = pages
        live.reserved_to = new_length

    def trim(self, request_id) -> None:
        """Give back pages that were reserved beyond what the request holds (a step that
        was reserved for but did not run)."""
        live = self._live[request_id]
        floor = max(live.length, live.held_to)
        keep = -(-floor // self.page_size)
        for g in self.groups:
            if g.pool is None:
                continue
            row = live.pages[g.index]
            extra = [p for p in row[keep:] if p != 0]
            if extra:
                g.pool.free(extra)
            del row[keep:]
            g.table[live.slot, keep:] = 0
        live.reserved_to = floor

    def commit(self, request_id, new_length: int) -> None:
        """The request now holds new_length tokens. Pages that a window has passed are freed."""
        live = self._live[request_id]
        if new_length > live.reserved_to:
            raise ValueError("commit beyond what was reserved")
        live.length = new_length
        for g in self.groups:
            if g.pool is None or (g.request.window is None and g.request.chunk is None):
                continue
            # the next query sits at position >= new_length and reads keys > position - window; a step
            # taken back (rollback) moves the request's end back by up to ROLLBACK_SLACK positions
            end = max(0, new_length - self.ROLLBACK_SLACK)
            first_needed = 0
            if g.request.window is not None:
                first_needed = max(0, end - g.request.window + 1)
            if g.request.chunk is not None:                  # ... and only keys of the chunk that holds it
                first_needed = max(first_needed, end // g.request.chunk * g.request.chunk)
            dead = first_needed // self.page_size            # pages wholly below first_needed
            row = live.pages[g.index]
            freed = [p for p in row[:dead] if p != 0]
            if freed:
                g.pool.free(freed)
                for i in range(dead):
                    row[i] = 0
                g.table[live.slot, :dead] = 0

    def has_windows(self) -> bool:
        return any(g.pool is not None and (g.request.window is not None or g.request.chunk is not None)
                   for g in self.groups)

    def rollback(self, request_id, length: int) -> None:
        """Take back a step that was committed ahead of time and then not used: the request holds
        `length` tokens again, pages beyond are given back. With windowed groups at most
        ROLLBACK_SLACK tokens can be taken back: that far behind its window a request keeps its pages."""
        live = self._live[request_id]
        if length > live.length:
            raise ValueError("rollback goes backwards only")
        if self.has_windows() and live.length - length > self.ROLLBACK_SLACK:
            raise RuntimeError(f"a cache with windowed groups can take back {self.ROLLBACK_SLACK} token(s), "
                               f"not {live.length - length}")
        live.length = length
        self.trim(request_id)

    def release(self, request_id) -> None:
        """The request ended: its pages and its slot are given back."""
        live = self._live.pop(request_id)
        for g in self.groups:
            if g.pool is not None:
                g.pool.free([p for p in live.pages[g.index] if p != 0])
                g.table[live.slot, :] = 0
        self._free_slots.append(live.slot)

    # ------------------------------------------------------------------ what a step needs
    def table_rows(self, group: int, slots: List[int], width: int = None) -> np.ndarray:
        """Block-table rows of the given slots: int32 [len(slots), width]."""
        rows = self.groups[group].table[slots]
        return rows if width is None else rows[:, :width]

    def paged_groups(self):
        return [g.index for g in self.groups if g.pool is not None]

    def view(self, entry: int, batch):
        """The cache view of a layer-order entry for this step (None if it has no cache)."""
        if entry not in self._unit_of_entry:
            return None
        where = self._unit_of_entry[entry]
        if where and isinstance(where[0], tuple):            # a unit for each mixer of a mixer made of mixers
            return tuple(self._view(gi, unit, batch) for gi, unit in where)
        return self._view(where[0], where[1], batch)

    def _view(self, gi: int, unit: int, batch):
        g = self.groups[gi]
        tensors = {name: tensor[unit] for name, tensor in g.storage.items()}
        if g.pool is not None:
            return g.request.view(tensors, block_table=batch.block_tables[gi], page_size=self.page_size)
        return g.request.view(tensors, slots=batch.seg_slot, slot_list=batch.seg_slot_list)

    # ------------------------------------------------------------------ invariants (tests)
    def audit(self) -> None:
        """Every page is free or held by exactly one live request; every slot likewise."""
        for g in self.groups:
            if g.pool is None:
                continue
            held = [p for live in self._live.values() for p in live.pages[g.index] if p != 0]
            if len(held) != len(set(held)):
                raise AssertionError(f"group {g.index}: a page is held twice")
            if len(held) != g.pool.held_count:
                raise AssertionError(f"group {g.index}: {g.pool.held_count} pages are out, {len(held)} are accounted for")
            free = set(g.pool._free)
            if free & set(held):
                raise AssertionError(f"group {g.index}: a held page is on the free list")
            if len(free) != len(g.pool._free):
                raise AssertionError(f"group {g.index}: a page is on the free list twice")
        slots = [live.slot for live in self._live.values()]
        if len(slots) != len(set(slots)) or set(slots) & set(self._free_slots):
            raise AssertionError("a slot is held twice")
        if len(slots) + len(self._free_slots) != self.max_slots:
            raise AssertionError("a slot was lost")
