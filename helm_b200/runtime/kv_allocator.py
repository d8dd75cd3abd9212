"""Page allocator over one page pool per tier (drop-in for helm.runtime.kv_allocator).

Mirrors KVAllocator of HELM (helm/runtime/kv_allocator.py:6-163): the same
constructor, free lists, page ids, batch reserves (8 GPU / 16 CPU pages), LIFO
reuse, DEAD pages after GPU->CPU moves and usage report.  What differs is the
storage: instead of one torch.empty pair per page, every page of a tier is a
slot of a single pool tensor

    pool[slot][kv][head][token][dim]      (kv 0 = K, 1 = V)

on the device (HBM) or in page-locked host memory (the cold tier), so a page
is one contiguous run that the copy engine moves in one transfer and the
attention kernel addresses as base + slot * page_bytes.  KVPage.k_tensor /
v_tensor are [1, H, P, D] views of the slot, exactly the reference's page
shape.  Pools grow by doubling; a grown pool re-points the views of every
live page (a caller holding an old view keeps reading the old storage).

Slots are this module's own detail (the reference has none), so the host tier
places evicted pages by layer: each layer fills an arena of ARENA_SLOTS
consecutive slots in token order, and the cold pages of one layer then move to
the device in a few long copies instead of one copy per page.
"""
from __future__ import annotations

from typing import Optional

import torch

_HOST_GROW_MIN = 16
_DEVICE_GROW_MIN = 8
ARENA_SLOTS = 64


class PagePool:
    """One tier's slot storage: [capacity, 2, H, P, D] on `device`."""

    def __init__(self, device: torch.device, num_kv_heads: int, page_size: int, head_dim: int,
                 dtype: torch.dtype, capacity: int = 0, allocator=None):
        self.device = device
        self.allocator = allocator
        self.shape_tail = (2, num_kv_heads, page_size, head_dim)
        self.dtype = dtype
        self.storage: Optional[torch.Tensor] = None
        self.capacity = 0
        self.next_slot = 0
        self.free_slots: list[int] = []      # slots released by DEAD pages
        self.pending_release: list[int] = []  # released once deferred copies are issued
        self.pages: dict[int, object] = {}    # slot -> page owning it (for re-pointing)
        self.staging: list[int] = []          # slots reserved for cold-page staging
        self.window: set = set()              # slots reserved as all-GPU decode windows
        self.page_bytes = 2 * num_kv_heads * page_size * head_dim * \
            torch.tensor([], dtype=dtype).element_size()
        self._arenas: dict = {}               # key -> (next slot, end) (host tier)
        self._carve_from = 0
        if capacity > 0:
            self._resize(capacity)

    @property
    def is_host(self) -> bool:
        return self.device.type != "cuda"

    def _alloc(self, capacity: int) -> torch.Tensor:
        shape = (capacity,) + self.shape_tail
        if self.is_host:
            pin = torch.cuda.is_available()
            return torch.empty(shape, dtype=self.dtype, pin_memory=pin)
        return torch.empty(shape, dtype=self.dtype, device=self.device)

    def _resize(self, capacity: int) -> None:
        new = self._alloc(capacity)
        if self.storage is not None and self.next_slot > 0:
            if not self.is_host:
                torch.cuda.synchronize(self.device)
            new[: self.next_slot].copy_(self.storage[: self.next_slot])
            if not self.is_host:
                torch.cuda.synchronize(self.device)
        self.storage = new
        self.capacity = capacity
        for slot, page in self.pages.items():
            page.k_tensor = new[slot, 0].unsqueeze(0)
            page.v_tensor = new[slot, 1].unsqueeze(0)

    def reserve_capacity(self, n_more: int) -> None:
        """Ensures `n_more` fresh slots exist beyond next_slot."""
        need = self.next_slot + n_more
        if need > self.capacity:
            grow = max(need, 2 * self.capacity,
                       _HOST_GROW_MIN if self.is_host else _DEVICE_GROW_MIN)
            self._resize(grow)

    def acquire(self, page) -> int:
        slot = -1
        while self.free_slots:
            s = self.free_slots.pop()
            if s not in self.pages:      # entries of slots an arena took since are stale
                slot = s
                break
        if slot < 0:
            self.reserve_capacity(1)
            slot = self.next_slot
            self.next_slot += 1
        self._bind(page, slot)
        return slot

    def _bind(self, page, slot: int) -> None:
        self.pages[slot] = page
        page.slot = slot
        page.k_tensor = self.storage[slot, 0].unsqueeze(0)
        page.v_tensor = self.storage[slot, 1].unsqueeze(0)

    # -- per-layer arenas (host tier) -------------------------------------------
    def place_in_arena(self, page, key) -> None:
        """Re-binds a page just allocated as an eviction target to the next slot
        of `key`'s arena (consecutive slots per layer, in eviction order)."""
        nxt, end = self._arenas.get(key, (0, 0))
        if nxt >= end or not self._takeable(nxt, page):
            nxt = self._carve(page)
            end = nxt + ARENA_SLOTS
        self._rebind(page, nxt)
        self._arenas[key] = (nxt + 1, end)

    def forget_arenas(self, keys) -> None:
        for k in keys:
            self._arenas.pop(k, None)
        if not self._arenas:
            self._carve_from = 0

    def _takeable(self, s: int, page) -> bool:
        if s >= self.next_slot:
            return True
        owner = self.pages.get(s)
        if owner is None:
            return s not in self.staging and s not in self.window
        return owner is page or owner.state == "FREE"

    def _carve(self, page) -> int:
        """Start of ARENA_SLOTS consecutive takeable slots: the first such run at
        or after the carve cursor, else fresh slots at the end of the pool."""
        n = ARENA_SLOTS
        run = 0
        s = self._carve_from
        while s < self.next_slot:
            run = run + 1 if self._takeable(s, page) else 0
            s += 1
            if run == n:
                self._carve_from = s
                return s - n
        start = self.next_slot - run
        self.reserve_capacity(n - run)
        self.next_slot = start + n
        self._carve_from = self.next_slot
        return start

    def _rebind(self, page, s: int) -> None:
        old = page.slot
        if s == old:
            return
        owner = self.pages.get(s)
        if owner is not None:          # a free page: the two trade slots
            self._bind(owner, old)
        else:
            if self.pages.get(old) is page:
                del self.pages[old]
            self.free_slots.append(old)
        self._bind(page, s)

    def release(self, slot: int, deferred: bool) -> None:
        self.pages.pop(slot, None)
        (self.pending_release if deferred else self.free_slots).append(slot)

    def flush_pending(self) -> None:
        self.free_slots.extend(self.pending_release)
        self.pending_release.clear()

    def reserve_window(self, n: int) -> list[int]:
        """n fresh slots reserved for a manager's decode window (never given to
        pages until release_window).  Raises when the pool cannot grow."""
        self.reserve_capacity(n)
        slots = list(range(self.next_slot, self.next_slot + n))
        self.next_slot += n
        self.window.update(slots)
        return slots

    def release_window(self, slots) -> None:
        for s in slots:
            if s in self.window:
                self.window.discard(s)
                self.free_slots.append(s)

    def staging_slots(self, n: int) -> list[int]:
        """At least n slots reserved for cold-page staging (never given to pages)."""
        while len(self.staging) < n:
            self.reserve_capacity(1)
            self.staging.append(self.next_slot)
            self.next_slot += 1
        return self.staging[:n]


class KVAllocator:
    """Drop-in for helm.runtime.kv_allocator.KVAllocator (kv_allocator.py:6-163).

    Extra keyword arguments (not in the reference): initial pool capacities in
    pages for the device and host tiers.
    """

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, page_size: int = 64,
                 dtype=torch.bfloat16, *, gpu_pool_pages: int = 0, cpu_pool_pages: int = 0):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.page_size = page_size
        self.dtype = dtype
        self.gpu_free_pool: list = []
        self.cpu_free_pool: list = []
        self.gpu_total_pages = 0
        self.cpu_total_pages = 0
        self._next_page_id = 0
        self._pools: dict = {}
        self._initial = {"cuda": gpu_pool_pages, "cpu": cpu_pool_pages}
        self._bpp_key = None
        self._bpp = 0
        # When a list, GPU->CPU data copies are recorded here instead of being
        # issued (KVCacheManager defers them until the pages' data is written).
        self._deferred: Optional[list] = None

    # ------------------------------------------------------------- pools --
    def pool_for(self, device: torch.device) -> PagePool:
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        key = (device.type, device.index)
        pool = self._pools.get(key)
        if pool is None:
            pool = PagePool(device, self.num_kv_heads, self.page_size, self.head_dim, self.dtype,
                            self._initial["cuda" if device.type == "cuda" else "cpu"],
                            allocator=self)
            self._pools[key] = pool
        return pool

    def pools(self):
        return list(self._pools.values())

    def forget_arenas(self, keys) -> None:
        keys = list(keys)
        for pool in self._pools.values():
            pool.forget_arenas(keys)

    @property
    def bytes_per_page(self) -> int:
        if self._bpp_key != self.dtype:
            self._bpp = 2 * self.num_kv_heads * self.page_size * self.head_dim * \
                torch.tensor([], dtype=self.dtype).element_size()
            self._bpp_key = self.dtype
        return self._bpp

    # --------------------------------------------------- reference API --
    def _create_page(self, device: torch.device):
        from .kv_cache import KVPage
        device = torch.device(device)
        page = KVPage(page_id=self._next_page_id, layer_id=-1, start_token=0, used_tokens=0,
                      capacity_tokens=self.page_size, k_tensor=None, v_tensor=None,
                      device=device, state="FREE")
        pool = self.pool_for(device)
        pool.acquire(page)
        page.pool = pool
        self._next_page_id += 1
        if device.type == "cuda":
            self.gpu_total_pages += 1
        else:
            self.cpu_total_pages += 1
        return page

    def reserve_batch(self, batch_size: int, device: torch.device):
        """Adds `batch_size` free pages on `device` (kv_allocator.py:50-57)."""
        device = torch.device(device)
        pool = self.pool_for(device)
        pool.reserve_capacity(max(0, batch_size - len(pool.free_slots)))
        for _ in range(batch_size):
            page = self._create_page(device)
            (self.gpu_free_pool if device.type == "cuda" else self.cpu_free_pool).append(page)

    def allocate(self, device: torch.device):
        """Pops the most recently freed page, growing the pool in batches of 8
        (GPU) or 16 (CPU) pages when empty (kv_allocator.py:59-78)."""
        device = torch.device(device)
        if device.type == "cuda":
            if not self.gpu_free_pool:
                self.reserve_batch(8, device)
            page = self.gpu_free_pool.pop()
            page.state = "GPU"
        else:
            if not self.cpu_free_pool:
                self.reserve_batch(16, device)
            page = self.cpu_free_pool.pop()
            page.state = "CPU"
        page.generation += 1  # content changes from here on (cold-page staging key)
        page.layer_id = -1
        page.start_token = 0
        page.used_tokens = 0
        page.device = device
        return page

    def free(self, page):
        """Returns a page to its free list; its data is left as is (kv_allocator.py:80-93)."""
        page.state = "FREE"
        page.layer_id = -1
        page.start_token = 0
        page.used_tokens = 0
        if page.device.type == "cuda":
            self.gpu_free_pool.append(page)
        else:
            self.cpu_free_pool.append(page)

    def move_page(self, page, target_device: torch.device, *, arena_key=None):
        """Moves a page to another tier (kv_allocator.py:95-144).  The data of the
        used tokens is copied by the copy engine on the current stream.  A GPU
        page that leaves for the host becomes DEAD and its slot returns to the
        device pool (the reference frees its VRAM).  arena_key (not in the
        reference): the host slot comes from that key's arena."""
        target_device = torch.device(target_device)
        if page.device == target_device:
            return page
        new_page = self.allocate(target_device)
        if arena_key is not None and target_device.type != "cuda":
            new_page.pool.place_in_arena(new_page, arena_key)
        used = page.used_tokens
        if used > 0:
            self._copy_page(new_page, page)
        new_page.layer_id = page.layer_id
        new_page.start_token = page.start_token
        new_page.used_tokens = used
        new_page.device = target_device
        if page.device.type == "cuda" and target_device.type != "cuda":
            pool = page.pool
            page.k_tensor = torch.empty(0, dtype=self.dtype)
            page.v_tensor = torch.empty(0, dtype=self.dtype)
            page.state = "DEAD"
            self.gpu_total_pages -= 1
            if pool is not None and page.slot >= 0:
                pool.release(page.slot, deferred=self._deferred is not None)
            page.slot = -1
            page.pool = None
        else:
            self.free(page)
        return new_page

    def _copy_page(self, dst, src) -> None:
        """Copies a whole page slot (K and V of every head).  Device<->host copies
        go through the native library (copy engine, current stream)."""
        if self._deferred is not None and src.device.type == "cuda" and dst.device.type != "cuda":
            self._deferred.append((dst, src.pool, src.slot))
            return
        if src.device.type != "cuda" and dst.device.type != "cuda":
            dst.k_tensor.copy_(src.k_tensor)
            dst.v_tensor.copy_(src.v_tensor)
            return
        from .. import _capi
        dev = src.device if src.device.type == "cuda" else dst.device
        _capi.copy_pages(dst.pool.storage, src.pool.storage, [dst.slot], [src.slot], dev)

    def flush_deferred(self, device: Optional[torch.device] = None) -> int:
        """Issues the recorded GPU->CPU copies (in order, runs merged) and
        releases the device slots they read.  Returns the number of pages."""
        jobs, self._deferred = self._deferred, None
        if not jobs:
            for pool in self._pools.values():
                pool.flush_pending()
            return 0
        from .. import _capi
        groups: dict = {}
        for dst, src_pool, src_slot in jobs:
            groups.setdefault((id(dst.pool), id(src_pool)), (dst.pool, src_pool, [], []))
            g = groups[(id(dst.pool), id(src_pool))]
            g[2].append(dst.slot)
            g[3].append(src_slot)
        for dst_pool, src_pool, dsts, srcs in groups.values():
            _capi.copy_pages(dst_pool.storage, src_pool.storage, dsts, srcs, src_pool.device)
        for pool in self._pools.values():
            pool.flush_pending()
        return len(jobs)

    def report_usage(self) -> dict:
        bytes_per_page = self.bytes_per_page
        gpu_used_pages = self.gpu_total_pages - len(self.gpu_free_pool)
        cpu_used_pages = self.cpu_total_pages - len(self.cpu_free_pool)
        return {
            "gpu_pool_size": self.gpu_total_pages,
            "cpu_pool_size": self.cpu_total_pages,
            "active_gpu_pages": gpu_used_pages,
            "active_cpu_pages": cpu_used_pages,
            "gpu_free_pages": len(self.gpu_free_pool),
            "cpu_free_pages": len(self.cpu_free_pool),
            "gpu_reserved_bytes": self.gpu_total_pages * bytes_per_page,
            "cpu_reserved_bytes": self.cpu_total_pages * bytes_per_page,
            "gpu_used_bytes": gpu_used_pages * bytes_per_page,
            "cpu_used_bytes": cpu_used_pages * bytes_per_page,
        }
