"""Paged KV cache and decode attention (drop-in for helm.runtime.kv_cache).

Same public names and semantics as HELM's helm/runtime/kv_cache.py:
KVPagingStats and its helpers (kv_cache.py:15-63), KVPage (:65-75),
LayerKVCache (:77-86), KVCacheManager (:88-375), the per-device copy stream
(:383-396) and perform_streaming_attention (:405-662).

What is different underneath:
  * pages are slots of a per-tier pool (see kv_allocator.py); the GPU tier is
    HBM, the CPU ("cold") tier is page-locked host memory;
  * K/V rows are written by the native fused append kernel, tier moves are
    copy-engine transfers (runs of slots merged into one cudaMemcpyAsync);
  * attention over the pages is the native split-KV kernel, fed an int32 page
    table that every layer keeps up to date incrementally; cold pages are
    staged into reserved HBM slots on the copy stream (one layer ahead when
    driven by _decode_batched) and the kernel reads them from there;
  * placement (page ids, tiers, start/used tokens, eviction order, stats) is
    identical to the reference; the data movement that the reference does page
    by page is issued in batches after the bookkeeping.

Queries on the CPU are not served here: CPU stages keep HELM's own
implementation.  K/V dtypes are bf16 and fp16; head_dim 64, 128 or 256.
"""
from __future__ import annotations

import heapq
import math
import os
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from .. import _capi


# ── paging instrumentation (kv_cache.py:15-63) ─────────────────────────────────
@dataclass
class KVPagingStats:
    evict_calls: int = 0
    pages_evicted: int = 0
    bytes_evicted: int = 0
    prefetch_calls: int = 0
    pages_prefetched: int = 0
    bytes_prefetched: int = 0


_PAGING_STATS = KVPagingStats()


def reset_paging_stats() -> None:
    """Zero the global paging counters."""
    global _PAGING_STATS
    _PAGING_STATS = KVPagingStats()


def get_paging_stats() -> dict:
    s = _PAGING_STATS
    return {
        "evict_calls": s.evict_calls,
        "pages_evicted": s.pages_evicted,
        "bytes_evicted": s.bytes_evicted,
        "prefetch_calls": s.prefetch_calls,
        "pages_prefetched": s.pages_prefetched,
        "bytes_prefetched": s.bytes_prefetched,
    }


def _record_eviction(n_pages: int, n_bytes: int) -> None:
    if n_pages <= 0:
        return
    _PAGING_STATS.evict_calls += 1
    _PAGING_STATS.pages_evicted += n_pages
    _PAGING_STATS.bytes_evicted += n_bytes


def _record_prefetch(n_pages: int, n_bytes: int) -> None:
    """One attention call that streamed n_pages (n_bytes) host->device."""
    if n_pages <= 0:
        return
    _PAGING_STATS.prefetch_calls += 1
    _PAGING_STATS.pages_prefetched += n_pages
    _PAGING_STATS.bytes_prefetched += n_bytes


# ── pages and layers ────────────────────────────────────────────────────────────
@dataclass
class KVPage:
    page_id: int
    layer_id: int
    start_token: int
    used_tokens: int
    capacity_tokens: int
    k_tensor: torch.Tensor
    v_tensor: torch.Tensor
    device: torch.device
    state: str  # 'FREE', 'GPU', 'CPU', 'DEAD'
    # pool slot and owning pool (set by KVAllocator; -1 / None for pages made by hand)
    slot: int = field(default=-1, compare=False)
    pool: Optional[object] = field(default=None, repr=False, compare=False)
    # bumped whenever the allocator hands the page out again (content changes)
    generation: int = field(default=0, repr=False, compare=False)


class LayerKVCache:
    """Ordered pages of one layer, plus the int32 page-table view of them that
    the decode kernel consumes (kept in step by KVCacheManager)."""

    def __init__(self, layer_id: int):
        self.layer_id = layer_id
        self.pages: List[KVPage] = []
        self.tail_page: Optional[KVPage] = None
        self.total_tokens: int = 0
        # slot of page i (>= 0: device pool; -1 - s: host-pool slot s), used tokens
        self._slots = np.zeros(16, np.int32)
        self._used = np.zeros(16, np.int32)
        self._n = 0
        self._ragged = False     # a page other than the last is not full
        self._cold = 0           # pages on the host tier
        self._epoch = 0          # bumped whenever the table is re-derived

    def append_page(self, page: KVPage):
        self.pages.append(page)
        self.tail_page = page

    # -- page-table bookkeeping ------------------------------------------------
    def _track_new(self, page: KVPage) -> None:
        n = self._n
        if n == len(self._slots):
            self._slots = np.concatenate([self._slots, np.zeros_like(self._slots)])
            self._used = np.concatenate([self._used, np.zeros_like(self._used)])
        if n > 0 and self._used[n - 1] != page.capacity_tokens:
            self._ragged = True
        self._slots[n] = _slot_code(page)
        self._used[n] = page.used_tokens
        if page.state == "CPU":
            self._cold += 1
        self._n = n + 1

    def _table_ok(self) -> bool:
        """True when the incremental table describes `pages` (callers may have
        edited the list directly; then the slow path rebuilds from the list)."""
        return self._n == len(self.pages) and (self._n == 0 or self.pages[-1] is self.tail_page)


def _slot_code(page: KVPage) -> int:
    if page.pool is None or page.slot < 0:
        return -(1 << 30)
    return page.slot if not page.pool.is_host else -1 - page.slot


# ── copy streams (kv_cache.py:378-396) ──────────────────────────────────────────
_kv_copy_streams: dict = {}


def _get_kv_copy_stream(device: torch.device) -> torch.cuda.Stream:
    """Per-device side stream for host<->device page copies."""
    device = torch.device(device)
    if device.type == "cuda" and device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    stream = _kv_copy_streams.get(device)
    if stream is None:
        stream = torch.cuda.Stream(device=device)
        _kv_copy_streams[device] = stream
    return stream


def _async_kv_prefetch_enabled() -> bool:
    """HELM_DISABLE_ASYNC_KV=1 stages cold pages on the compute stream instead."""
    return not bool(os.environ.get("HELM_DISABLE_ASYNC_KV"))


# ── cold-page staging ───────────────────────────────────────────────────────────
class ColdPageStager:
    """Stages host-tier pages into reserved HBM slots of a device pool.

    Two halves of staging slots alternate by layer parity, so the copies of
    layer l+1's cold pages (issued on the copy stream while layer l computes)
    never overwrite what layer l's attention reads.  Before a half is refilled
    for another layer, the copy stream waits for the event recorded after the
    last kernel that read it.  Within a half, pages already staged for the same
    layer (same page id and generation) are not copied again.
    """

    def __init__(self, pool):
        self.pool = pool
        self.halves: list[list[int]] = [[], []]
        self.maps: list[dict] = [{}, {}]          # (page_id, generation) -> slot
        self.owner: list = [None, None]           # layer key staged in the half
        self.pending: list = [None, None]         # copy-completion events
        self.released: list = [None, None]        # last-reader events

    def _slot(self, parity: int, i: int) -> int:
        half = self.halves[parity]
        while len(half) <= i:
            self.pool.reserve_capacity(1)
            slot = self.pool.next_slot
            self.pool.next_slot += 1
            self.pool.staging.append(slot)
            half.append(slot)
        return half[i]

    def issue(self, key, parity: int, pages: list, device: torch.device) -> None:
        """Starts host->device copies of the pages not yet staged in `parity`."""
        if self.owner[parity] != key:
            self.owner[parity] = key
            self.maps[parity] = {}
        m = self.maps[parity]
        todo = [p for p in pages if (p.page_id, p.generation) not in m]
        if not todo:
            return
        dst, src_by_pool = [], {}
        for p in todo:
            s = self._slot(parity, len(m))
            m[(p.page_id, p.generation)] = s
            src_by_pool.setdefault(id(p.pool), (p.pool, [], []))
            src_by_pool[id(p.pool)][1].append(s)
            src_by_pool[id(p.pool)][2].append(p.slot)
        compute = torch.cuda.current_stream(device)
        stream = _get_kv_copy_stream(device) if _async_kv_prefetch_enabled() else compute
        if stream is not compute:
            queued = torch.cuda.Event()     # evictions queued so far on the compute stream
            queued.record(compute)
            stream.wait_event(queued)
            if self.released[parity] is not None:
                stream.wait_event(self.released[parity])
        for src_pool, dsts, srcs in src_by_pool.values():
            _capi.copy_pages(self.pool.storage, src_pool.storage, dsts, srcs, device,
                             stream=stream)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.pending[parity] = ev

    def take(self, key, parity: int, pages: list, device: torch.device) -> list:
        """Slots holding `pages`, ready for the next kernel on the compute stream."""
        self.issue(key, parity, pages, device)
        if self.pending[parity] is not None:
            torch.cuda.current_stream(device).wait_event(self.pending[parity])
        m = self.maps[parity]
        return [m[(p.page_id, p.generation)] for p in pages]

    def release(self, parity: int, device: torch.device) -> None:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        self.released[parity] = ev


def _stager_for(pool) -> ColdPageStager:
    st = getattr(pool, "_stager", None)
    if st is None:
        st = pool._stager = ColdPageStager(pool)
    return st


# ── attention over page lists ──────────────────────────────────────────────────
def _check_cuda_query(query: torch.Tensor) -> None:
    if query.device.type != "cuda":
        raise NotImplementedError(
            "helm_b200 serves GPU-stage attention; CPU-stage layers keep HELM's own "
            "perform_streaming_attention")
    if query.dtype not in (torch.bfloat16, torch.float16):
        raise NotImplementedError(f"helm_b200 paged attention supports bf16/fp16, got {query.dtype}")
    if query.size(-1) not in (64, 128, 256):
        raise NotImplementedError(f"head_dim {query.size(-1)} unsupported (64, 128, 256)")


def _page_bytes_used(p: KVPage) -> int:
    return p.k_tensor[:, :, :p.used_tokens, :].numel() * p.k_tensor.element_size() * 2


class _Tables:
    """Page table of several sequences in pool-slot form, before staging."""

    def __init__(self, slots: np.ndarray, used: np.ndarray, nump: np.ndarray, ragged: bool,
                 cold: list, cold_pos: list):
        self.slots, self.used, self.nump, self.ragged = slots, used, nump, ragged
        self.cold, self.cold_pos = cold, cold_pos   # [(item, [pages])], [(item, idx array)]


def _tables_from_lists(lists: list, dev_pool) -> Optional[_Tables]:
    """Slow path: build the table from page objects.  None if some page is
    not a slot of `dev_pool` or of a host pool of the same allocator."""
    nseq = len(lists)
    maxp = max(1, max(len(s) for s in lists))
    slots = np.zeros((nseq, maxp), np.int32)
    used = np.zeros((nseq, maxp), np.int32)
    nump = np.array([len(s) for s in lists], np.int32)
    P = dev_pool.shape_tail[2]
    ragged = False
    cold, cold_pos = [], []
    for b, pages in enumerate(lists):
        cp, ci = [], []
        for i, p in enumerate(pages):
            if p.pool is None or p.pool.shape_tail != dev_pool.shape_tail or \
                    p.pool.dtype != dev_pool.dtype:
                return None
            if p.pool is dev_pool:
                slots[b, i] = p.slot
            elif p.pool.is_host and p.pool.allocator is dev_pool.allocator:
                cp.append(p)
                ci.append(i)
            else:
                return None
            used[b, i] = p.used_tokens
            if p.used_tokens != P and i != len(pages) - 1:
                ragged = True
        if cp:
            cold.append((b, cp))
            cold_pos.append((b, np.array(ci, np.int64)))
    return _Tables(slots, used, nump, ragged, cold, cold_pos)


def _run_kernel(query: torch.Tensor, pool, t: _Tables, scale, mask2d, softcap, lse,
                shared: bool = False):
    """Copies the table to the device (one pinned transfer) and launches."""
    dev = query.device
    B = query.shape[0]
    nseq, maxp = t.slots.shape
    lens = t.used.sum(axis=1).astype(np.int32)
    parts = [lens, t.slots.reshape(-1)]
    if t.ragged:
        start = np.zeros_like(t.used)
        if maxp > 1:
            start[:, 1:] = np.cumsum(t.used, axis=1)[:, :-1]
        parts += [t.nump, t.used.reshape(-1), start.reshape(-1)]
    host = torch.from_numpy(np.concatenate(parts).astype(np.int32)).pin_memory()
    blob = host.to(dev, non_blocking=True)
    kl = blob[:nseq]
    pt = blob[nseq:nseq + nseq * maxp].view(nseq, maxp)
    kw = {}
    if t.ragged:
        o = nseq + nseq * maxp
        kw = dict(num_pages=blob[o:o + nseq],
                  page_used=blob[o + nseq:o + nseq + nseq * maxp].view(nseq, maxp),
                  page_start=blob[o + nseq + nseq * maxp:].view(nseq, maxp))
    if shared and B > 1:  # every batch row attends to the same pages
        pt = pt.expand(B, maxp).contiguous()
        kl = kl.expand(B).contiguous()
        kw = {k: (v.expand(B) if v.dim() == 1 else v.expand(B, maxp)).contiguous()
              for k, v in kw.items()}
    q3 = query if query.stride(-1) == 1 else query.contiguous()
    out, _ = _capi.paged_decode_attention(
        q3, pool.storage, pt, kl, num_kv_heads=pool.shape_tail[1],
        page_size=pool.shape_tail[2], scale=scale, softcap=softcap, mask=mask2d, lse=lse,
        max_kv_len_hint=int(lens.max()) if lens.size else 0, **kw)
    return out


def _stage_and_run(query, dev_pool, t: _Tables, scale, mask2d, softcap, lse=None,
                   stage_key=None, parity: int = 0, shared: bool = False, record=True):
    """Stages cold pages (if any) and runs the kernel."""
    dev = query.device
    stager = None
    if t.cold:
        stager = _stager_for(dev_pool)
        flat = [p for _, pages in t.cold for p in pages]
        if record:
            for _, pages in t.cold:
                _record_prefetch(len(pages), sum(_page_bytes_used(p) for p in pages))
        staged = stager.take(stage_key, parity, flat, dev)
        k = 0
        for b, idx in t.cold_pos:
            t.slots[b, idx] = staged[k:k + len(idx)]
            k += len(idx)
    out = _run_kernel(query, dev_pool, t, scale, mask2d, softcap, lse, shared=shared)
    if stager is not None:
        stager.release(parity, dev)
    return out


def _attend_lists(query: torch.Tensor, lists: list, scale: float,
                  mask2d: Optional[torch.Tensor], softcap: Optional[float],
                  lse: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention: query [B, Hq, D]; lists[b] = active pages of sequence b
    (or one list shared by every b).  Returns out [B, Hq, D]."""
    B = query.shape[0]
    shared = len(lists) == 1 and B > 1
    all_pages = [p for pages in lists for p in pages]
    if not all_pages:
        if lse is not None:
            lse.fill_(-math.inf)
        return torch.zeros_like(query)
    dev_pool = None
    for p in all_pages:
        if p.pool is not None and p.pool.allocator is not None:
            dev_pool = p.pool.allocator.pool_for(query.device)
            break
    t = _tables_from_lists(lists, dev_pool) if dev_pool is not None else None
    if t is None:
        return _attend_foreign(query, lists, shared, scale, mask2d, softcap, lse)
    if dev_pool.storage is None:
        dev_pool.reserve_capacity(1)
    return _stage_and_run(query, dev_pool, t, scale, mask2d, softcap, lse,
                          stage_key=("direct", id(lists)), parity=0, shared=shared)


class _ScratchPool:
    """Page pool made for pages that are not slots of an allocator pool."""

    def __init__(self, storage):
        self.storage = storage
        self.shape_tail = tuple(storage.shape[1:])


def _attend_foreign(query, lists, shared, scale, mask2d, softcap, lse):
    """Pages made by hand (any tensors): copied into a scratch pool first."""
    dev = query.device
    p0 = lists[0][0]
    Hkv, D = p0.k_tensor.shape[1], p0.k_tensor.shape[3]
    Pt = max(p.used_tokens for s in lists for p in s)
    n = sum(len(s) for s in lists)
    scratch = torch.empty(n, 2, Hkv, Pt, D, dtype=query.dtype, device=dev)
    maxp = max(len(s) for s in lists)
    slots = np.zeros((len(lists), maxp), np.int32)
    used = np.zeros((len(lists), maxp), np.int32)
    k = 0
    cpu_pages = []
    for b, pages in enumerate(lists):
        for i, p in enumerate(pages):
            u = p.used_tokens
            scratch[k, 0, :, :u].copy_(p.k_tensor[0, :, :u], non_blocking=True)
            scratch[k, 1, :, :u].copy_(p.v_tensor[0, :, :u], non_blocking=True)
            if p.k_tensor.device.type != "cuda":
                cpu_pages.append(p)
            slots[b, i] = k
            used[b, i] = u
            k += 1
    if cpu_pages:
        _record_prefetch(len(cpu_pages), sum(_page_bytes_used(p) for p in cpu_pages))
    t = _Tables(slots, used, np.array([len(s) for s in lists], np.int32), True, [], [])
    return _run_kernel(query, _ScratchPool(scratch), t, scale, mask2d, softcap, lse, shared)


def _mask_2d(attention_mask: Optional[torch.Tensor], T: int, dev) -> Optional[torch.Tensor]:
    """[B|1, 1, q, >=T] additive mask -> [B|1, T] (last query row; dtype kept)."""
    if attention_mask is None:
        return None
    m = attention_mask
    if m.dim() == 4:
        m = m[:, 0, -1, :T]
    elif m.dim() == 2:
        m = m[:, :T]
    else:
        raise ValueError(f"unsupported attention_mask shape {tuple(attention_mask.shape)}")
    if m.shape[-1] < T:  # the kernel indexes the mask by token position
        raise ValueError(f"attention_mask covers {m.shape[-1]} keys, the cache holds {T}")
    if m.stride(-1) != 1:
        m = m.contiguous()
    if m.device != dev:
        m = m.to(dev)
    if m.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        m = m.float()
    return m


def perform_streaming_attention(query: torch.Tensor, pages: List[KVPage], scale: float = None,
                                attention_mask: Optional[torch.Tensor] = None,
                                softcap: Optional[float] = None):
    """Attention of `query` [B, Hq, q_len, D] over the used tokens of `pages`
    (helm/runtime/kv_cache.py:405-662): empty and DEAD pages are skipped,
    GQA maps query head h to KV head h // (Hq/Hkv), scores are scaled
    (default 1/sqrt(D)), optionally soft-capped and masked, accumulated in
    fp32 and returned in the query dtype.  No active page -> zeros.

    q_len == 1 runs the native split-KV decode kernel.  q_len > 1 (a prefill
    chunk over cached pages) gathers the pages and runs the fp32 math with the
    library matmul/softmax.
    """
    active = [p for p in pages if p.used_tokens > 0 and p.state != "DEAD"]
    if scale is None:
        scale = 1.0 / math.sqrt(query.size(-1))
    if not active:
        return torch.zeros_like(query)
    _check_cuda_query(query)
    B, Hq, q_len, D = query.shape
    T = sum(p.used_tokens for p in active)
    if q_len == 1:
        mask2d = _mask_2d(attention_mask, T, query.device)
        out = _attend_lists(query[:, :, 0, :], [active], scale, mask2d, softcap)
        return out.unsqueeze(2)
    return _prefill_over_pages(query, [active], scale, attention_mask, softcap)


def _prefill_over_pages(query, lists, scale, attention_mask, softcap):
    """q_len > 1 over cached pages: dense K/V from the pages, fp32 math."""
    dev = query.device
    if any(p.k_tensor.device.type != "cuda" for ps in lists for p in ps):
        for ps in lists:
            cpu = [p for p in ps if p.k_tensor.device.type != "cuda"]
            if cpu:
                _record_prefetch(len(cpu), sum(_page_bytes_used(p) for p in cpu))
    outs = []
    for b in range(query.shape[0]):
        pages = lists[b] if len(lists) > 1 else lists[0]
        K = torch.cat([p.k_tensor[:, :, :p.used_tokens, :].to(dev, non_blocking=True)
                       for p in pages], dim=2)
        V = torch.cat([p.v_tensor[:, :, :p.used_tokens, :].to(dev, non_blocking=True)
                       for p in pages], dim=2)
        q = query[b:b + 1].float()
        Kf, Vf = K.float(), V.float()
        groups = q.shape[1] // Kf.shape[1]
        if groups > 1:
            Kf = Kf.repeat_interleave(groups, dim=1)
            Vf = Vf.repeat_interleave(groups, dim=1)
        w = torch.matmul(q, Kf.transpose(-2, -1)) * scale
        if softcap is not None:
            w = torch.tanh(w / softcap) * softcap
        if attention_mask is not None:
            m = attention_mask[b:b + 1] if attention_mask.shape[0] > 1 else attention_mask
            w = w + m[..., :Kf.shape[2]].to(device=dev, dtype=torch.float32)
        w = torch.softmax(w, dim=-1)
        outs.append(torch.matmul(w, Vf).to(query.dtype))
    return torch.cat(outs, dim=0)


# ── cache manager ────────────────────────────────────────────────────────────────
class KVCacheManager:
    """Owns the per-layer page lists of one sequence (kv_cache.py:88-375).

    Extra keyword (not in the reference): sync_evictions (default True) makes
    every eviction finish before the call returns, as the reference's
    synchronous move does, so host code may read evicted pages at once.  With
    False the device->host copies stay queued on the current stream and later
    kernels and prefetches are ordered after them by the stream.
    """

    def __init__(self, allocator, gpu_high_watermark_bytes: int = 512 * 1024 * 1024, *,
                 sync_evictions: bool = True):
        self.allocator = allocator
        self.layers: dict = {}
        self.gpu_high_watermark_bytes = gpu_high_watermark_bytes
        self.sync_evictions = sync_evictions
        self._evicted = False
        # Residency bookkeeping kept in step with every append and eviction so
        # that the watermark check is O(1) and eviction O(log n), instead of
        # the reference's scan of every page of every layer per append.  Same
        # decisions: a heap of the evictable pages (GPU, full, not a tail)
        # keyed (start_token, layer order, page index) is the reference's
        # stable sort by start_token over layers in dict order.
        self._heap: list = []
        self._n_evictable = 0
        self._rank_counter = 0
        self._fingerprint: tuple = ()
        # all-GPU window (build_contiguous): layer -> reserved device-pool slots
        self._window: dict = {}
        self._window_pool = None
        self.cont_capacity: int = 0
        self.cont_num_layers: int = 0
        self.cont_seq_len: int = 0
        self.cont_prefill_len: int = 0
        self.use_contiguous: bool = False

    def initialize_layer_caches(self, num_layers: int):
        for i in range(num_layers):
            self._insert_layer(i)

    def _insert_layer(self, layer_id: int) -> LayerKVCache:
        layer = LayerKVCache(layer_id)
        layer._rank = self._rank_counter
        self._rank_counter += 1
        self.layers[layer_id] = layer
        self._fingerprint = tuple(map(id, self.layers.values()))
        return layer

    def _layer(self, layer_id: int) -> LayerKVCache:
        if layer_id not in self.layers:
            return self._insert_layer(layer_id)
        return self.layers[layer_id]

    # -- incremental residency tracking -------------------------------------------
    @staticmethod
    def _is_evictable(layer: LayerKVCache, page: KVPage) -> bool:
        return page.state == "GPU" and page.device.type == "cuda" and page is not layer.tail_page \
            and page.used_tokens == page.capacity_tokens

    def _tracking_ok(self) -> bool:
        if self._fingerprint != tuple(map(id, self.layers.values())):
            return False
        return all(hasattr(L, "_rank") and L._table_ok() for L in self.layers.values())

    def _retrack(self) -> None:
        """Rebuilds the evictable heap from a scan (after direct edits)."""
        for layer in self.layers.values():
            if not hasattr(layer, "_rank"):
                layer._rank = self._rank_counter
                self._rank_counter += 1
            if not layer._table_ok():
                _rebuild_table(layer)
        # ranks must follow the dict order of self.layers
        order = sorted(self.layers.values(), key=lambda L: L._rank)
        if [id(L) for L in order] != [id(L) for L in self.layers.values()]:
            for L in self.layers.values():
                L._rank = self._rank_counter
                self._rank_counter += 1
        self._heap = []
        for layer in self.layers.values():
            for idx, page in enumerate(layer.pages):
                if self._is_evictable(layer, page):
                    self._heap.append((page.start_token, layer._rank, idx, id(page), layer, page))
        heapq.heapify(self._heap)
        self._n_evictable = len(self._heap)
        self._fingerprint = tuple(map(id, self.layers.values()))

    def _note_new_tail(self, layer: LayerKVCache, old_tail: Optional[KVPage]) -> None:
        """A page was appended: the previous tail may have become evictable."""
        if old_tail is not None and self._is_evictable(layer, old_tail):
            idx = len(layer.pages) - 2
            heapq.heappush(self._heap, (old_tail.start_token, layer._rank, idx, id(old_tail),
                                        layer, old_tail))
            self._n_evictable += 1

    # -- appends: bookkeeping in the reference's order, data in one transfer --
    def _new_page(self, layer: LayerKVCache, layer_id: int, device, used: int) -> KVPage:
        page = self.allocator.allocate(device)
        page.layer_id = layer_id
        page.start_token = layer.total_tokens
        page.used_tokens = used
        if not layer._table_ok():
            _rebuild_table(layer)
        old_tail = layer.tail_page
        layer.append_page(page)
        layer._track_new(page)
        if hasattr(layer, "_rank"):
            self._note_new_tail(layer, old_tail)
        return page

    def _begin(self):
        if self.allocator._deferred is None:
            self.allocator._deferred = []

    def append_prefill(self, layer_id: int, K_prefill: torch.Tensor, V_prefill: torch.Tensor):
        """Appends a [1, H, S, D] chunk in page-size pieces, enforcing residency
        after every page (kv_cache.py:113-143)."""
        layer = self._layer(layer_id)
        seq_len = K_prefill.size(2)
        P = self.allocator.page_size
        device = K_prefill.device
        placed = []
        self._begin()
        try:
            for start in range(0, seq_len, P):
                n = min(P, seq_len - start)
                page = self._new_page(layer, layer_id, device, n)
                placed.append((page, page.pool, page.slot, start, n, 0))
                layer.total_tokens += n
                self._enforce_residency_policy()
            self._write_rows(placed, K_prefill, V_prefill)
        finally:
            self._finish(device)

    def append_decode(self, layer_id: int, K_new: torch.Tensor, V_new: torch.Tensor,
                      skip_residency: bool = False):
        """Appends one token [1, H, 1, D] to the tail page (kv_cache.py:145-171)."""
        device = K_new.device
        self._begin()
        try:
            place = self._reserve_decode_row(layer_id, device)
            if not skip_residency:
                self._enforce_residency_policy()
            self._write_rows([place], K_new, V_new)
        finally:
            self._finish(device)

    def _reserve_decode_row(self, layer_id: int, device):
        """Bookkeeping of one decode append; returns the row placement."""
        layer = self._layer(layer_id)
        if layer.tail_page is None or layer.tail_page.used_tokens == layer.tail_page.capacity_tokens:
            self._new_page(layer, layer_id, device, 0)
        elif not layer._table_ok():
            _rebuild_table(layer)
        page = layer.tail_page
        idx = page.used_tokens
        page.used_tokens += 1
        layer.total_tokens += 1
        layer._used[layer._n - 1] = page.used_tokens
        return (page, page.pool, page.slot, 0, 1, idx)

    def _write_rows(self, placed, K, V):
        """Writes K/V rows [1, H, S, D]; placed = [(page, pool, slot, src_start,
        n, dst_row0)] captured when the pages were placed (a page may have been
        evicted since: its data is written to the old slot, which the deferred
        device->host copy reads afterwards)."""
        if not placed:
            return
        if K.device.type != "cuda":
            for page, pool, slot, s, n, r0 in placed:
                pool.storage[slot, 0, :, r0:r0 + n, :].copy_(K[0, :, s:s + n, :])
                pool.storage[slot, 1, :, r0:r0 + n, :].copy_(V[0, :, s:s + n, :])
            return
        P = self.allocator.page_size
        pool = placed[0][1]
        rows = np.empty(sum(x[4] for x in placed), np.int64)
        k = 0
        for page, pl, slot, s, n, r0 in placed:
            if pl is not pool:
                raise RuntimeError("rows of one append must land in one pool")
            rows[k:k + n] = np.arange(slot * P + r0, slot * P + r0 + n)
            k += n
        rows_t = torch.from_numpy(rows).pin_memory().to(K.device, non_blocking=True)
        kt = K[0].transpose(0, 1)  # [S, H, D]
        vt = V[0].transpose(0, 1)
        if kt.dtype != pool.dtype:
            kt, vt = kt.to(pool.dtype), vt.to(pool.dtype)
        _capi.kv_append(k=kt, v=vt, pool=pool.storage, slot_rows=rows_t, page_size=P)

    def _finish(self, device):
        """Issues deferred evictions; waits for them when sync_evictions."""
        self.allocator.flush_deferred()
        if self.sync_evictions and self._evicted and torch.device(device).type == "cuda":
            torch.cuda.current_stream(device).synchronize()
        self._evicted = False

    def iterate_layer_pages(self, layer_id: int):
        if layer_id not in self.layers:
            return []
        return list(self.layers[layer_id].pages)

    # -- residency ----------------------------------------------------------
    def _evictable(self):
        out = []
        for layer in self.layers.values():
            tail = layer.tail_page
            for page in layer.pages:
                if page.state == "GPU" and page.device.type == "cuda" and page is not tail \
                        and page.used_tokens == page.capacity_tokens:
                    out.append((layer, page))
        return out

    def evict_pages(self, bytes_to_evict: int):
        """Global oldest-page-first eviction to the host tier (kv_cache.py:179-222)."""
        if bytes_to_evict <= 0:
            return
        if not self._tracking_ok():
            self._retrack()
        evicted_bytes = 0
        n_moved = 0
        direct = self.allocator._deferred is None
        dev = None
        while self._heap and evicted_bytes < bytes_to_evict:
            _, _, idx, _, layer, page = heapq.heappop(self._heap)
            if not (idx < len(layer.pages) and layer.pages[idx] is page
                    and self.layers.get(layer.layer_id) is layer
                    and self._is_evictable(layer, page)):
                continue  # stale entry
            self._n_evictable -= 1
            original_start = page.start_token
            dev = page.device
            new_page = self.allocator.move_page(page, torch.device("cpu"), arena_key=id(layer))
            assert new_page.start_token == original_start, "Page invariant broken during migration"
            layer.pages[idx] = new_page
            if layer.tail_page is page:
                layer.tail_page = new_page
            layer._slots[idx] = _slot_code(new_page)
            layer._cold += 1
            evicted_bytes += new_page.k_tensor.numel() * new_page.k_tensor.element_size() * 2
            n_moved += 1
        if n_moved:
            self._evicted = True
            if direct and self.sync_evictions and dev is not None:
                torch.cuda.current_stream(dev).synchronize()
                self._evicted = False
        _record_eviction(n_moved, evicted_bytes)

    def _evictable_count(self) -> int:
        if not self._tracking_ok():
            self._retrack()
        if os.environ.get("HELM_B200_CHECK_RESIDENCY"):
            assert self._n_evictable == len(self._evictable()), "residency tracking diverged"
        return self._n_evictable

    def _enforce_residency_policy(self):
        gpu_bytes = self.allocator.bytes_per_page * self._evictable_count()
        if gpu_bytes > self.gpu_high_watermark_bytes:
            self.evict_pages(gpu_bytes - self.gpu_high_watermark_bytes)

    def _enforce_residency_tracked(self):
        """The same policy for a caller that validated the tracking this step
        (_tracking_ok) and has changed pages only through this manager since."""
        if os.environ.get("HELM_B200_CHECK_RESIDENCY"):
            return self._enforce_residency_policy()
        gpu_bytes = self.allocator.bytes_per_page * self._n_evictable
        if gpu_bytes > self.gpu_high_watermark_bytes:
            self.evict_pages(gpu_bytes - self.gpu_high_watermark_bytes)

    # -- queries --------------------------------------------------------------
    def seq_len(self):
        if 0 in self.layers:
            return self.layers[0].total_tokens
        return 0

    def num_layers(self):
        return len(self.layers)

    def clear(self):
        self.allocator.forget_arenas(id(L) for L in self.layers.values())
        for layer in self.layers.values():
            for page in layer.pages:
                if page.state != "DEAD":
                    self.allocator.free(page)
            layer.pages.clear()
            layer.tail_page = None
            layer.total_tokens = 0
            _rebuild_table(layer)
        self.layers.clear()
        self._heap = []
        self._n_evictable = 0
        self._fingerprint = ()

    def all_gpu_resident(self, layer_id: int) -> bool:
        if layer_id not in self.layers:
            return True
        for page in self.layers[layer_id].pages:
            if page.used_tokens > 0 and page.state != "GPU":
                return False
        return True

    # -- all-GPU window: the reference's contiguous buffers (kv_cache.py:269-354) --
    # For all-GPU plans the reference keeps a second, dense [1, H, capacity, D]
    # copy of every layer's K/V (its page path re-concatenates pages on every
    # step).  Here the paged kernel reads pages at full bandwidth, so the
    # capacity becomes a reservation of device-pool slots per layer, the
    # "window": decode tokens of the window phase are written into it (one
    # fused-append row each) and attention reads the layer's pages plus the
    # window through one page table.  Nothing is held twice and prefill is not
    # copied again.  The observable contract is the reference's:
    # use_contiguous, cont_capacity, cont_seq_len and cont_prefill_len change
    # under the same rules, decode tokens stay out of the page lists until
    # cont_seq_len reaches the capacity, and migrate_contiguous_to_pages then
    # appends them as append_prefill does (same page ids, start/used tokens
    # and residency decisions).
    def build_contiguous(self, num_layers: int, num_kv_heads: int, head_dim: int,
                         capacity: int, device: torch.device, dtype: torch.dtype) -> bool:
        """Reserves ceil(capacity / page_size) pool slots per layer on `device`;
        when the pool cannot grow that far, retries with half the capacity
        down to min(capacity, 1024) tokens.  False if every attempt fails."""
        a = self.allocator
        if (num_kv_heads, head_dim, dtype) != (a.num_kv_heads, a.head_dim, a.dtype):
            raise ValueError("build_contiguous: geometry differs from the allocator's pages")
        P = a.page_size
        pool = a.pool_for(device)
        cap = capacity
        floor = max(1, min(capacity, 1024))
        while cap >= floor:
            self._release_window()
            per_layer = -(-cap // P)
            try:
                slots = pool.reserve_window(per_layer * num_layers)
            except (torch.cuda.OutOfMemoryError, RuntimeError):
                if pool.device.type == "cuda":
                    torch.cuda.empty_cache()
                cap //= 2
                continue
            self._window = {lid: slots[lid * per_layer:(lid + 1) * per_layer]
                            for lid in range(num_layers)}
            self._window_pool = pool
            self.cont_capacity = cap
            self.cont_num_layers = num_layers
            self.use_contiguous = True
            return True
        self.use_contiguous = False
        return False

    def _release_window(self) -> None:
        if self._window_pool is not None:
            self._window_pool.release_window([s for v in self._window.values() for s in v])
        self._window = {}
        self._window_pool = None

    def prefill_contiguous(self, layer_id: int, K: torch.Tensor, V: torch.Tensor):
        """Called after append_prefill (kv_offload.py:197-204): the pages already
        hold the chunk, so only the counters move (layer 0 sets them, as the
        reference does)."""
        if layer_id == 0:
            self.cont_prefill_len = K.shape[2]
            self.cont_seq_len = K.shape[2]

    def _window_row(self, layer_id: int) -> int:
        """Pool row of the decode token being written (window position
        cont_seq_len - cont_prefill_len)."""
        P = self.allocator.page_size
        i = self.cont_seq_len - self.cont_prefill_len
        return self._window[layer_id][i // P] * P + i % P

    def _window_pages(self, layer_id: int, n: int):
        """(slots, used) of the first n window tokens."""
        P = self.allocator.page_size
        k = -(-n // P)
        used = np.full(k, P, np.int32)
        if k:
            used[-1] = n - (k - 1) * P
        return np.asarray(self._window[layer_id][:k], np.int32), used

    def write_decode_contiguous(self, layer_id: int, K_new: torch.Tensor, V_new: torch.Tensor):
        """Writes one decode token [1, H, 1, D] at the next window position."""
        P = self.allocator.page_size
        row = self._window_row(layer_id)
        pool = self._window_pool
        if pool.is_host:
            pool.storage[row // P, 0, :, row % P].copy_(K_new[0, :, 0])
            pool.storage[row // P, 1, :, row % P].copy_(V_new[0, :, 0])
            return
        rows = torch.tensor([row], dtype=torch.int64).pin_memory().to(pool.device,
                                                                     non_blocking=True)
        _capi.kv_append(k=K_new[:, :, 0, :].to(pool.dtype), v=V_new[:, :, 0, :].to(pool.dtype),
                        pool=pool.storage, slot_rows=rows, page_size=P)

    def _window_dense(self, layer_id: int, n: int) -> tuple:
        """The first n window tokens as dense K, V [1, H, n, D] (a copy)."""
        slots, _ = self._window_pages(layer_id, n)
        st = self._window_pool.storage
        idx = torch.as_tensor(slots.astype(np.int64), device=st.device)
        H, P, D = st.shape[2], st.shape[3], st.shape[4]
        blk = st.index_select(0, idx)                       # [k, 2, H, P, D]
        kv = blk.permute(1, 2, 0, 3, 4).reshape(2, H, -1, D)[:, :, :n]
        return kv[0].unsqueeze(0), kv[1].unsqueeze(0)

    def _layer_dense(self, layer_id: int, n_window: int) -> tuple:
        """Every cached token of the layer (pages, then window) as dense
        K, V [1, H, T, D] (a copy)."""
        ks, vs = [], []
        for p in self.iterate_layer_pages(layer_id):
            if p.used_tokens > 0 and p.state != "DEAD":
                ks.append(p.k_tensor[:, :, :p.used_tokens])
                vs.append(p.v_tensor[:, :, :p.used_tokens])
        if n_window > 0:
            k, v = self._window_dense(layer_id, n_window)
            ks.append(k.to(ks[0].device) if ks else k)
            vs.append(v.to(vs[0].device) if vs else v)
        if not ks:
            a = self.allocator
            z = torch.zeros(1, a.num_kv_heads, 0, a.head_dim, dtype=a.dtype)
            return z, z.clone()
        dev = ks[-1].device
        return torch.cat([k.to(dev) for k in ks], dim=2), torch.cat([v.to(dev) for v in vs], dim=2)

    def get_kv_contiguous(self, layer_id: int):
        """K, V [1, H, T, D] of the layer through the token just written (a
        dense copy; the decode path itself reads pages and window in place)."""
        return self._layer_dense(layer_id, self.cont_seq_len - self.cont_prefill_len + 1)

    def advance_contiguous(self):
        """Commits the current decode token (after the last layer)."""
        self.cont_seq_len += 1

    def migrate_contiguous_to_pages(self):
        """Appends the window's decode tokens to every layer's pages, as the
        reference's bulk append_prefill of them does, then drops the window."""
        if not self._window:
            return
        s, e = self.cont_prefill_len, self.cont_seq_len
        if e > s:
            for lid in range(self.cont_num_layers):
                k, v = self._window_dense(lid, e - s)
                self.append_prefill(lid, k, v)
        self.drop_contiguous()

    def drop_contiguous(self):
        """Returns the window's slots to the pool; decode continues on pages."""
        self._release_window()
        self.use_contiguous = False

    def reset_contiguous(self):
        """Re-arms the window for the next generate() when it is still reserved."""
        if self._window:
            self.use_contiguous = True
            self.cont_seq_len = 0
            self.cont_prefill_len = 0

    @property
    def cont_K(self) -> dict:
        """The reference's per-layer buffers, [1, H, capacity, D]: assembled on
        access from pages and window (zeros past the cached tokens)."""
        return self._window_buffers(0)

    @property
    def cont_V(self) -> dict:
        return self._window_buffers(1)

    def _window_buffers(self, kv: int) -> dict:
        out = {}
        for lid in self._window:
            n_win = max(0, self.cont_seq_len - self.cont_prefill_len)
            dense = self._layer_dense(lid, n_win)[kv]
            a = self.allocator
            buf = torch.zeros(1, a.num_kv_heads, self.cont_capacity, a.head_dim, dtype=a.dtype,
                              device=self._window_pool.device)
            n = min(dense.shape[2], self.cont_capacity)
            buf[:, :, :n] = dense[:, :, :n].to(buf.device)
            out[lid] = buf
        return out

    def layers_keys(self):
        return sorted(self.layers.keys())

    def report_bytes_per_tier(self) -> dict:
        gpu_bytes = 0
        cpu_bytes = 0
        for layer in self.layers.values():
            for page in layer.pages:
                if page.state == "DEAD":
                    continue
                page_bytes = page.k_tensor.numel() * page.k_tensor.element_size() * 2
                if page.state == "GPU":
                    gpu_bytes += page_bytes
                elif page.state == "CPU":
                    cpu_bytes += page_bytes
        return {"gpu_active_bytes": gpu_bytes, "cpu_active_bytes": cpu_bytes}


def _rebuild_table(layer: LayerKVCache) -> None:
    """Re-derives a layer's page-table arrays from its page list."""
    layer._slots = np.zeros(max(16, 2 * len(layer.pages)), np.int32)
    layer._used = np.zeros_like(layer._slots)
    layer._n = 0
    layer._ragged = False
    layer._cold = 0
    layer._epoch = getattr(layer, "_epoch", 0) + 1
    tail, pages = layer.tail_page, list(layer.pages)
    for p in pages:
        layer._track_new(p)
    layer.tail_page = tail


def _layer_tables(kvcms: list, layer_id: int, dev_pool) -> Optional[_Tables]:
    """Page table of one layer over several sequences from the incremental
    per-layer arrays (no per-page Python work except for cold pages)."""
    layers = []
    for kvcm in kvcms:
        layer = kvcm.layers.get(layer_id)
        if layer is not None and not layer._table_ok():
            _rebuild_table(layer)
        layers.append(layer)
    maxp = max(1, max((L._n for L in layers if L is not None), default=1))
    nseq = len(kvcms)
    slots = np.zeros((nseq, maxp), np.int32)
    used = np.zeros((nseq, maxp), np.int32)
    nump = np.zeros(nseq, np.int32)
    ragged = False
    cold, cold_pos = [], []
    for b, L in enumerate(layers):
        if L is None or L._n == 0:
            continue
        n = L._n
        nump[b] = n
        slots[b, :n] = L._slots[:n]
        used[b, :n] = L._used[:n]
        if L._ragged or np.any(L._used[:n] == 0):
            ragged = True
        if L._cold:
            idx = np.nonzero(L._slots[:n] < 0)[0]
            if np.any(L._slots[idx] == -(1 << 30)):
                return None
            cold.append((b, [L.pages[i] for i in idx]))
            cold_pos.append((b, idx))
    if ragged:
        # pages with no tokens are dropped from the ragged lists
        keep = used > 0
        if not keep.all():
            for b in range(nseq):
                k = keep[b, :nump[b]]
                if k.all():
                    continue
                sel = np.nonzero(k)[0]
                remap = -np.ones(maxp, np.int64)
                remap[sel] = np.arange(sel.size)
                slots[b, :sel.size] = slots[b, sel]
                used[b, :sel.size] = used[b, sel]
                used[b, sel.size:] = 0
                nump[b] = sel.size
                for ci, (cb, idx) in enumerate(cold_pos):
                    if cb == b:
                        cold_pos[ci] = (b, remap[idx])
    return _Tables(slots, used, nump, ragged, cold, cold_pos)
