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
    table; cold pages are staged into reserved HBM slots on the copy stream
    (per-layer, one layer ahead when driven by _decode_batched) and the kernel
    reads them from there;
  * placement (page ids, tiers, start/used tokens, eviction order, stats) is
    bit-identical to the reference; the data movement that the reference does
    page by page is issued in batches after the bookkeeping.

Queries on the CPU are not served here: CPU stages keep HELM's own
implementation.  K/V dtypes are bf16 and fp16; head_dim 64, 128 or 256.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch
import torch.nn.functional as F

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


class LayerKVCache:
    def __init__(self, layer_id: int):
        self.layer_id = layer_id
        self.pages: List[KVPage] = []
        self.tail_page: Optional[KVPage] = None
        self.total_tokens: int = 0

    def append_page(self, page: KVPage):
        self.pages.append(page)
        self.tail_page = page


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

    Two halves of staging slots alternate by layer parity, so the copy of
    layer l+1's cold pages (issued on the copy stream while layer l computes)
    never overwrites what layer l's attention is reading.  Before a half is
    refilled the copy stream waits for the event recorded after the last
    kernel that read it.
    """

    def __init__(self, pool):
        self.pool = pool
        self.halves: list[list[int]] = [[], []]
        self.released: list[Optional[torch.cuda.Event]] = [None, None]
        self.ready: dict = {}  # key -> (page ids, slots, event, parity)

    def _slots(self, parity: int, n: int) -> list[int]:
        half = self.halves[parity]
        while len(half) < n:
            self.pool.reserve_capacity(1)
            slot = self.pool.next_slot
            self.pool.next_slot += 1
            self.pool.staging.append(slot)
            half.append(slot)
        return half[:n]

    def issue(self, key, parity: int, pages: list, device: torch.device) -> None:
        """Starts the host->device copies of `pages` into half `parity`."""
        ids = tuple(p.page_id for p in pages)
        slots = self._slots(parity, len(pages))
        compute = torch.cuda.current_stream(device)
        use_side = _async_kv_prefetch_enabled()
        stream = _get_kv_copy_stream(device) if use_side else compute
        # pages evicted by this step's appends were queued on the compute stream
        after_evictions = torch.cuda.Event()
        after_evictions.record(compute)
        with torch.cuda.stream(stream):
            stream.wait_event(after_evictions)
            if self.released[parity] is not None:
                stream.wait_event(self.released[parity])
            by_pool: dict = {}
            for p, s in zip(pages, slots):
                by_pool.setdefault(id(p.pool), (p.pool, [], []))
                by_pool[id(p.pool)][1].append(s)
                by_pool[id(p.pool)][2].append(p.slot)
            for src_pool, dsts, srcs in by_pool.values():
                _capi.copy_pages(self.pool.storage, src_pool.storage, dsts, srcs, device,
                                 stream=stream)
            ev = torch.cuda.Event()
            ev.record(stream)
        self.ready[key] = (ids, slots, ev, parity)

    def take(self, key, parity: int, pages: list, device: torch.device) -> list[int]:
        """Slots holding `pages` for the next kernel on the compute stream."""
        ids = tuple(p.page_id for p in pages)
        entry = self.ready.pop(key, None)
        if entry is None or entry[0] != ids or entry[3] != parity:
            self.issue(key, parity, pages, device)
            entry = self.ready.pop(key)
        torch.cuda.current_stream(device).wait_event(entry[2])
        return entry[1]

    def release(self, parity: int, device: torch.device) -> None:
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(device))
        self.released[parity] = ev


_stagers: dict = {}


def _stager_for(pool) -> ColdPageStager:
    st = _stagers.get(id(pool))
    if st is None or st.pool is not pool:
        st = ColdPageStager(pool)
        _stagers[id(pool)] = st
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


def _attend_lists(query: torch.Tensor, lists: list, scale: float,
                  mask2d: Optional[torch.Tensor], softcap: Optional[float],
                  lse: Optional[torch.Tensor] = None, stage_key=None,
                  prefetch_next=None) -> torch.Tensor:
    """Decode attention: query [B, Hq, D]; lists[b] = active pages of sequence b
    (lists may be one shared list for all b).  Returns out [B, Hq, D]."""
    dev = query.device
    B = query.shape[0]
    shared = len(lists) == 1 and B > 1
    seqs = lists if not shared else lists[:1]
    all_pages = [p for pages in seqs for p in pages]
    if not all_pages:
        out = torch.zeros_like(query)
        if lse is not None:
            lse.fill_(-math.inf)
        return out
    Hkv = all_pages[0].k_tensor.shape[1]
    # Pool path: every page lives in this device's pool or in a host pool of
    # the same geometry.  Otherwise the pages are copied into a scratch pool.
    dev_pool = None
    for p in all_pages:
        if p.pool is not None and not p.pool.is_host and p.pool.device == dev:
            dev_pool = p.pool
            break
    if dev_pool is None:
        for p in all_pages:
            if p.pool is not None and p.pool.is_host:
                alloc_pool = _device_pool_like(p.pool, dev)
                if alloc_pool is not None:
                    dev_pool = alloc_pool
                break
    pool_ok = dev_pool is not None and all(
        p.pool is not None and p.pool.shape_tail == dev_pool.shape_tail
        and p.pool.dtype == query.dtype and (p.pool is dev_pool or p.pool.is_host)
        for p in all_pages)
    if not pool_ok:
        return _attend_foreign(query, seqs, shared, scale, mask2d, softcap, lse)

    P = dev_pool.shape_tail[2]
    nseq = len(seqs)
    maxp = max(len(s) for s in seqs)
    table = np.zeros((nseq, maxp), np.int32)
    used = np.zeros((nseq, maxp), np.int32)
    cold, cold_pos = [], []
    ragged = False
    for b, pages in enumerate(seqs):
        for i, p in enumerate(pages):
            used[b, i] = p.used_tokens
            if p.pool is dev_pool:
                table[b, i] = p.slot
            else:
                cold.append(p)
                cold_pos.append((b, i))
            if p.used_tokens != P and i != len(pages) - 1:
                ragged = True
    if cold:
        _record_prefetch(len(cold), sum(_page_bytes_used(p) for p in cold))
        stager = _stager_for(dev_pool)
        parity = 0 if stage_key is None else (stage_key[-1] & 1)
        slots = stager.take(stage_key, parity, cold, dev)
        for (b, i), s in zip(cold_pos, slots):
            table[b, i] = s
    out = _launch(query, dev_pool, table, used, ragged, shared, scale, mask2d, softcap, lse)
    if cold:
        stager.release(parity, dev)
    if prefetch_next is not None:
        prefetch_next(dev_pool)
    return out


def _device_pool_like(host_pool, dev):
    """The device pool of the allocator that owns `host_pool` (pages of one
    allocator share geometry), if it exists already."""
    for p in list(host_pool.pages.values())[:1]:
        alloc = getattr(p, "_allocator", None)
        if alloc is not None:
            return alloc.pool_for(dev)
    return _ALLOCATOR_POOLS.get((id(host_pool), dev.index))


_ALLOCATOR_POOLS: dict = {}


def _launch(query, pool, table, used, ragged, shared, scale, mask2d, softcap, lse):
    dev = query.device
    B = query.shape[0]
    nseq = table.shape[0]
    lens = used.sum(axis=1).astype(np.int32)
    parts = [lens, table.reshape(-1)]
    if ragged:
        start = np.zeros_like(used)
        if used.shape[1] > 1:
            start[:, 1:] = np.cumsum(used, axis=1)[:, :-1]
        nump = np.array([int((used[b] > 0).sum()) if False else used.shape[1] for b in range(nseq)],
                        np.int32)
        parts += [nump, used.reshape(-1), start.reshape(-1)]
    host = torch.from_numpy(np.concatenate(parts).astype(np.int32)).pin_memory()
    blob = host.to(dev, non_blocking=True)
    maxp = table.shape[1]
    kl = blob[:nseq]
    pt = blob[nseq:nseq + nseq * maxp].view(nseq, maxp)
    kw = {}
    if ragged:
        o = nseq + nseq * maxp
        kw = dict(num_pages=blob[o:o + nseq], page_used=blob[o + nseq:o + nseq + nseq * maxp].view(nseq, maxp),
                  page_start=blob[o + nseq + nseq * maxp:].view(nseq, maxp))
    if shared:  # every batch row attends to the same pages
        pt = pt.expand(B, maxp)
        kl = kl.expand(B)
        if ragged:
            kw = {k: (v.expand(B) if v.dim() == 1 else v.expand(B, maxp)) for k, v in kw.items()}
        pt, kl = pt.contiguous(), kl.contiguous()
        kw = {k: v.contiguous() for k, v in kw.items()}
    q3 = query if query.stride(-1) == 1 else query.contiguous()
    out, _ = _capi.paged_decode_attention(
        q3, pool.storage, pt, kl, num_kv_heads=pool.shape_tail[1], page_size=pool.shape_tail[2],
        scale=scale, softcap=softcap, mask=mask2d, lse=lse,
        max_kv_len_hint=int(lens.max()) if lens.size else 0, **kw)
    return out


def _attend_foreign(query, seqs, shared, scale, mask2d, softcap, lse):
    """Pages that are not pool slots (made by hand): copied into a scratch pool."""
    dev = query.device
    B = query.shape[0]
    Hkv, D = seqs[0][0].k_tensor.shape[1], seqs[0][0].k_tensor.shape[3]
    Pt = max(p.used_tokens for s in seqs for p in s)
    n = sum(len(s) for s in seqs)
    scratch = torch.empty(n, 2, Hkv, Pt, D, dtype=query.dtype, device=dev)
    maxp = max(len(s) for s in seqs)
    table = np.zeros((len(seqs), maxp), np.int32)
    used = np.zeros((len(seqs), maxp), np.int32)
    k = 0
    cpu_pages = []
    for b, pages in enumerate(seqs):
        for i, p in enumerate(pages):
            u = p.used_tokens
            scratch[k, 0, :, :u].copy_(p.k_tensor[0, :, :u], non_blocking=True)
            scratch[k, 1, :, :u].copy_(p.v_tensor[0, :, :u], non_blocking=True)
            if p.k_tensor.device.type != "cuda":
                cpu_pages.append(p)
            table[b, i] = k
            used[b, i] = u
            k += 1
    if cpu_pages:
        _record_prefetch(len(cpu_pages), sum(_page_bytes_used(p) for p in cpu_pages))

    class _Scratch:
        storage = scratch
        shape_tail = tuple(scratch.shape[1:])

    ragged = bool(np.any((used != Pt) & (np.arange(maxp)[None, :] <
                                        np.array([len(s) for s in seqs])[:, None] - 1)))
    return _launch(query, _Scratch, table, used, True or ragged, shared, scale, mask2d, softcap,
                   lse)


def _mask_2d(attention_mask: Optional[torch.Tensor], B: int, T: int, dev) -> Optional[torch.Tensor]:
    """[B|1, 1, 1, >=T] additive mask -> [B|1, T] view (dtype kept)."""
    if attention_mask is None:
        return None
    m = attention_mask
    if m.dim() == 4:
        m = m[:, 0, -1, :T]
    elif m.dim() == 2:
        m = m[:, :T]
    else:
        raise ValueError(f"unsupported attention_mask shape {tuple(attention_mask.shape)}")
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
    chunk over cached pages) gathers the pages and calls the library SDPA.
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
        mask2d = _mask_2d(attention_mask, B, T, query.device)
        out = _attend_lists(query[:, :, 0, :], [active], scale, mask2d, softcap)
        return out.unsqueeze(2)
    return _prefill_over_pages(query, [active], scale, attention_mask, softcap)


def _prefill_over_pages(query, lists, scale, attention_mask, softcap):
    """q_len > 1 over cached pages: dense K/V from the pages, fp32 SDPA."""
    dev = query.device
    cpu = [p for ps in lists for p in ps if p.k_tensor.device.type != "cuda"]
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
    False the device->host copies stay queued on the current stream.
    """

    def __init__(self, allocator, gpu_high_watermark_bytes: int = 512 * 1024 * 1024, *,
                 sync_evictions: bool = True):
        self.allocator = allocator
        self.layers: dict = {}
        self.gpu_high_watermark_bytes = gpu_high_watermark_bytes
        self.sync_evictions = sync_evictions
        self.cont_K: dict = {}
        self.cont_V: dict = {}
        self.cont_capacity: int = 0
        self.cont_num_layers: int = 0
        self.cont_seq_len: int = 0
        self.cont_prefill_len: int = 0
        self.use_contiguous: bool = False

    def initialize_layer_caches(self, num_layers: int):
        for i in range(num_layers):
            self.layers[i] = LayerKVCache(layer_id=i)

    def _layer(self, layer_id: int) -> LayerKVCache:
        if layer_id not in self.layers:
            self.layers[layer_id] = LayerKVCache(layer_id)
        return self.layers[layer_id]

    # -- appends: bookkeeping in the reference's order, data in one transfer --
    def _new_page(self, layer: LayerKVCache, layer_id: int, device, used: int) -> KVPage:
        page = self.allocator.allocate(device)
        page.layer_id = layer_id
        page.start_token = layer.total_tokens
        page.used_tokens = used
        layer.append_page(page)
        return page

    def append_prefill(self, layer_id: int, K_prefill: torch.Tensor, V_prefill: torch.Tensor):
        """Appends a [1, H, S, D] chunk in page-size pieces, enforcing residency
        after every page (kv_cache.py:113-143)."""
        layer = self._layer(layer_id)
        seq_len = K_prefill.size(2)
        P = self.allocator.page_size
        device = K_prefill.device
        placed = []
        self.allocator._deferred = []
        try:
            for start in range(0, seq_len, P):
                n = min(P, seq_len - start)
                page = self._new_page(layer, layer_id, device, n)
                placed.append((page, start, n))
                layer.total_tokens += n
                self._enforce_residency_policy()
            self._write_rows(placed, K_prefill, V_prefill)
        finally:
            self._finish_appends(device)

    def append_decode(self, layer_id: int, K_new: torch.Tensor, V_new: torch.Tensor,
                      skip_residency: bool = False):
        """Appends one token [1, H, 1, D] to the tail page (kv_cache.py:145-171)."""
        device = K_new.device
        self.allocator._deferred = []
        try:
            page, idx = self._reserve_decode_row(layer_id, device)
            if not skip_residency:
                self._enforce_residency_policy()
            self._write_rows([(page, 0, 1)], K_new, V_new, dst_row0=idx)
        finally:
            self._finish_appends(device)

    def _reserve_decode_row(self, layer_id: int, device):
        layer = self._layer(layer_id)
        if layer.tail_page is None or layer.tail_page.used_tokens == layer.tail_page.capacity_tokens:
            self._new_page(layer, layer_id, device, 0)
        page = layer.tail_page
        idx = page.used_tokens
        page.used_tokens += 1
        layer.total_tokens += 1
        return page, idx

    def _write_rows(self, placed, K, V, dst_row0: int = 0):
        """Writes K/V rows [1, H, S, D]: placed = [(page, src_start, n)], each
        page receiving rows dst_row0.. (prefill pages start at row 0)."""
        if not placed:
            return
        if K.device.type != "cuda":
            for page, s, n in placed:
                page.k_tensor[:, :, dst_row0:dst_row0 + n, :].copy_(K[:, :, s:s + n, :])
                page.v_tensor[:, :, dst_row0:dst_row0 + n, :].copy_(V[:, :, s:s + n, :])
            return
        P = self.allocator.page_size
        rows = []
        for page, s, n in placed:
            base = page.slot * P + dst_row0
            rows.extend(range(base, base + n))
        pool = placed[0][0].pool
        rows_t = torch.tensor(rows, dtype=torch.int64).pin_memory().to(K.device, non_blocking=True)
        kt = K[0].transpose(0, 1)  # [S, H, D]
        vt = V[0].transpose(0, 1)
        if kt.dtype != pool.dtype:
            kt, vt = kt.to(pool.dtype), vt.to(pool.dtype)
        _capi.kv_append(k=kt, v=vt, pool=pool.storage, slot_rows=rows_t, page_size=P)

    def _finish_appends(self, device):
        self.allocator.flush_deferred()
        if self.sync_evictions and self._evicted_since_sync:
            if torch.device(device).type == "cuda":
                torch.cuda.current_stream(device).synchronize()
        self._evicted_since_sync = False

    _evicted_since_sync = False

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
        gpu_pages = self._evictable()
        gpu_pages.sort(key=lambda t: t[1].start_token)
        evicted_bytes = 0
        n_moved = 0
        deferred_outside = self.allocator._deferred is None
        dev = None
        for layer, page in gpu_pages:
            if evicted_bytes >= bytes_to_evict:
                break
            original_start = page.start_token
            dev = page.device
            new_page = self.allocator.move_page(page, torch.device("cpu"))
            assert new_page.start_token == original_start, "Page invariant broken during migration"
            idx = next(i for i, p in enumerate(layer.pages) if p is page)
            layer.pages[idx] = new_page
            if layer.tail_page is page:
                layer.tail_page = new_page
            evicted_bytes += new_page.k_tensor.numel() * new_page.k_tensor.element_size() * 2
            n_moved += 1
        if n_moved:
            self._evicted_since_sync = True
            if deferred_outside and self.sync_evictions and dev is not None:
                torch.cuda.current_stream(dev).synchronize()
                self._evicted_since_sync = False
        _record_eviction(n_moved, evicted_bytes)

    def _enforce_residency_policy(self):
        bpp = self.allocator.bytes_per_page
        gpu_bytes = bpp * len(self._evictable())
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
        for layer in self.layers.values():
            for page in layer.pages:
                if page.state != "DEAD":
                    self.allocator.free(page)
            layer.pages.clear()
            layer.tail_page = None
            layer.total_tokens = 0
        self.layers.clear()

    def all_gpu_resident(self, layer_id: int) -> bool:
        if layer_id not in self.layers:
            return True
        for page in self.layers[layer_id].pages:
            if page.used_tokens > 0 and page.state != "GPU":
                return False
        return True

    # -- contiguous buffers (kv_cache.py:269-354) --------------------------------
    # The paged kernel reads pages at full bandwidth, so the decode path here
    # always uses pages; these buffers are kept for API compatibility.
    def build_contiguous(self, num_layers: int, num_kv_heads: int, head_dim: int,
                         capacity: int, device: torch.device, dtype: torch.dtype) -> bool:
        cap = capacity
        floor = max(1, min(capacity, 1024))
        while cap >= floor:
            try:
                self.cont_K.clear()
                self.cont_V.clear()
                for lid in range(num_layers):
                    self.cont_K[lid] = torch.zeros(1, num_kv_heads, cap, head_dim, device=device,
                                                   dtype=dtype)
                    self.cont_V[lid] = torch.zeros(1, num_kv_heads, cap, head_dim, device=device,
                                                   dtype=dtype)
                self.cont_capacity = cap
                self.cont_num_layers = num_layers
                self.use_contiguous = True
                return True
            except (torch.cuda.OutOfMemoryError, RuntimeError):
                self.cont_K.clear()
                self.cont_V.clear()
                if torch.device(device).type == "cuda":
                    torch.cuda.empty_cache()
                cap //= 2
        self.use_contiguous = False
        return False

    def prefill_contiguous(self, layer_id: int, K: torch.Tensor, V: torch.Tensor):
        n = K.shape[2]
        self.cont_K[layer_id][:, :, :n, :].copy_(K)
        self.cont_V[layer_id][:, :, :n, :].copy_(V)
        if layer_id == 0:
            self.cont_prefill_len = n
            self.cont_seq_len = n

    def write_decode_contiguous(self, layer_id: int, K_new: torch.Tensor, V_new: torch.Tensor):
        idx = self.cont_seq_len
        self.cont_K[layer_id][:, :, idx:idx + 1, :].copy_(K_new)
        self.cont_V[layer_id][:, :, idx:idx + 1, :].copy_(V_new)

    def get_kv_contiguous(self, layer_id: int):
        n = self.cont_seq_len + 1
        return self.cont_K[layer_id][:, :, :n, :], self.cont_V[layer_id][:, :, :n, :]

    def advance_contiguous(self):
        self.cont_seq_len += 1

    def migrate_contiguous_to_pages(self):
        if not self.cont_K:
            return
        s, e = self.cont_prefill_len, self.cont_seq_len
        if e > s:
            for lid in range(self.cont_num_layers):
                self.append_prefill(lid, self.cont_K[lid][:, :, s:e, :], self.cont_V[lid][:, :, s:e, :])
        self.drop_contiguous()

    def drop_contiguous(self):
        self.cont_K.clear()
        self.cont_V.clear()
        self.use_contiguous = False

    def reset_contiguous(self):
        if self.cont_K:
            self.use_contiguous = True
            self.cont_seq_len = 0
            self.cont_prefill_len = 0

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
