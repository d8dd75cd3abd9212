"""Host-side behaviour of the drop-in runtime (no GPU needed).

Mirrors the CPU cases of the reference's tests/unit/runtime/test_kv_allocator.py,
test_kv_cache.py and test_batch_kv_offload.py against helm_b200.runtime, and
replays the host-tier placement scenario of tests/golden/placement.json.
"""
import pytest
import torch

from helm_b200.runtime.kv_allocator import KVAllocator
from helm_b200.runtime.kv_cache import (KVCacheManager, LayerKVCache, _record_eviction,
                                        _record_prefetch, get_paging_stats,
                                        perform_streaming_attention, reset_paging_stats)

CPU = torch.device("cpu")


def _alloc(**kw):
    d = dict(num_layers=2, num_kv_heads=2, head_dim=8, page_size=4, dtype=torch.float32)
    d.update(kw)
    return KVAllocator(**d)


# ── allocator (reference test_kv_allocator.py) ──────────────────────────────────
def test_allocate_cpu_state_and_reset_metadata():
    a = _alloc()
    page = a.allocate(CPU)
    assert page.state == "CPU" and page.device.type == "cpu"
    page.layer_id, page.start_token, page.used_tokens = 99, 500, 3
    a.free(page)
    p2 = a.allocate(CPU)
    assert (p2.layer_id, p2.start_token, p2.used_tokens) == (-1, 0, 0)


def test_batch_reserve_and_lifo_reuse():
    a = _alloc()
    assert a.cpu_total_pages == 0
    p1 = a.allocate(CPU)
    assert a.cpu_total_pages == 16          # an empty CPU pool grows by 16
    a.free(p1)
    assert a.allocate(CPU) is p1            # pops the last freed page
    a.reserve_batch(3, CPU)
    a.reserve_batch(4, CPU)
    assert a.cpu_total_pages == 23


def test_page_shape_dtype_unique_ids():
    a = KVAllocator(num_layers=2, num_kv_heads=3, head_dim=16, page_size=8, dtype=torch.float16)
    p0, p1 = a.allocate(CPU), a.allocate(CPU)
    assert p0.k_tensor.shape == (1, 3, 8, 16) and p0.v_tensor.shape == (1, 3, 8, 16)
    assert p0.k_tensor.dtype == torch.float16
    assert p0.page_id != p1.page_id
    # the views alias one pool tensor
    assert p0.k_tensor.untyped_storage().data_ptr() == p1.k_tensor.untyped_storage().data_ptr()


def test_move_page_same_device_and_data():
    a = _alloc()
    page = a.allocate(CPU)
    page.used_tokens = 2
    page.k_tensor[:, :, :2, :] = 42.0
    page.v_tensor[:, :, :2, :] = 99.0
    assert a.move_page(page, CPU) is page
    assert torch.all(page.k_tensor[:, :, :2] == 42.0) and torch.all(page.v_tensor[:, :, :2] == 99.0)


def test_report_usage():
    a = _alloc()
    a.allocate(CPU)
    r = a.report_usage()
    for key in ("gpu_pool_size", "cpu_pool_size", "active_gpu_pages", "active_cpu_pages",
                "gpu_free_pages", "cpu_free_pages", "gpu_reserved_bytes", "cpu_reserved_bytes",
                "gpu_used_bytes", "cpu_used_bytes"):
        assert key in r
    assert r["active_cpu_pages"] == 1
    assert r["cpu_used_bytes"] == 2 * 2 * 4 * 8 * 4 <= r["cpu_reserved_bytes"]


def test_pool_growth_keeps_page_contents():
    a = _alloc()
    pages = [a.allocate(CPU) for _ in range(16)]
    for i, p in enumerate(pages):
        p.k_tensor.fill_(i)
    more = [a.allocate(CPU) for _ in range(40)]  # forces the host pool to grow
    assert a.cpu_total_pages >= 56 and more
    for i, p in enumerate(pages):
        assert torch.all(p.k_tensor == i)


def test_host_arenas_give_each_layer_consecutive_slots():
    """Eviction targets of interleaved layers land in per-layer runs of slots;
    page ids and free lists are untouched; slots are reused after a reset."""
    from helm_b200.runtime.kv_allocator import ARENA_SLOTS
    a = _alloc()
    pool = a.pool_for(CPU)
    layers = 3
    placed = {k: [] for k in range(layers)}
    ids = []
    for i in range(3 * ARENA_SLOTS):            # round-robin over layers, like evictions
        page = a.allocate(CPU)
        ids.append(page.page_id)
        pool.place_in_arena(page, i % layers)
        page.k_tensor.fill_(i)
        placed[i % layers].append(page)
    for pages in placed.values():
        slots = [p.slot for p in pages]
        assert slots == list(range(slots[0], slots[0] + len(slots)))
    owners = {p.slot: p for ps in placed.values() for p in ps}
    assert len(owners) == 3 * ARENA_SLOTS        # no slot given twice
    for i, page in enumerate(p for k in range(layers) for p in placed[k]):
        assert pool.pages[page.slot] is page
        assert torch.all(page.k_tensor == pool.storage[page.slot, 0])
    # reference page ids: batches of 16 created, popped last-first
    assert ids == [16 * (i // 16) + 15 - i % 16 for i in range(3 * ARENA_SLOTS)]
    top = pool.next_slot
    for pages in placed.values():
        for p in pages:
            a.free(p)
    a.forget_arenas(range(layers))
    again = []
    for i in range(2 * ARENA_SLOTS):             # allocate + place, as move_page does
        again.append(a.allocate(CPU))
        pool.place_in_arena(again[-1], 10 + i % 2)   # carved from the freed slots
    assert pool.next_slot == top
    for k in (0, 1):
        slots = [p.slot for p in again[k::2]]
        assert slots == list(range(slots[0], slots[0] + len(slots)))
    assert len({p.slot for p in again}) == len(again)
    spare = a.allocate(CPU)                       # plain allocations still get a free slot
    assert spare.slot not in {p.slot for p in again}


# ── cache manager (reference test_kv_cache.py) ─────────────────────────────────
@pytest.fixture()
def cache():
    mgr = KVCacheManager(_alloc(num_layers=4), gpu_high_watermark_bytes=0)
    mgr.initialize_layer_caches(num_layers=4)
    return mgr


def _kv(n):
    return torch.randn(1, 2, n, 8), torch.randn(1, 2, n, 8)


def test_layer_cache_tail():
    a = _alloc()
    layer = LayerKVCache(0)
    p1, p2 = a.allocate(CPU), a.allocate(CPU)
    layer.append_page(p1)
    layer.append_page(p2)
    assert layer.tail_page is p2 and len(layer.pages) == 2


def test_prefill_pages_and_data(cache):
    k, v = _kv(9)
    cache.append_prefill(0, k, v)
    L = cache.layers[0]
    assert len(L.pages) == 3 and L.total_tokens == 9
    assert [p.start_token for p in L.pages] == [0, 4, 8]
    assert torch.equal(L.pages[0].k_tensor[:, :, :4], k[:, :, :4])
    assert torch.equal(L.pages[2].v_tensor[:, :, :1], v[:, :, 8:9])


def test_decode_within_and_across_pages(cache):
    k, v = _kv(2)
    cache.append_prefill(0, k, v)
    kd, vd = _kv(1)
    cache.append_decode(0, kd, vd)
    assert len(cache.layers[0].pages) == 1 and cache.layers[0].tail_page.used_tokens == 3
    assert torch.equal(cache.layers[0].tail_page.k_tensor[:, :, 2:3], kd)
    for _ in range(4):
        cache.append_decode(0, *_kv(1))
    assert len(cache.layers[0].pages) == 2 and cache.seq_len() == 7


def test_iterate_clear_and_report(cache):
    cache.append_prefill(0, *_kv(3))
    assert isinstance(cache.iterate_layer_pages(0), list)
    assert cache.iterate_layer_pages(99) == []
    r = cache.report_bytes_per_tier()
    assert r["gpu_active_bytes"] == 0 and r["cpu_active_bytes"] > 0
    free_before = len(cache.allocator.cpu_free_pool)
    cache.clear()
    assert cache.num_layers() == 0 and cache.seq_len() == 0
    assert len(cache.allocator.cpu_free_pool) > free_before


def test_evict_without_gpu_pages_is_noop(cache):
    cache.append_prefill(0, *_kv(8))
    cache.evict_pages(99999)
    assert all(p.state == "CPU" for p in cache.layers[0].pages)


def test_contiguous_capacities():
    """reference test_kv_cache.py:501-513: small capacities are honoured; the
    window is a reservation of ceil(capacity / page_size) slots per layer."""
    alloc = _alloc()
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=0)
    pool = alloc.pool_for(CPU)
    for cap in (64, 640, 768, 2048):
        assert mgr.build_contiguous(2, 2, 8, cap, CPU, torch.float32)
        assert mgr.use_contiguous and mgr.cont_capacity == cap
        assert mgr.cont_K[0].shape == (1, 2, cap, 8)
        assert len(pool.window) == 2 * -(-cap // alloc.page_size)
    mgr.drop_contiguous()
    assert not pool.window and not mgr.use_contiguous


def test_contiguous_window_halves_when_the_pool_cannot_grow(monkeypatch):
    """build_contiguous retries with half the capacity down to
    min(capacity, 1024) tokens (kv_cache.py:272-300)."""
    alloc = _alloc()
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=0)
    pool = alloc.pool_for(CPU)
    real = pool.reserve_window

    def limited(n):           # room for 1024 tokens per layer at most
        if n > 2 * 1024 // alloc.page_size:
            raise RuntimeError("out of memory")
        return real(n)
    monkeypatch.setattr(pool, "reserve_window", limited)
    assert mgr.build_contiguous(2, 2, 8, 2048, CPU, torch.float32)
    assert mgr.cont_capacity == 1024 and mgr.use_contiguous
    # 3000 -> 1500 -> 750 < the floor of 1024: gives up
    assert not mgr.build_contiguous(2, 2, 8, 3000, CPU, torch.float32)
    assert not mgr.use_contiguous and not pool.window


def test_contiguous_window_slots_are_never_given_to_pages():
    alloc = _alloc()
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 9)
    assert mgr.build_contiguous(2, 2, 8, 40, CPU, torch.float32)
    window = set(alloc.pool_for(CPU).window)
    k = torch.randn(1, 2, 50, 8)
    mgr.append_prefill(0, k, k)
    mgr.append_prefill(1, k, k)
    slots = {p.slot for L in mgr.layers.values() for p in L.pages}
    assert not slots & window
    mgr.drop_contiguous()
    mgr.append_prefill(0, k, k)   # released slots are reused
    assert {p.slot for p in mgr.layers[0].pages} & window


# ── stats (reference test_kv_cache.py:321-362) ─────────────────────────────────
def test_paging_stats():
    reset_paging_stats()
    assert all(v == 0 for v in get_paging_stats().values())
    _record_eviction(2, 1000)
    _record_eviction(3, 1500)
    _record_prefetch(4, 4096)
    _record_eviction(0, 0)
    _record_prefetch(0, 0)
    s = get_paging_stats()
    assert (s["evict_calls"], s["pages_evicted"], s["bytes_evicted"]) == (2, 5, 2500)
    assert (s["prefetch_calls"], s["pages_prefetched"], s["bytes_prefetched"]) == (1, 4, 4096)
    reset_paging_stats()


# ── batch of items on one allocator (reference test_batch_kv_offload.py) ─────────
def test_batch_items_independent_and_reclaimed():
    a = _alloc(num_layers=4, head_dim=16, page_size=8)
    kvcms = [KVCacheManager(a, gpu_high_watermark_bytes=0) for _ in range(3)]
    kvcms[0].append_prefill(0, torch.randn(1, 2, 4, 16), torch.randn(1, 2, 4, 16))
    assert 0 in kvcms[0].layers and 0 not in kvcms[1].layers
    kvcms[1].append_prefill(0, torch.randn(1, 2, 8, 16), torch.randn(1, 2, 8, 16))
    kvcms[1].append_decode(0, torch.randn(1, 2, 1, 16), torch.randn(1, 2, 1, 16))
    assert kvcms[0].layers[0].total_tokens == 4 and kvcms[1].layers[0].total_tokens == 9
    assert a.report_usage()["active_cpu_pages"] > 0
    for k in kvcms:
        k.clear()
    assert a.report_usage()["active_cpu_pages"] == 0


def test_cpu_query_is_left_to_the_reference():
    a = _alloc()
    mgr = KVCacheManager(a)
    mgr.append_prefill(0, *_kv(4))
    with pytest.raises(NotImplementedError):
        perform_streaming_attention(torch.randn(1, 2, 1, 8), mgr.iterate_layer_pages(0))


# ── placement parity on the host tier (golden: the reference itself) ────────────
def _snapshot(mgrs, alloc):
    items = []
    for m in mgrs:
        layers = []
        for lid in sorted(m.layers):
            L = m.layers[lid]
            layers.append([lid, L.total_tokens,
                           None if L.tail_page is None else L.tail_page.page_id,
                           [[p.page_id, p.layer_id, p.start_token, p.used_tokens,
                             p.capacity_tokens, p.state, p.device.type] for p in L.pages]])
        items.append(layers)
    return {"items": items,
            "alloc": {"gpu_total": alloc.gpu_total_pages, "cpu_total": alloc.cpu_total_pages,
                      "gpu_free": [p.page_id for p in alloc.gpu_free_pool],
                      "cpu_free": [p.page_id for p in alloc.cpu_free_pool]},
            "stats": get_paging_stats()}


def replay(sc, device_kind="cpu", check_data=True):
    """Replays a placement scenario on helm_b200.runtime; returns snapshots.
    Every appended K/V row carries a unique value so that data placement can be
    verified against the page metadata after every operation."""
    dtype = {4: torch.float32, 2: torch.bfloat16}[sc["elem_bytes"]]
    alloc = KVAllocator(sc["num_layers"], sc["num_kv_heads"], sc["head_dim"],
                        page_size=sc["page_size"], dtype=dtype)
    reset_paging_stats()
    mgrs = [KVCacheManager(alloc, gpu_high_watermark_bytes=sc["watermark_per_item"])
            for _ in range(sc["batch"])]
    H, D = sc["num_kv_heads"], sc["head_dim"]
    dev = torch.device("cuda:0") if device_kind == "cuda" else CPU
    counter = [0]
    written = {}   # (item, layer, token) -> value

    def rows(item, lid, n, start):
        vals = torch.arange(counter[0], counter[0] + n, dtype=torch.float32)
        counter[0] += n
        for i in range(n):
            written[(item, lid, start + i)] = float(vals[i])
        t = vals.view(1, 1, n, 1).expand(1, H, n, D).to(dtype)
        return t.to(dev if dev.type == "cuda" else CPU)

    snaps = []
    for op in sc["ops"]:
        kind = op[0]
        if kind == "prefill":
            item, lid, n, devk = op[1], op[2], op[3], op[4]
            L = mgrs[item].layers.get(lid)
            t = rows(item, lid, n, 0 if L is None else L.total_tokens)
            t = t.to(dev) if devk == "cuda" else t.cpu()
            mgrs[item].append_prefill(lid, t, -t)
        elif kind in ("decode", "decode_skip"):
            item, lid, devk = op[1], op[2], op[3]
            L = mgrs[item].layers.get(lid)
            t = rows(item, lid, 1, 0 if L is None else L.total_tokens)
            t = t.to(dev) if devk == "cuda" else t.cpu()
            mgrs[item].append_decode(lid, t, -t, skip_residency=(kind == "decode_skip"))
        elif kind == "evict":
            mgrs[op[1]].evict_pages(op[2])
        elif kind == "clear":
            mgrs[op[1]].clear()
            for key in [k for k in written if k[0] == op[1]]:
                del written[key]
        elif kind == "snap":
            snaps.append(_snapshot(mgrs, alloc))
            if check_data:
                if dev.type == "cuda":
                    torch.cuda.synchronize()
                for item, m in enumerate(mgrs):
                    for lid, L in m.layers.items():
                        for p in L.pages:
                            if p.state == "DEAD" or p.used_tokens == 0:
                                continue
                            k = p.k_tensor[0, :, :p.used_tokens, :].float().cpu()
                            v = p.v_tensor[0, :, :p.used_tokens, :].float().cpu()
                            want = torch.tensor([written[(item, lid, p.start_token + i)]
                                                 for i in range(p.used_tokens)])
                            want = want.to(dtype).float().view(1, -1, 1)
                            assert torch.equal(k, want.expand_as(k)), (item, lid, p.page_id)
                            assert torch.equal(v, -want.expand_as(v)), (item, lid, p.page_id)
    return snaps


def test_host_tier_placement_matches_reference(placement_golden):
    for entry in placement_golden:
        sc = entry["scenario"]
        if any(len(op) > 3 and op[-1] == "cuda" for op in sc["ops"]):
            continue
        snaps = replay(sc)
        assert snaps == entry["snapshots"], sc["name"]


def test_chunk_causal_mask_detection():
    """HELM's chunk-prefill mask (pipeline_runtime.py:96-112) is recognised as
    the causal limit plus a first visible key per sequence (the native kernel
    then reads no mask): without padding the starts are 0, with left key
    padding they are the padded lengths.  A visible future key, other lengths,
    padding with a hole, or padding that leaves a row without any key are not
    recognised."""
    import numpy as np
    from helm_b200.runtime.kv_offload import _chunk_mask_starts
    S, T = 6, 20
    i = torch.arange(S).view(S, 1)
    j = torch.arange(T).view(1, T)
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        mn = torch.finfo(dtype).min
        m = torch.where(j <= T - S + i, 0.0, mn).to(dtype).view(1, 1, S, T)
        assert _chunk_mask_starts(m, m, np.array([T], np.int32), S).tolist() == [0]
        two = m.expand(2, 1, S, T)
        assert _chunk_mask_starts(two, two, np.array([T, T], np.int32), S).tolist() == [0, 0]
        # HELM adds the key padding to the causal mask (min + min = -inf there)
        pads = torch.tensor([3, 0, 14])
        keep = (j >= pads.view(3, 1, 1)).to(dtype)
        padded = (m + ((1.0 - keep) * mn).view(3, 1, 1, T)).to(dtype)
        got = _chunk_mask_starts(padded, padded, np.array([T, T, T], np.int32), S)
        assert got is not None and got.tolist() == [3, 0, 14]
        lone = padded.clone()
        lone[2, 0, :, :15] = mn      # row 0 of sequence 2 sees no key
        assert _chunk_mask_starts(lone, lone, np.array([T, T, T], np.int32), S) is None
        hole = padded.clone()
        hole[1, 0, :, 5] = mn        # a masked key after a visible one
        assert _chunk_mask_starts(hole, hole, np.array([T, T, T], np.int32), S) is None
        future = m.clone()
        future[0, 0, 0, T - 1] = 0
        assert _chunk_mask_starts(future, future, np.array([T], np.int32), S) is None
        assert _chunk_mask_starts(m, m, np.array([T - 1], np.int32), S) is None
