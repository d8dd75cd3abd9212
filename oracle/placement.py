"""ORACLE — test infrastructure only.

Metadata-only restatement of HELM's KV page placement policy: which page ids
exist, which tier holds them, their token ranges, the LIFO free pools and the
eviction order.  No tensors are involved.

Rules restated (reference file:line):
  * page ids count up from 0 in creation order          kv_allocator.py:20-41
  * an empty pool grows by 8 pages (GPU) / 16 (CPU), appended in creation
    order; allocate pops the LAST free page (LIFO)      kv_allocator.py:50-70
  * allocate/free reset layer_id=-1, start=0, used=0    kv_allocator.py:72-93
  * move GPU->CPU: allocate on CPU, copy metadata, the old GPU page becomes
    DEAD and leaves the GPU total (never re-pooled); any other move frees the
    old page back to its pool                           kv_allocator.py:95-144
  * append_prefill: one new page per page_size chunk, start = layer total,
    residency enforced after every page                 kv_cache.py:113-143
  * append_decode: new page only when there is no tail or the tail is full;
    residency enforced unless skipped                   kv_cache.py:145-171
  * residency: bytes of (GPU, non-tail, full) pages over all layers; evict
    only when strictly greater than the watermark       kv_cache.py:224-235
  * eviction: candidates = GPU, non-tail, full pages in layer order then page
    order, stable-sorted by start_token; move until the moved bytes reach the
    request; one stats record per call with >0 pages   kv_cache.py:179-222
  * clear: free every non-DEAD page, drop all layers   kv_cache.py:246-256
Bytes of a page = 2 * H * page_size * D * element size (full capacity).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass
class Page:
    page_id: int
    layer_id: int = -1
    start_token: int = 0
    used_tokens: int = 0
    capacity: int = 0
    device: str = "cpu"   # 'cuda' | 'cpu'
    state: str = "FREE"   # FREE | GPU | CPU | DEAD


class Stats:
    def __init__(self):
        self.evict_calls = self.pages_evicted = self.bytes_evicted = 0
        self.prefetch_calls = self.pages_prefetched = self.bytes_prefetched = 0

    def as_dict(self):
        return dict(evict_calls=self.evict_calls, pages_evicted=self.pages_evicted,
                    bytes_evicted=self.bytes_evicted, prefetch_calls=self.prefetch_calls,
                    pages_prefetched=self.pages_prefetched, bytes_prefetched=self.bytes_prefetched)


class Allocator:
    def __init__(self, num_kv_heads: int, head_dim: int, page_size: int, elem_bytes: int):
        self.page_size = page_size
        self.page_bytes = 2 * num_kv_heads * page_size * head_dim * elem_bytes
        self.free_pool = {"cuda": [], "cpu": []}
        self.total = {"cuda": 0, "cpu": 0}
        self.next_id = 0

    def _grow(self, n: int, dev: str):
        for _ in range(n):
            self.free_pool[dev].append(Page(self.next_id, capacity=self.page_size, device=dev))
            self.next_id += 1
            self.total[dev] += 1

    def allocate(self, dev: str) -> Page:
        if not self.free_pool[dev]:
            self._grow(8 if dev == "cuda" else 16, dev)
        p = self.free_pool[dev].pop()
        p.state = "GPU" if dev == "cuda" else "CPU"
        p.layer_id, p.start_token, p.used_tokens, p.device = -1, 0, 0, dev
        return p

    def free(self, p: Page):
        p.state, p.layer_id, p.start_token, p.used_tokens = "FREE", -1, 0, 0
        self.free_pool[p.device].append(p)

    def move(self, p: Page, dev: str) -> Page:
        if p.device == dev:
            return p
        q = self.allocate(dev)
        q.layer_id, q.start_token, q.used_tokens, q.device = p.layer_id, p.start_token, \
            p.used_tokens, dev
        if p.device == "cuda" and dev != "cuda":
            p.state = "DEAD"
            self.total["cuda"] -= 1
        else:
            self.free(p)
        return q


class Layer:
    def __init__(self):
        self.pages: list[Page] = []
        self.tail: Page | None = None
        self.total = 0


class CacheManager:
    def __init__(self, alloc: Allocator, watermark: int, stats: Stats):
        self.alloc = alloc
        self.watermark = watermark
        self.stats = stats
        self.layers: dict[int, Layer] = {}

    def _layer(self, lid: int) -> Layer:
        if lid not in self.layers:
            self.layers[lid] = Layer()
        return self.layers[lid]

    def prefill(self, lid: int, n: int, dev: str):
        layer = self._layer(lid)
        for start in range(0, n, self.alloc.page_size):
            chunk = min(self.alloc.page_size, n - start)
            p = self.alloc.allocate(dev)
            p.layer_id, p.start_token, p.used_tokens = lid, layer.total, chunk
            layer.pages.append(p)
            layer.tail = p
            layer.total += chunk
            self.enforce()

    def decode(self, lid: int, dev: str, skip_residency: bool = False):
        layer = self._layer(lid)
        if layer.tail is None or layer.tail.used_tokens == layer.tail.capacity:
            p = self.alloc.allocate(dev)
            p.layer_id, p.start_token, p.used_tokens = lid, layer.total, 0
            layer.pages.append(p)
            layer.tail = p
        layer.tail.used_tokens += 1
        layer.total += 1
        if not skip_residency:
            self.enforce()

    def _candidates(self):
        out = []
        for layer in self.layers.values():
            for p in layer.pages:
                if p.state == "GPU" and p.device == "cuda" and p is not layer.tail \
                        and p.used_tokens == p.capacity:
                    out.append((layer, p))
        return out

    def evict(self, nbytes: int):
        if nbytes <= 0:
            return
        cands = sorted(self._candidates(), key=lambda lp: lp[1].start_token)
        moved = moved_bytes = 0
        for layer, p in cands:
            if moved_bytes >= nbytes:
                break
            q = self.alloc.move(p, "cpu")
            layer.pages[layer.pages.index(p)] = q
            if layer.tail is p:
                layer.tail = q
            moved_bytes += self.alloc.page_bytes
            moved += 1
        if moved > 0:
            self.stats.evict_calls += 1
            self.stats.pages_evicted += moved
            self.stats.bytes_evicted += moved_bytes

    def enforce(self):
        hot = self.alloc.page_bytes * len(self._candidates())
        if hot > self.watermark:
            self.evict(hot - self.watermark)

    def clear(self):
        for layer in self.layers.values():
            for p in layer.pages:
                if p.state != "DEAD":
                    self.alloc.free(p)
        self.layers.clear()


def snapshot(mgrs, alloc: Allocator, stats: Stats) -> dict:
    """The comparable state: per item, per layer (sorted) the page records."""
    items = []
    for m in mgrs:
        layers = []
        for lid in sorted(m.layers):
            L = m.layers[lid]
            layers.append([lid, L.total, None if L.tail is None else L.tail.page_id,
                           [[p.page_id, p.layer_id, p.start_token, p.used_tokens, p.capacity,
                             p.state, p.device] for p in L.pages]])
        items.append(layers)
    return {"items": items,
            "alloc": {"gpu_total": alloc.total["cuda"], "cpu_total": alloc.total["cpu"],
                      "gpu_free": [p.page_id for p in alloc.free_pool["cuda"]],
                      "cpu_free": [p.page_id for p in alloc.free_pool["cpu"]]},
            "stats": stats.as_dict()}


def run_scenario(sc: dict) -> list:
    """Replays a scenario (see tests/golden/make_golden.py) and returns its snapshots."""
    alloc = Allocator(sc["num_kv_heads"], sc["head_dim"], sc["page_size"], sc["elem_bytes"])
    stats = Stats()
    mgrs = [CacheManager(alloc, sc["watermark_per_item"], stats) for _ in range(sc["batch"])]
    snaps = []
    for op in sc["ops"]:
        kind = op[0]
        if kind == "prefill":
            mgrs[op[1]].prefill(op[2], op[3], op[4])
        elif kind == "decode":
            mgrs[op[1]].decode(op[2], op[3])
        elif kind == "decode_skip":
            mgrs[op[1]].decode(op[2], op[3], skip_residency=True)
        elif kind == "evict":
            mgrs[op[1]].evict(op[2])
        elif kind == "clear":
            mgrs[op[1]].clear()
        elif kind == "snap":
            snaps.append(snapshot(mgrs, alloc, stats))
        else:
            raise ValueError(kind)
    return snaps
