"""Decode steps replayed as CUDA graphs.

The eager decode path (DecodeLoop + KVOffloadManager) launches ~15 kernels per
layer from Python; at batch 1 that launch cost, not HBM, bounds the step.  Here
one decode step of the whole model -- projections, fused append, paged
attention, MLP, lm_head and the argmax that feeds the next step -- is captured
once and replayed.  Everything that changes between steps lives in static
device buffers refreshed by one host->device copy before each replay:

  * the pool row of every layer's new K/V row (page bookkeeping, evictions and
    their device->host copies run on the host first, in the reference's order);
  * every layer's page table and length;
  * the key mask row and the position counter.

Cold (host-resident) pages are copied into per-layer staging slots INSIDE the
graph on the copy stream: layer l's copy waits only for the attention of layer
l-2 (the previous user of its staging half) and runs while layers l-1 and l
compute; attention(l) waits for it.  The copy nodes have fixed addresses, so
the graph is captured again whenever the set of cold pages changes (when pages
are evicted: once per page-fill period at most).  Pools are sized up front so
that no captured pointer moves.
"""
from __future__ import annotations

import math
import time
from typing import Optional

import numpy as np
import torch

from .. import _capi
from .kv_allocator import ARENA_SLOTS
from .kv_cache import _page_bytes_used, _record_prefetch, _stager_for


class _ColdPages:
    """A layer's host-resident pages as the step plan needs them; rebuilt only
    when the layer's cold set changes (an eviction or a re-derived table)."""
    __slots__ = ("key", "idx", "host_slots", "groups", "sig", "used_bytes")


def _cold_pages(layer) -> _ColdPages:
    key = (layer._cold, layer._epoch, layer._n)
    cc = getattr(layer, "_graph_cold", None)
    if cc is not None and cc.key[:2] == key[:2] and cc.key[2] <= key[2]:
        return cc   # only hot pages were appended since
    cc = _ColdPages()
    cc.key = key
    cc.idx = np.nonzero(layer._slots[:layer._n] < 0)[0]
    pages = [layer.pages[i] for i in cc.idx]
    cc.host_slots = np.array([p.slot for p in pages], np.int64)
    pools: dict = {}
    for j, p in enumerate(pages):
        pools.setdefault(id(p.pool), (p.pool, []))[1].append(j)
    cc.groups = [(pool, np.array(sel, np.intp)) for pool, sel in pools.values()]
    cc.sig = tuple((p.page_id, p.generation) for p in pages)
    cc.used_bytes = sum(_page_bytes_used(p) for p in pages)
    layer._graph_cold = cc
    return cc


def _stage_slots(stager, parity: int, a: int, b: int) -> np.ndarray:
    """Staging slots [a, b) of one half as an array (the half grows on demand)."""
    if b > a:
        stager._slot(parity, b - 1)
    half = stager.halves[parity]
    cache = stager.__dict__.setdefault("_graph_np", [None, None])
    arr = cache[parity]
    if arr is None or len(arr) != len(half):
        arr = cache[parity] = np.asarray(half, np.int64)
    return arr[a:b]


class _GraphContext:
    """Static device state read by the patched attention forwards."""

    def __init__(self, mgr, B: int, Hq: int, D: int, L: int, max_len: int, dtype, dev):
        self.mgr = mgr
        self.B, self.Hq, self.D, self.L = B, Hq, D, L
        self.max_len = max_len
        self.P = mgr.config.page_size
        self.maxp = -(-max_len // self.P)
        self.dev = dev
        self.pool = mgr.allocator.pool_for(dev)
        self.q_out = torch.empty(L, B, Hq, D, dtype=dtype, device=dev)
        self.attn_out = torch.empty(L, B, Hq, D, dtype=dtype, device=dev)
        # blob: rows int64 [L, B] | lens int32 [L, B] | tables int32 [L, B, maxp]
        n32 = L * B + L * B * self.maxp
        self.blob_bytes = L * B * 8 + n32 * 4
        self.blob = torch.zeros(self.blob_bytes, dtype=torch.uint8, device=dev)
        self.rows = self.blob[:L * B * 8].view(torch.int64).view(L, B)
        rest = self.blob[L * B * 8:].view(torch.int32)
        self.lens = rest[:L * B].view(L, B)
        self.tables = rest[L * B:].view(L, B, self.maxp)
        self.host = [torch.zeros(self.blob_bytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
        self.host_views = []
        for h in self.host:
            hv = h.numpy()
            r = hv[:L * B * 8].view(np.int64).reshape(L, B)
            rest = hv[L * B * 8:].view(np.int32)
            self.host_views.append((r, rest[:L * B].reshape(L, B),
                                    rest[L * B:].reshape(L, B, self.maxp)))
        self.host_ev = [None, None]
        self.flip = 0
        self.mask2d = torch.zeros(B, max_len, dtype=dtype, device=dev)
        self.mask4d = self.mask2d.view(B, 1, 1, max_len)
        # cold pages: per layer [(host pool, host slots, staging slots)]
        self.cold_plan: list = [[] for _ in range(L)]
        self.copy_stream = torch.cuda.Stream(dev)
        self.copy_done = [torch.cuda.Event() for _ in range(L)]
        self.attn_done = [torch.cuda.Event() for _ in range(L)]
        self.capturing = False

    # -- copies of cold pages inside the captured step --------------------------
    def _issue_copies(self, l: int) -> None:
        for host_pool, srcs, dsts in self.cold_plan[l]:
            _capi.copy_pages(self.pool.storage, host_pool.storage, dsts, srcs, self.dev,
                             stream=self.copy_stream)
        self.copy_done[l].record(self.copy_stream)

    def begin_step(self) -> None:
        cur = torch.cuda.current_stream(self.dev)
        self.copy_stream.wait_stream(cur)
        for l in (0, 1):
            if l < self.L and self.cold_plan[l]:
                with torch.cuda.stream(self.copy_stream):
                    self._issue_copies(l)

    def before_attention(self, l: int) -> None:
        if self.cold_plan[l]:
            torch.cuda.current_stream(self.dev).wait_event(self.copy_done[l])

    def after_attention(self, l: int) -> None:
        nxt = l + 2
        if nxt < self.L and self.cold_plan[nxt]:
            self.attn_done[l].record(torch.cuda.current_stream(self.dev))
            self.copy_stream.wait_event(self.attn_done[l])
            with torch.cuda.stream(self.copy_stream):
                self._issue_copies(nxt)

    def end_step(self) -> None:
        torch.cuda.current_stream(self.dev).wait_stream(self.copy_stream)


def graph_attention_forward(attn_self, kvcms, ctx: _GraphContext, hidden_states,
                            position_embeddings, q_norm=None, k_norm=None):
    """Decode forward of one attention module inside a captured step."""
    l = attn_self.layer_idx
    B = hidden_states.shape[0]
    D = attn_self.head_dim
    q = attn_self.q_proj(hidden_states).view(B, -1, D)
    k = attn_self.k_proj(hidden_states).view(B, -1, D)
    v = attn_self.v_proj(hidden_states).view(B, -1, D)
    cos, sin = position_embeddings
    _capi.kv_append(q=q, k=k, v=v, q_out=ctx.q_out[l],
                    q_norm_w=None if q_norm is None else q_norm.weight,
                    k_norm_w=None if k_norm is None else k_norm.weight,
                    eps=1e-6 if q_norm is None else q_norm.variance_epsilon,
                    cos=cos.reshape(B, D), sin=sin.reshape(B, D), pool=ctx.pool.storage,
                    slot_rows=ctx.rows[l], page_size=ctx.P)
    ctx.before_attention(l)
    _capi.paged_decode_attention(ctx.q_out[l], ctx.pool.storage, ctx.tables[l], ctx.lens[l],
                                 num_kv_heads=k.shape[1], page_size=ctx.P,
                                 scale=1.0 / math.sqrt(D), mask=None,
                                 out=ctx.attn_out[l], max_kv_len_hint=ctx.max_len)
    ctx.after_attention(l)
    return attn_self.o_proj(ctx.attn_out[l].view(B, 1, -1)), None


class GraphDecoder:
    """Greedy generation with graph-replayed decode steps (batch of equal-length
    prompts, dense page lists).  Produces the same tokens as DecodeLoop."""

    def __init__(self, model, kv_offload_mgr, max_len: int, fused: bool = False,
                 max_batch: int = 16):
        """fused: run the decode step as FusedDecodeStage (seven launches per
        layer) instead of the HF modules with the patched attention."""
        self.model = model
        self.mgr = kv_offload_mgr
        self.max_len = max_len
        cfg = model.config
        self.L = cfg.num_hidden_layers
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        self.Hq = cfg.num_attention_heads
        self.dtype = next(model.parameters()).dtype
        self.dev = next(model.parameters()).device
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.ctx: Optional[_GraphContext] = None
        self.cold_sig = None
        self.captures = 0
        self.stage = None
        if fused:
            from .decode_stage import FusedDecodeStage
            self.stage = FusedDecodeStage(model, max_batch)
        self.h2d_bytes = 0
        self._steady = None

    # -- host side of a step ------------------------------------------------------
    def _plan(self) -> None:
        """Bookkeeping of one decode token on every layer (reference order), then
        the per-layer rows, lengths and page tables, written straight into the
        pinned upload buffer of this step."""
        ctx = self.ctx
        if ctx.host_ev[ctx.flip] is not None:   # the buffer's previous upload is done
            t0 = time.perf_counter()
            ctx.host_ev[ctx.flip].synchronize()
            self.plan_wait_seconds += time.perf_counter() - t0
        if not self._plan_steady():
            self._plan_full()
        ctx.blob.copy_(ctx.host[ctx.flip], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.dev))
        ctx.host_ev[ctx.flip] = ev
        ctx.flip ^= 1

    def _plan_steady(self) -> bool:
        """The common step: every layer's tail page has room for the new row.
        Then the reference's bookkeeping reduces to advancing each tail page
        and layer by one token -- no page is allocated, the evictable set and
        so the residency check's outcome are those of the previous step, and
        page tables and cold-page copies are unchanged -- so only the rows and
        lengths of the upload buffer are rewritten (the tables too when this
        buffer was last written before the previous full plan).  False when
        the step needs the full plan."""
        st = self._steady
        if st is None:
            return False
        kvcms, P = self.mgr.kvcms, self.ctx.P
        layers = st["layers"]
        if self.mgr.allocator._deferred is not None:
            return False
        for b, kvcm in enumerate(kvcms):
            if kvcm._fingerprint is not st["fingerprints"][b]:
                return False
            for layer, n, tail in zip(layers[b], st["npages"][b], st["tails"][b]):
                if layer._n != n or layer.tail_page is not tail or \
                        tail.used_tokens >= tail.capacity_tokens:
                    return False
        rows, lens, tables = self.ctx.host_views[self.ctx.flip]
        for b in range(len(kvcms)):
            tails = st["tails"][b]
            idx = tails[0].used_tokens
            same = True
            for layer, tail in zip(layers[b], tails):
                u = tail.used_tokens
                same = same and u == idx
                tail.used_tokens = u + 1
                layer.total_tokens += 1
                layer._used[layer._n - 1] = u + 1
            if same:
                rows[:, b] = st["tail_slots"][:, b] * P + idx
                lens[:, b] = layers[b][0].total_tokens
            else:   # layers out of step (not produced by this decoder, but kept exact)
                rows[:, b] = [t.slot * P + t.used_tokens - 1 for t in tails]
                lens[:, b] = [layer.total_tokens for layer in layers[b]]
        if st["buf_epoch"][self.ctx.flip] != st["epoch"]:
            tables[...] = self.ctx.host_views[self.ctx.flip ^ 1][2]
            st["buf_epoch"][self.ctx.flip] = st["epoch"]
        for n_cold, cold_bytes in st["prefetch"]:
            _record_prefetch(n_cold, cold_bytes)
        self.h2d_bytes += st["h2d"]
        return True

    def _plan_full(self) -> None:
        from .kv_offload import _finish_rows
        ctx, kvcms, P = self.ctx, self.mgr.kvcms, self.ctx.P
        rows, lens, tables = ctx.host_views[ctx.flip]
        for kvcm in kvcms:
            kvcm._begin()
            if not kvcm._tracking_ok():
                kvcm._retrack()
        try:
            for l in range(self.L):
                for b, kvcm in enumerate(kvcms):
                    _, _, slot, _, _, r0 = kvcm._reserve_decode_row(l, self.dev)
                    rows[l, b] = slot * P + r0
                    kvcm._enforce_residency_tracked()
        finally:
            _finish_rows(kvcms, self.dev)   # eviction copies queue before the replay
        stager = _stager_for(ctx.pool)
        plans, cold_sig, prefetch, h2d = [], [], [], 0
        for l in range(self.L):
            parity, n_staged, sig, groups = l & 1, 0, [], {}
            n_cold, cold_bytes = 0, 0
            for b, kvcm in enumerate(kvcms):
                layer = kvcm.layers[l]
                if layer._ragged or not layer._table_ok():
                    raise NotImplementedError("graph decode needs dense page lists "
                                              "(prefill chunks that are a multiple of the page size)")
                n = layer._n
                if n > ctx.maxp:
                    raise ValueError("sequence longer than the graph's max_len")
                lens[l, b] = layer.total_tokens
                tables[l, b, :n] = layer._slots[:n]
                if not layer._cold:
                    continue
                cc = _cold_pages(layer)
                k = len(cc.idx)
                stage = _stage_slots(stager, parity, n_staged, n_staged + k)
                tables[l, b, cc.idx] = stage
                for pool, sel in cc.groups:
                    g = groups.setdefault(id(pool), (pool, [], []))
                    g[1].append(cc.host_slots[sel])
                    g[2].append(stage[sel])
                sig.append(cc.sig)
                n_staged += k
                n_cold += k
                cold_bytes += cc.used_bytes
            plans.append([(pool, np.concatenate(src), np.concatenate(dst))
                          for pool, src, dst in groups.values()])
            cold_sig.append(tuple(sig))
            if n_cold:   # same accounting as the eager path: one streamed call per layer
                _record_prefetch(n_cold, cold_bytes)
                prefetch.append((n_cold, cold_bytes))
                h2d += n_cold * ctx.pool.page_bytes
        self.h2d_bytes += h2d
        ctx.cold_plan = plans
        ptrs = tuple(p.storage.data_ptr() for p in self.mgr.allocator.pools()
                     if p.storage is not None)
        self._pending_sig = (tuple(cold_sig), ptrs)
        # what the steady-step plan checks against (see _plan_steady)
        epoch = (self._steady["epoch"] + 1) if self._steady is not None else 0
        buf_epoch = self._steady["buf_epoch"] if self._steady is not None else [-1, -1]
        buf_epoch[ctx.flip] = epoch
        layers = [[kvcm.layers[l] for l in range(self.L)] for kvcm in kvcms]
        tails = [[layer.tail_page for layer in ls] for ls in layers]
        self._steady = dict(
            epoch=epoch, buf_epoch=buf_epoch, layers=layers, tails=tails,
            npages=[[layer._n for layer in ls] for ls in layers],
            fingerprints=[kvcm._fingerprint for kvcm in kvcms],
            tail_slots=np.array([[t.slot for t in ts] for ts in tails], np.int64).T.copy(),
            prefetch=prefetch, h2d=h2d)

    def _step_body(self) -> None:
        ctx = self.ctx
        ctx.begin_step()
        if self.stage is not None:
            self.stage.step(self.ids, self.pos, self.logits, ctx)
        else:
            out = self.model(input_ids=self.ids, attention_mask=ctx.mask4d, position_ids=self.pos,
                             use_cache=False, logits_to_keep=1)
            self.logits.copy_(out.logits[:, -1, :])
        self.ids.copy_(torch.argmax(self.logits, dim=-1, keepdim=True))
        self.pos.add_(1)
        ctx.end_step()

    def _capture(self) -> None:
        self.graph = None
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        saved = (self.ids.clone(), self.pos.clone())
        self.mgr.kvcms[0]._graph = self.ctx
        try:
            # decode overlap: inside the step the kernel before each attention
            # is the fused append, which writes no page table or length
            with torch.cuda.graph(g, stream=side), _capi.decode_overlap():
                self._step_body()
        finally:
            self.mgr.kvcms[0]._graph = None
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        # capture does not execute: state is unchanged, but be explicit
        self.ids.copy_(saved[0])
        self.pos.copy_(saved[1])
        self.graph = g
        self.captures += 1
        self.cold_sig = self._pending_sig

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens: int, keep_logits: bool = False,
                 reserve_pages: bool = True, forced_tokens=None):
        """Greedy tokens [B, n] (and, with keep_logits, each step's logits).
        forced_tokens [B, >= n-1] (teacher forcing): step s+1 is fed
        forced_tokens[:, s] instead of the argmax, which is still returned."""
        from .decode_loop import DecodeLoop
        B, S = input_ids.shape
        if S + max_new_tokens > self.max_len:
            raise ValueError("prompt + new tokens exceed max_len")
        loop = DecodeLoop(self.model, self.mgr)
        self.mgr.reset()
        pool = self.mgr.allocator.pool_for(self.dev)
        if reserve_pages:  # pointers captured in the graph must never move
            pages = self.L * B * (-(-self.max_len // self.mgr.config.page_size))
            if pool.capacity - pool.next_slot < 2 * pages + 16:
                pool.reserve_capacity(2 * pages + 16)
            host = self.mgr.allocator.pool_for(torch.device("cpu"))
            need = pages + self.L * B * ARENA_SLOTS   # a part-used arena per layer
            if host.capacity - host.next_slot < need:
                host.reserve_capacity(need)
        logits0 = loop.prefill(input_ids)
        for kvcm in self.mgr.kvcms:   # the replayed step reads pages only: no all-GPU window
            kvcm.migrate_contiguous_to_pages()
        self._steady = None
        self.ctx = _GraphContext(self.mgr, B, self.Hq, self.D, self.L, self.max_len, self.dtype,
                                 self.dev)
        self.ids = torch.argmax(logits0, dim=-1, keepdim=True)
        self.pos = torch.full((B, 1), S, dtype=torch.long, device=self.dev)
        self.logits = torch.empty_like(logits0)
        history = torch.empty(B, max_new_tokens, dtype=torch.long, device=self.dev)
        history[:, 0] = self.ids[:, 0]
        if forced_tokens is not None:
            forced_tokens = forced_tokens.to(self.dev)
            self.ids.copy_(forced_tokens[:, 0:1])
        all_logits = [logits0.float()] if keep_logits else None
        # decode-phase timing (CUDA events around steps 1.., host planning time)
        self.decode_events = (torch.cuda.Event(enable_timing=True),
                              torch.cuda.Event(enable_timing=True))
        self.plan_seconds = 0.0        # host time of the step plans, waits included
        self.plan_wait_seconds = 0.0   # of which: waiting for an upload buffer (GPU behind)
        self.h2d_bytes = 0
        self.decode_events[0].record()
        # one eager step primes workspaces and attributes before any capture
        for step in range(1, max_new_tokens):
            t0 = time.perf_counter()
            self._plan()
            self.plan_seconds += time.perf_counter() - t0
            if self.graph is None or self._pending_sig != self.cold_sig:
                if step == 1:
                    self._eager_step()
                    history[:, step] = self.ids[:, 0]
                    if keep_logits:
                        all_logits.append(self.logits.float().clone())
                    if forced_tokens is not None and step < forced_tokens.shape[1]:
                        self.ids.copy_(forced_tokens[:, step:step + 1])
                    continue
                self._capture()
            self.graph.replay()
            history[:, step] = self.ids[:, 0]
            if keep_logits:
                all_logits.append(self.logits.float().clone())
            if forced_tokens is not None and step < forced_tokens.shape[1]:
                self.ids.copy_(forced_tokens[:, step:step + 1])
        self.decode_events[1].record()
        out = (history, all_logits) if keep_logits else history
        self.graph = None   # captured pointers belong to this request
        return out

    def decode_ms(self) -> float:
        """Device time of the last generate's decode steps 1..n-1 (synchronises)."""
        self.decode_events[1].synchronize()
        return self.decode_events[0].elapsed_time(self.decode_events[1])

    def _eager_step(self) -> None:
        """The captured body run once without capture (same bookkeeping)."""
        self.mgr.kvcms[0]._graph = self.ctx
        try:
            with _capi.decode_overlap():
                self._step_body()
        finally:
            self.mgr.kvcms[0]._graph = None
