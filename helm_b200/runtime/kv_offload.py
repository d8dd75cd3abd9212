"""KV offload integration (drop-in for helm.runtime.kv_offload).

Same names as HELM's helm/runtime/kv_offload.py: KVOffloadConfig (:33-79),
_decode_batched (:86-186), the prefill helpers (:189-227), the per-arch
attention forwards (:291-651) and KVOffloadManager (:658-831).

The patched GPU-stage forwards here run, per layer and per decode step:
  projections (library GEMMs)
  -> one fused append kernel: QK-RMSNorm (Qwen3), RoPE, K/V rows into the
     page pool for every batch item
  -> page bookkeeping and evictions exactly as the reference orders them
  -> one paged decode-attention kernel over all items (cold pages staged one
     layer ahead on the copy stream)
  -> o_proj.
"""
from __future__ import annotations

import math
import os
import weakref
from dataclasses import dataclass
from types import MethodType
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from .. import _capi
from .kv_allocator import KVAllocator
from .kv_cache import (KVCacheManager, _attend_lists, _layer_tables, _mask_2d,
                       _prefill_over_pages, _stage_and_run, _stager_for)
# re-exported: the reference module exposes it under this name (kv_offload.py:26)
from .kv_cache import perform_streaming_attention  # noqa: F401


@dataclass
class KVOffloadConfig:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    page_size: int = 64
    dtype: torch.dtype = torch.float16
    # bytes of full, non-tail GPU pages kept before evicting to host memory;
    # default: 512 tokens per layer (kv_offload.py:48-53)
    gpu_watermark_bytes: Optional[int] = None
    cont_capacity: int = 0

    def __post_init__(self):
        if self.gpu_watermark_bytes is None:
            elem = torch.tensor([], dtype=self.dtype).element_size()
            per_token_bytes = 2 * self.num_kv_heads * self.head_dim * elem
            self.gpu_watermark_bytes = 512 * per_token_bytes * self.num_layers

    @staticmethod
    def from_model(model, page_size: int = 64, gpu_watermark_bytes: Optional[int] = None,
                   cont_capacity: Optional[int] = None) -> "KVOffloadConfig":
        cfg = model.config
        num_kv_heads = getattr(cfg, "num_key_value_heads", cfg.num_attention_heads)
        head_dim = getattr(cfg, "head_dim", None) or (cfg.hidden_size // cfg.num_attention_heads)
        return KVOffloadConfig(num_layers=cfg.num_hidden_layers, num_kv_heads=num_kv_heads,
                               head_dim=head_dim, page_size=page_size,
                               dtype=next(model.parameters()).dtype,
                               gpu_watermark_bytes=gpu_watermark_bytes,
                               cont_capacity=0 if cont_capacity is None else cont_capacity)


# ── decode step ─────────────────────────────────────────────────────────────────
def _in_window(kvcms) -> bool:
    """Path 1 of kv_offload.py:115-142: while the all-GPU window has room the
    decode token goes to the window; at capacity every item's window is
    migrated to pages and the step continues on pages."""
    k0 = kvcms[0]
    if not k0.use_contiguous:
        return False
    if k0.cont_seq_len < k0.cont_capacity:
        return True
    for kvcm in kvcms:
        kvcm.migrate_contiguous_to_pages()
    return False


def _reserve_rows(kvcms, layer_idx: int, device) -> np.ndarray:
    """Reference-order bookkeeping of one decode append per item
    (append_decode + residency, kv_offload.py:146-148), with the eviction
    copies deferred until the new rows are written.  Returns pool rows (the
    window rows during the all-GPU window phase)."""
    if _in_window(kvcms):
        return np.array([kvcm._window_row(layer_idx) for kvcm in kvcms], np.int64)
    rows = np.empty(len(kvcms), np.int64)
    P = kvcms[0].allocator.page_size
    for kvcm in kvcms:
        kvcm._begin()
    for i, kvcm in enumerate(kvcms):
        page, pool, slot, _, _, r0 = kvcm._reserve_decode_row(layer_idx, device)
        rows[i] = slot * P + r0
        kvcm._enforce_residency_policy()
    return rows


def _finish_rows(kvcms, device) -> None:
    for kvcm in kvcms:
        kvcm._finish(device)


def _device_pool(kvcms, device):
    return kvcms[0].allocator.pool_for(device)


def _attend_layer(kvcms, layer_idx: int, q3: torch.Tensor, scale: float,
                  attention_mask: Optional[torch.Tensor], softcap: Optional[float] = None):
    """Decode attention of layer `layer_idx` for every item: q3 [B, Hq, D]."""
    dev = q3.device
    pool = _device_pool(kvcms, dev)
    t = _layer_tables(kvcms, layer_idx, pool)
    if kvcms[0].use_contiguous:
        if t is None:
            raise RuntimeError("all-GPU window over pages edited by hand")
        t = _with_window(kvcms, layer_idx, t, pool)
        out = _attend_tables(kvcms, layer_idx, q3, pool, t, scale, attention_mask, softcap)
        if layer_idx == kvcms[0].cont_num_layers - 1:
            for kvcm in kvcms:
                kvcm.advance_contiguous()
        return out
    if t is None:  # pages edited by hand: page-object path
        lists = [[p for p in k.iterate_layer_pages(layer_idx)
                  if p.used_tokens > 0 and p.state != "DEAD"] for k in kvcms]
        T = max(sum(p.used_tokens for p in l) for l in lists)
        return _attend_lists(q3, lists, scale, _mask_2d(attention_mask, T, dev), softcap)
    return _attend_tables(kvcms, layer_idx, q3, pool, t, scale, attention_mask, softcap)


def _attend_tables(kvcms, layer_idx, q3, pool, t, scale, attention_mask, softcap):
    dev = q3.device
    T = int(t.used.sum(axis=1).max()) if t.used.size else 0
    mask2d = _mask_2d(attention_mask, T, dev)
    key = (id(kvcms[0]), layer_idx)
    out = _stage_and_run(q3, pool, t, scale, mask2d, softcap, stage_key=key,
                         parity=layer_idx & 1)
    _prefetch_layer(kvcms, layer_idx + 1, pool, dev)
    return out


def _with_window(kvcms, layer_idx: int, t, pool):
    """Appends every item's window pages (decode tokens through the current
    one) to its page list; ragged when a list's last page before the window is
    partial (the prefill's tail)."""
    if any(k._window_pool is not pool for k in kvcms):
        raise RuntimeError("all-GPU window on another device than the query")
    n_win = kvcms[0].cont_seq_len - kvcms[0].cont_prefill_len + 1
    extra = -(-n_win // kvcms[0].allocator.page_size)
    nseq, maxp = t.slots.shape
    slots = np.zeros((nseq, maxp + extra), np.int32)
    used = np.zeros_like(slots)
    nump = t.nump.copy()
    ragged = t.ragged
    P = kvcms[0].allocator.page_size
    for b, kvcm in enumerate(kvcms):
        n = int(t.nump[b])
        slots[b, :n] = t.slots[b, :n]
        used[b, :n] = t.used[b, :n]
        if n and used[b, n - 1] != P:
            ragged = True
        s_b, u_b = kvcm._window_pages(layer_idx, n_win)
        slots[b, n:n + extra] = s_b
        used[b, n:n + extra] = u_b
        nump[b] = n + extra
    return type(t)(slots, used, nump, ragged, t.cold, t.cold_pos)


def _prefetch_layer(kvcms, layer_idx: int, pool, dev) -> None:
    """Starts copying layer `layer_idx`'s cold pages while this layer computes."""
    if not any(layer_idx in k.layers for k in kvcms):
        return
    cold = []
    for kvcm in kvcms:
        L = kvcm.layers.get(layer_idx)
        if L is None or not L._cold or not L._table_ok():
            continue
        idx = np.nonzero(L._slots[:L._n] < 0)[0]
        cold.extend(L.pages[i] for i in idx)
    if cold:
        _stager_for(pool).issue((id(kvcms[0]), layer_idx), layer_idx & 1, cold, dev)


def _check_gpu(q: torch.Tensor) -> None:
    if q.device.type != "cuda":
        raise NotImplementedError("helm_b200 serves GPU-stage attention; CPU-stage layers keep "
                                  "HELM's own kv_offload forwards")


def _decode_batched(kvcms, q, k, v, layer_idx: int, scale: float,
                    attention_mask: Optional[torch.Tensor] = None):
    """One decode step of one layer for every batch item (kv_offload.py:86-186):
    q [B, Hq, 1, D] and k, v [B, Hkv, 1, D] already normed/rotated.  Appends
    the new K/V rows, enforces residency, and attends over all cached pages.
    Returns out [B, Hq, 1, D]."""
    _check_gpu(q)
    dev = q.device
    B = q.shape[0]
    pool = _device_pool(kvcms, dev)
    try:
        rows = _reserve_rows(kvcms, layer_idx, dev)
        rows_t = torch.from_numpy(rows).pin_memory().to(dev, non_blocking=True)
        kt, vt = k[:, :, 0, :], v[:, :, 0, :]
        if kt.dtype != pool.dtype:
            kt, vt = kt.to(pool.dtype), vt.to(pool.dtype)
        _capi.kv_append(k=kt, v=vt, pool=pool.storage, slot_rows=rows_t,
                        page_size=kvcms[0].allocator.page_size)
    finally:
        _finish_rows(kvcms, dev)
    out = _attend_layer(kvcms, layer_idx, q[:, :, 0, :], scale, attention_mask)
    return out.unsqueeze(2)


def _fused_decode(attn_self, kvcms, hidden_states, position_embeddings, attention_mask,
                  q_norm=None, k_norm=None, softcap=None, scale=None):
    """Decode for a GPU-stage attention module: projections, then one fused
    append kernel (norm + RoPE + page write), then paged attention."""
    B = hidden_states.shape[0]
    D = attn_self.head_dim
    dev = hidden_states.device
    q = attn_self.q_proj(hidden_states).view(B, -1, D)   # [B, Hq, D] (S = 1)
    k = attn_self.k_proj(hidden_states).view(B, -1, D)
    v = attn_self.v_proj(hidden_states).view(B, -1, D)
    Hq = q.shape[1]
    cos, sin = position_embeddings
    cos2 = cos.reshape(B, D)
    sin2 = sin.reshape(B, D)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    pool = _device_pool(kvcms, dev)
    q_out = torch.empty(B, Hq, D, dtype=q.dtype, device=dev)
    try:
        rows = _reserve_rows(kvcms, attn_self.layer_idx, dev)
        rows_t = torch.from_numpy(rows).pin_memory().to(dev, non_blocking=True)
        _capi.kv_append(q=q, k=k, v=v, q_out=q_out,
                        q_norm_w=None if q_norm is None else q_norm.weight,
                        k_norm_w=None if k_norm is None else k_norm.weight,
                        eps=1e-6 if q_norm is None else q_norm.variance_epsilon,
                        cos=cos2, sin=sin2, pool=pool.storage, slot_rows=rows_t,
                        page_size=kvcms[0].allocator.page_size)
    finally:
        _finish_rows(kvcms, dev)
    out = _attend_layer(kvcms, attn_self.layer_idx, q_out, scale, attention_mask, softcap)
    out = out.reshape(B, 1, Hq * D)
    return attn_self.o_proj(out), None


# ── prefill helpers (kv_offload.py:189-227) ─────────────────────────────────────
def _cached_tokens(kvcm, layer_idx: int) -> int:
    return sum(page.used_tokens for page in kvcm.iterate_layer_pages(layer_idx)
               if page.used_tokens > 0 and getattr(page, "state", None) != "DEAD")


def _append_prefill_batched(kvcms, k, v, layer_idx: int) -> list:
    past_lengths = []
    for i in range(k.shape[0]):
        past_lengths.append(_cached_tokens(kvcms[i], layer_idx))
        kvcms[i].append_prefill(layer_idx, k[i:i + 1], v[i:i + 1])
        if getattr(kvcms[i], "use_contiguous", False):
            kvcms[i].prefill_contiguous(layer_idx, k[i:i + 1], v[i:i + 1])
    return past_lengths


_CAUSAL_MEMO: list = []  # [(weakref to the caller's mask tensor, key, starts)], newest last


def _chunk_mask_starts(attention_mask: torch.Tensor, mask: torch.Tensor, lens: np.ndarray,
                       S: int) -> Optional[np.ndarray]:
    """The first visible key of each sequence when mask [B|1, 1, S, T] (a
    slice of attention_mask) is HELM's chunk mask (pipeline_runtime.py:96-112)
    with or without left key padding: 0 exactly where
    starts[b] <= key j <= lens[b] - S + i, and <= -1e4 everywhere else, with
    every row seeing at least one key.  Returns starts (int32, one entry per
    mask row; all zero without padding), or None when the mask is anything
    else.  The kernel then applies the causal limit and the key start itself
    and reads no mask: the masked keys get weight exp(<= -1e4) = 0 in fp32
    either way.  Decided once per mask tensor and lengths (one device
    reduction + sync): the same mask object serves every layer of a chunk."""
    base = attention_mask._base if attention_mask._base is not None else attention_mask
    key = (tuple(mask.shape), tuple(mask.stride()), mask.storage_offset(), base._version,
           lens.tobytes(), S)
    for ref, k, starts in _CAUSAL_MEMO:
        if ref() is base and k == key:
            return starts
    B, T = mask.shape[0], mask.shape[3]
    starts = None
    if B == len(lens) or bool(np.all(lens == lens[0])):
        dev = mask.device
        past = torch.as_tensor(lens[:B].astype(np.int64) - S, device=dev).view(-1, 1, 1)
        m = mask[:, 0]
        # candidate start: the first visible key of the last row (the widest)
        zero = m[:, S - 1, :] == 0
        first = torch.where(zero.any(dim=1), zero.to(torch.int32).argmax(dim=1),
                            torch.full((B,), T, dtype=torch.int64, device=dev))
        i = torch.arange(S, device=dev).view(1, S, 1)
        j = torch.arange(T, device=dev).view(1, 1, T)
        allowed = (j >= first.view(-1, 1, 1)) & (j <= past + i)
        ok = torch.where(allowed, m == 0, m <= -1e4).all() & (first.view(-1) <= past.view(-1)).all()
        res = torch.cat([ok.view(1).to(torch.int64), first.to(torch.int64)]).cpu().numpy()
        if res[0]:
            starts = res[1:].astype(np.int32)
    _CAUSAL_MEMO.append((weakref.ref(base), key, starts))
    del _CAUSAL_MEMO[:-4]
    return starts


def _kernel_prefill(q, pool, slots, kl, lens, T: int, P: int, scale: float, attention_mask,
                    mask, softcap):
    """helm_paged_prefill_attention when the chunk's mask lets the kernel serve
    it: HELM's chunk mask, with or without left key padding (recognised, then
    applied as the causal limit and a per-sequence first key without reading
    it), no mask, or a soft-cap (the mask read); None otherwise (see
    _prefill_dense_pages for the environment switch)."""
    Hkv = pool.shape[2]
    native = (pool.dtype == q.dtype and _capi.prefill_supported(q.dtype, q.shape[-1], P)
              and (mask is None or (mask.dim() == 4 and mask.shape[1] == 1
                                    and mask.shape[2] == q.shape[2] and mask.shape[3] == T
                                    and mask.dtype in (torch.float32, torch.bfloat16,
                                                       torch.float16))))
    choice = os.environ.get("HELM_B200_NATIVE_PREFILL")
    use_kernel = False
    starts = None
    if native and (choice != "0" or softcap is not None):
        if mask is not None:
            starts = _chunk_mask_starts(attention_mask, mask, lens, q.shape[2])
        use_kernel = softcap is not None or choice == "1" or mask is None or starts is not None
    if not use_kernel:
        return None
    causal = starts is not None
    kv_starts = None
    if causal and starts.any():
        B = q.shape[0]
        kv_starts = torch.from_numpy(np.ascontiguousarray(
            np.broadcast_to(starts, (B,)) if starts.size == 1 else starts)).to(q.device)
    return _capi.paged_prefill_attention(q, pool, slots, kl, num_kv_heads=Hkv, page_size=P,
                                         scale=scale, max_kv_len=T,
                                         mask=None if causal else mask, causal=causal,
                                         softcap=softcap, kv_starts=kv_starts)


def _prefill_first_chunk(q, k, v, attention_mask, scale: float, softcap):
    """The first chunk of a prompt (no cached keys before it) on the prefill
    kernel, from the chunk's own K/V laid out as a small page pool (one copy
    of the chunk's K/V, 64-token pages): the same arithmetic whether or not
    the pages just appended stayed resident, so offload does not change the
    result.  None when the mask is one the kernel does not serve."""
    B, Hkv, S, D = k.shape
    P = 64
    if not _capi.prefill_supported(q.dtype, D, P) or k.dtype != q.dtype:
        return None
    npg = -(-S // P)
    pad = npg * P - S

    def pages(t):   # [B, Hkv, S, D] -> [B, npg, Hkv, P, D]
        if pad:
            t = F.pad(t, (0, 0, 0, pad))
        return t.view(B, Hkv, npg, P, D).permute(0, 2, 1, 3, 4)
    pool = torch.stack([pages(k), pages(v)], dim=2).reshape(B * npg, 2, Hkv, P, D)
    dev = q.device
    slots = torch.arange(B * npg, dtype=torch.int32, device=dev).view(B, npg)
    lens = np.full(B, S, np.int32)
    kl = torch.full((B,), S, dtype=torch.int32, device=dev)
    mask = None if attention_mask is None else attention_mask[..., :S].to(device=dev)
    return _kernel_prefill(q, pool, slots, kl, lens, S, P, scale, attention_mask, mask, softcap)


def _prefill_dense_pages(kvcms, q, layer_idx: int, scale: float,
                         attention_mask: Optional[torch.Tensor],
                         softcap: Optional[float] = None) -> Optional[torch.Tensor]:
    """A prefill chunk over the cached pages (the chunk's own rows included)
    when every item's pages are full, device-resident slots of the pool.

    Two device paths, both with HELM's additive mask (chunk-causal + padding,
    kv_offload.py:206-227):
      * helm_paged_prefill_attention, reading K/V in place from the pool (no
        dense copy; tcgen05 kernel): used when the mask is HELM's chunk mask
        with or without left key padding (recognised once per mask, then
        applied as the kernel's causal limit and per-sequence first key
        without reading it), when there is no mask, and for soft-capped
        scores;
      * K/V gathered to dense [B, Hkv, T, D] by one gather_kv launch, then one
        library attention (torch SDPA): used for other masks (arbitrary
        patterns, or padding that leaves a query row without any key), which
        the kernel would read element by element.
    HELM_B200_NATIVE_PREFILL=1 sends every chunk to the kernel, =0 every chunk
    without softcap to the library.  The kernel needs bf16/fp16, head dim 64
    or 128 and a page size that is a multiple of 16.  None when the page lists
    are ragged or partly on the host, or when a softcap needs the kernel and
    the shape is not one of those (the caller walks the pages)."""
    dev = q.device
    pool = _device_pool(kvcms, dev)
    t = _layer_tables(kvcms, layer_idx, pool)
    if t is None or t.ragged or t.cold:
        return None
    lens = t.used.sum(axis=1).astype(np.int32)
    T = int(lens.max()) if lens.size else 0
    if T == 0:
        return None
    P = kvcms[0].allocator.page_size
    Hkv = pool.shape_tail[1]
    slots = torch.from_numpy(np.ascontiguousarray(t.slots)).pin_memory().to(dev, non_blocking=True)
    kl = torch.from_numpy(lens).pin_memory().to(dev, non_blocking=True)
    mask = None if attention_mask is None else attention_mask[..., :T].to(device=dev)
    out = _kernel_prefill(q, pool.storage, slots, kl, lens, T, P, scale, attention_mask, mask,
                          softcap)
    if out is not None or softcap is not None:
        return out
    k, v = _capi.gather_kv(pool.storage, slots, kl, T, num_kv_heads=Hkv, page_size=P)
    if k.dtype != q.dtype:
        k, v = k.to(q.dtype), v.to(q.dtype)
    if mask is not None:
        mask = mask.to(dtype=q.dtype)
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=scale,
                                          enable_gqa=q.shape[1] != k.shape[1])


def _stream_prefill_batched(kvcms, q, layer_idx: int, scale: float,
                            attention_mask: Optional[torch.Tensor] = None,
                            softcap: Optional[float] = None):
    """Prefill chunk attending over all cached pages (kv_offload.py:203-227)."""
    if q.device.type == "cuda":
        out = _prefill_dense_pages(kvcms, q, layer_idx, scale, attention_mask, softcap)
        if out is not None:
            return out
    lists = [[p for p in kvcms[i].iterate_layer_pages(layer_idx)
              if p.used_tokens > 0 and p.state != "DEAD"] for i in range(q.shape[0])]
    return _prefill_over_pages(q, lists, scale, attention_mask, softcap)


def _prefill(attn_self, kvcms, q, k, v, attention_mask, scale, softcap=None):
    """q [B, Hq, S, D], k/v [B, Hkv, S, D] (normed + rotated)."""
    past_lengths = _append_prefill_batched(kvcms, k, v, attn_self.layer_idx)
    if any(past > 0 for past in past_lengths):
        return _stream_prefill_batched(kvcms, q, attn_self.layer_idx, scale, attention_mask,
                                       softcap)
    # first chunk: the chunk-prefill kernel (HELM's chunk-causal mask, no mask,
    # or a soft-cap); the reference's dense attention over k, v for other
    # masks (kv_offload.py:387-395)
    if q.device.type == "cuda":
        out = _prefill_first_chunk(q, k, v, attention_mask, scale, softcap)
        if out is not None:
            return out
    groups = q.shape[1] // k.shape[1]
    if softcap is None:
        return F.scaled_dot_product_attention(q, k, v, attn_mask=attention_mask, scale=scale,
                                              enable_gqa=groups > 1)
    kx = k.repeat_interleave(groups, dim=1)
    vx = v.repeat_interleave(groups, dim=1)
    w = torch.matmul(q, kx.transpose(2, 3)) * scale
    w = torch.tanh(w / softcap) * softcap
    if attention_mask is not None:
        w = w + attention_mask[:, :, :, :kx.shape[-2]].to(w.dtype)
    w = F.softmax(w, dim=-1, dtype=torch.float32).to(q.dtype)
    return torch.matmul(w, vx)


def _prefill_qkv(attn_self, hidden_states, position_embeddings, q_norm=None, k_norm=None,
                 norm_whole=False):
    """Projections + norms + RoPE for a prefill chunk, via the fused kernel
    (norm per head) or the module's own norm over the whole projection."""
    B, S, _ = hidden_states.shape
    D = attn_self.head_dim
    q = attn_self.q_proj(hidden_states)
    k = attn_self.k_proj(hidden_states)
    v = attn_self.v_proj(hidden_states).view(B, S, -1, D)
    if norm_whole:  # OLMo-2 normalises the full projection (kv_offload.py:429-430)
        q, k = q_norm(q), k_norm(k)
        q_norm = k_norm = None
    q = q.view(B * S, -1, D)
    k = k.view(B * S, -1, D)
    Hq, Hkv = q.shape[1], k.shape[1]
    cos, sin = position_embeddings
    q_out = torch.empty(B * S, Hq, D, dtype=q.dtype, device=q.device)
    k_out = torch.empty(B * S, Hkv, D, dtype=q.dtype, device=q.device)
    v_out = torch.empty_like(k_out)
    _capi.kv_append(q=q, k=k, v=v.reshape(B * S, Hkv, D), q_out=q_out,
                    q_norm_w=None if q_norm is None else q_norm.weight,
                    k_norm_w=None if k_norm is None else k_norm.weight,
                    eps=1e-6 if q_norm is None else q_norm.variance_epsilon,
                    cos=cos.reshape(B * S, D), sin=sin.reshape(B * S, D),
                    pool=None, slot_rows=None, page_size=1, k_out=k_out, v_out=v_out)
    shape = lambda t, H: t.view(B, S, H, D).transpose(1, 2)  # noqa: E731
    return shape(q_out, Hq), shape(k_out, Hkv), shape(v_out, Hkv)


# ── per-architecture forwards (kv_offload.py:291-651) ───────────────────────────
def _make_forward(kvcms, *, qk_norm: bool = False, norm_whole: bool = False,
                  gemma2: bool = False):
    def forward(attn_self, hidden_states, position_embeddings, attention_mask=None,
                past_key_values=None, cache_position=None, **kwargs):
        _check_gpu(hidden_states)
        B, q_len, _ = hidden_states.shape
        qn = getattr(attn_self, "q_norm", None) if qk_norm else None
        kn = getattr(attn_self, "k_norm", None) if qk_norm else None
        scale = getattr(attn_self, "scaling", 1.0 / math.sqrt(attn_self.head_dim)) if gemma2 \
            else 1.0 / math.sqrt(attn_self.head_dim)
        softcap = getattr(attn_self, "attn_logit_softcapping", None) if gemma2 else None
        ctx = getattr(kvcms[0], "_graph", None)
        if ctx is not None and q_len == 1 and not norm_whole and not gemma2:
            from .graph_decode import graph_attention_forward
            return graph_attention_forward(attn_self, kvcms, ctx, hidden_states,
                                           position_embeddings, qn, kn)
        if q_len == 1 and not norm_whole:
            mask = attention_mask
            if gemma2:
                mask = _gemma2_decode_mask(attn_self, kvcms, attention_mask, cache_position,
                                           hidden_states.dtype)
            return _fused_decode(attn_self, kvcms, hidden_states, position_embeddings, mask,
                                 q_norm=qn, k_norm=kn, softcap=softcap, scale=scale)
        q, k, v = _prefill_qkv(attn_self, hidden_states, position_embeddings, qn, kn,
                               norm_whole=norm_whole)
        if q_len == 1:  # OLMo-2 decode: whole-projection norm done, pages via _decode_batched
            out = _decode_batched(kvcms, q, k, v, attn_self.layer_idx, scale, attention_mask)
        else:
            mask = attention_mask
            if gemma2:
                key_len = max(_cached_tokens(c, attn_self.layer_idx) for c in kvcms) + q_len
                mask = _gemma2_window(attn_self, attention_mask, cache_position, key_len,
                                      q.device, q.dtype)
            out = _prefill(attn_self, kvcms, q, k, v, mask, scale, softcap)
        out = out.transpose(1, 2).contiguous().reshape(B, q_len, -1)
        return attn_self.o_proj(out), None

    return forward


def _make_qwen3_forward(kvcms):
    """Qwen3: per-head q_norm/k_norm, RoPE, paged cache (kv_offload.py:349-403)."""
    return _make_forward(kvcms, qk_norm=True)


def _make_qwen2_forward(kvcms):
    return _make_forward(kvcms)


def _make_llama_forward(kvcms):
    """Llama / Mistral / Ministral (kv_offload.py:467-519)."""
    return _make_forward(kvcms)


def _make_olmo2_forward(kvcms):
    """OLMo-2: q_norm/k_norm over the whole projection (kv_offload.py:406-464)."""
    return _make_forward(kvcms, qk_norm=True, norm_whole=True)


def _make_gemma2_forward(kvcms):
    """Gemma-2: soft-capped scores and a per-layer sliding window (kv_offload.py:551-651)."""
    return _make_forward(kvcms, gemma2=True)


def _gemma2_window(attn_self, attention_mask, cache_position, key_length, device, dtype):
    """Caller mask with Gemma-2's sliding window overlaid (kv_offload.py:240-288)."""
    if attention_mask is not None:
        query_length = attention_mask.shape[-2]
        attention_mask = attention_mask[:, :, :query_length, :key_length]
    elif cache_position is not None:
        query_length = int(cache_position.numel())
    else:
        query_length = key_length
    window = getattr(attn_self, "sliding_window", None)
    if window is None:
        return attention_mask
    if cache_position is None:
        qpos = torch.arange(query_length, device=device, dtype=torch.long)
    else:
        qpos = cache_position.to(device=device, dtype=torch.long).reshape(-1)
        if qpos.numel() != query_length:
            raise ValueError("Gemma2 sliding-window mask requires cache_position to match "
                             f"query length ({query_length}), got {qpos.numel()}.")
    kpos = torch.arange(key_length, device=device, dtype=torch.long)
    allowed = (kpos[None, :] <= qpos[:, None]) & (kpos[None, :] > qpos[:, None] - window)
    sliding = torch.full((query_length, key_length), torch.finfo(dtype).min, device=device,
                         dtype=dtype)
    sliding.masked_fill_(allowed, 0)
    sliding = sliding[None, None]
    return sliding if attention_mask is None else attention_mask + sliding


def _gemma2_decode_mask(attn_self, kvcms, attention_mask, cache_position, dtype):
    key_len = max(_cached_tokens(c, attn_self.layer_idx) for c in kvcms) + 1
    dev = kvcms[0].allocator.pool_for(torch.device("cuda", torch.cuda.current_device())).device \
        if attention_mask is None else attention_mask.device
    return _gemma2_window(attn_self, attention_mask, cache_position, key_len, dev, dtype)


# ── manager (kv_offload.py:658-831) ─────────────────────────────────────────────
class KVOffloadManager:
    """Installs paged-KV attention forwards on a model's GPU attention modules
    and manages the cache lifecycle across generate() calls.  One
    KVCacheManager per batch item, all on one KVAllocator; the GPU watermark is
    split across items (kv_offload.py:683-689).

    Only modules whose parameters live on a CUDA device are patched; CPU-stage
    layers keep the model's own forward.  config.cont_capacity > 0 on a CUDA
    model reserves the all-GPU decode window of every item
    (KVCacheManager.build_contiguous; kv_offload.py:697-713): all or none.
    """

    _ARCHS = ("qwen3", "qwen2", "gemma2", "ministral", "olmo2", "mistral", "llama")

    def __init__(self, model, config: KVOffloadConfig, batch_size: int = 1, *,
                 sync_evictions: bool = False):
        self.config = config
        self.batch_size = batch_size
        self.allocator = KVAllocator(num_layers=config.num_layers,
                                     num_kv_heads=config.num_kv_heads,
                                     head_dim=config.head_dim, page_size=config.page_size,
                                     dtype=config.dtype)
        watermark_per_item = max(config.gpu_watermark_bytes // batch_size, 1)
        self.kvcms = [KVCacheManager(self.allocator, gpu_high_watermark_bytes=watermark_per_item,
                                     sync_evictions=sync_evictions)
                      for _ in range(batch_size)]
        self._patched: dict = {}
        self._patched_instance_forwards: dict = {}
        self._apply_patches(model)
        self.patch_module_roots(model)
        if config.cont_capacity > 0:
            device = next(model.parameters()).device
            if device.type == "cuda":
                built = [kvcm.build_contiguous(num_layers=config.num_layers,
                                               num_kv_heads=config.num_kv_heads,
                                               head_dim=config.head_dim,
                                               capacity=config.cont_capacity, device=device,
                                               dtype=config.dtype)
                         for kvcm in self.kvcms]
                if not all(built):
                    for kvcm in self.kvcms:
                        kvcm.drop_contiguous()

    def reset(self):
        """Clears every paged cache (kv_offload.py:717-721)."""
        for kvcm in self.kvcms:
            kvcm.clear()
            kvcm.reset_contiguous()

    def restore(self):
        """Restores the original attention forwards (kv_offload.py:723-731)."""
        for module, had_instance_forward, original_forward in \
                self._patched_instance_forwards.values():
            if had_instance_forward:
                module.forward = original_forward
            else:
                module.__dict__.pop("forward", None)
        self._patched_instance_forwards.clear()
        self._patched.clear()

    def report(self) -> dict:
        return self.allocator.report_usage()

    def patch_module_roots(self, *roots):
        """Binds the paged forward to every matching attention instance under
        `roots` whose parameters are on a CUDA device (kv_offload.py:736-762)."""
        for root in roots:
            if root is None:
                continue
            for cls, patched_forward in self._patched.values():
                for module in root.modules():
                    if not isinstance(module, cls):
                        continue
                    key = id(module)
                    if key in self._patched_instance_forwards:
                        continue
                    param = next(module.parameters(), None)
                    if param is None or param.device.type != "cuda":
                        continue
                    had = "forward" in module.__dict__
                    original = module.__dict__.get("forward")
                    module.forward = MethodType(patched_forward, module)
                    self._patched_instance_forwards[key] = (module, had, original)

    def _apply_patches(self, model):
        name = model.__class__.__name__.lower()
        for arch in self._ARCHS:
            if arch in name:
                self._patch(arch)
                return
        raise NotImplementedError(
            f"KVOffloadManager: no attention patch for {model.__class__.__name__}")

    def _patch(self, arch: str):
        if arch == "qwen3":
            import transformers.models.qwen3.modeling_qwen3 as m
            cls, fwd = m.Qwen3Attention, _make_qwen3_forward(self.kvcms)
        elif arch == "qwen2":
            import transformers.models.qwen2.modeling_qwen2 as m
            cls, fwd = m.Qwen2Attention, _make_qwen2_forward(self.kvcms)
        elif arch == "llama":
            import transformers.models.llama.modeling_llama as m
            cls, fwd = m.LlamaAttention, _make_llama_forward(self.kvcms)
        elif arch == "gemma2":
            import transformers.models.gemma2.modeling_gemma2 as m
            cls, fwd = m.Gemma2Attention, _make_gemma2_forward(self.kvcms)
        elif arch == "mistral":
            import transformers.models.mistral.modeling_mistral as m
            cls, fwd = m.MistralAttention, _make_llama_forward(self.kvcms)
        elif arch == "ministral":
            import transformers.models.ministral.modeling_ministral as m
            cls, fwd = m.MinistralAttention, _make_llama_forward(self.kvcms)
        elif arch == "olmo2":
            import transformers.models.olmo2.modeling_olmo2 as m
            cls, fwd = m.Olmo2Attention, _make_olmo2_forward(self.kvcms)
        else:
            raise ValueError(arch)
        self._patched[arch] = (cls, fwd)
