"""GPU behaviour of the drop-in runtime.

* Placement parity: every GPU-tier scenario of tests/golden/placement.json
  (produced by running the reference's KVAllocator/KVCacheManager) replayed on
  helm_b200.runtime with real HBM and pinned-host pages: identical page ids,
  tiers, token ranges, free lists and stats after every step, and every cached
  row bit-exact where the metadata says it is.
* perform_streaming_attention: the cases of the reference's
  tests/unit/runtime/test_streaming_attention.py (hand-made pages, masks,
  soft-cap, GQA, fp16, empty pages) on CUDA at head_dim 64, against an eager
  fp32 computation; plus pool pages with mixed GPU/host residency.
Tolerance as in the kernel tests: bf16 1e-2 + 1e-2|ref|, fp16 2e-3 + 4e-3|ref|.
"""
import math

import numpy as np
import pytest
import torch

from helm_b200.runtime.kv_allocator import KVAllocator
from helm_b200.runtime.kv_cache import (KVCacheManager, KVPage, _get_kv_copy_stream,
                                        get_paging_stats, perform_streaming_attention,
                                        reset_paging_stats)
from test_runtime_cpu import replay

pytestmark = pytest.mark.gpu
TOL = {torch.bfloat16: (1e-2, 1e-2), torch.float16: (2e-3, 4e-3)}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def _close(got, ref, dtype):
    atol, rtol = TOL[dtype]
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.all((got - ref).abs() <= atol + rtol * ref.abs()), (got - ref).abs().max()


# ── placement ──────────────────────────────────────────────────────────────────
def test_gpu_tier_placement_matches_reference(dev, placement_golden, monkeypatch):
    # also assert, at every residency decision, that the incremental evictable
    # count equals a full scan of the pages
    monkeypatch.setenv("HELM_B200_CHECK_RESIDENCY", "1")
    n = 0
    for entry in placement_golden:
        sc = entry["scenario"]
        if not any(len(op) > 3 and op[-1] == "cuda" for op in sc["ops"]):
            continue
        snaps = replay(sc, "cuda")
        assert snaps == entry["snapshots"], sc["name"]
        n += 1
    assert n >= 9


def test_tail_page_protected_and_eviction_counted(dev):
    alloc = KVAllocator(2, 2, 8, page_size=4, dtype=torch.float32)
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12)
    k = torch.randn(1, 2, 8, 8, device=dev)
    mgr.append_prefill(0, k, k)
    tail = mgr.layers[0].tail_page
    reset_paging_stats()
    mgr.evict_pages(999999)
    assert tail is mgr.layers[0].tail_page and tail.state == "GPU"
    s = get_paging_stats()
    assert s["pages_evicted"] == 1 and s["bytes_evicted"] > 0 and s["evict_calls"] == 1
    ev = mgr.layers[0].pages[0]
    assert ev.state == "CPU" and ev.k_tensor.is_pinned()
    assert torch.equal(ev.k_tensor[0, :, :4].cpu(), k[0, :, :4].cpu())


def test_move_page_cpu_to_gpu(dev):
    a = KVAllocator(2, 2, 8, page_size=4, dtype=torch.float32)
    page = a.allocate(torch.device("cpu"))
    page.layer_id, page.start_token, page.used_tokens = 2, 8, 3
    page.k_tensor[:, :, :3] = 7.0
    page.v_tensor[:, :, :3] = 8.0
    free_before = len(a.cpu_free_pool)
    new = a.move_page(page, dev)
    torch.cuda.synchronize()
    assert new.device.type == "cuda" and (new.layer_id, new.start_token, new.used_tokens) == (2, 8, 3)
    assert torch.all(new.k_tensor[:, :, :3].cpu() == 7.0) and torch.all(new.v_tensor[:, :, :3].cpu() == 8.0)
    assert len(a.cpu_free_pool) == free_before + 1


def test_copy_stream_memoized(dev):
    assert _get_kv_copy_stream(dev) is _get_kv_copy_stream(dev)
    assert _get_kv_copy_stream(dev).device == dev


# ── perform_streaming_attention (reference test_streaming_attention.py) ────────
def _page(k, v, page_id=0, start=0, state="CPU"):
    return KVPage(page_id=page_id, layer_id=0, start_token=start, used_tokens=k.size(2),
                  capacity_tokens=k.size(2), k_tensor=k.clone(), v_tensor=v.clone(),
                  device=k.device, state=state)


def _eager(q, k, v, scale=None, mask=None, softcap=None):
    if scale is None:
        scale = 1.0 / math.sqrt(q.size(-1))
    if k.size(1) != q.size(1):
        g = q.size(1) // k.size(1)
        k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
    w = torch.matmul(q.float(), k.float().transpose(-2, -1)) * scale
    if softcap is not None:
        w = torch.tanh(w / softcap) * softcap
    if mask is not None:
        w = w + mask.float()
    return torch.matmul(torch.softmax(w, -1), v.float())


def _paged(sizes, H=2, D=64, kv_heads=None, dtype=torch.bfloat16, dev="cuda", state="GPU"):
    kv_heads = kv_heads or H
    pages, ks, vs, start = [], [], [], 0
    for i, sz in enumerate(sizes):
        k = torch.randn(1, kv_heads, sz, D).to(dtype).to(dev)
        v = torch.randn(1, kv_heads, sz, D).to(dtype).to(dev)
        pages.append(_page(k, v, i, start, state))
        ks.append(k)
        vs.append(v)
        start += sz
    return pages, torch.cat(ks, 2), torch.cat(vs, 2)


@pytest.mark.parametrize("sizes", [[4], [4, 3], [3, 5, 2]])
def test_pages_match_eager(dev, sizes):
    torch.manual_seed(len(sizes))
    pages, K, V = _paged(sizes)
    q = torch.randn(1, 2, 1, 64).to(torch.bfloat16).to(dev)
    out = perform_streaming_attention(q, pages)
    assert out.shape == q.shape and out.dtype == q.dtype
    _close(out, _eager(q, K, V), torch.bfloat16)


def test_no_pages_and_empty_pages(dev):
    q = torch.randn(1, 2, 1, 64, dtype=torch.bfloat16, device=dev)
    assert torch.all(perform_streaming_attention(q, []) == 0)
    pages, K, V = _paged([4])
    pages[0].used_tokens = 0
    assert torch.all(perform_streaming_attention(q, pages) == 0)
    real, K2, V2 = _paged([4])
    empty, _, _ = _paged([4])
    empty[0].used_tokens = 0
    a = perform_streaming_attention(q, empty + real)
    b = perform_streaming_attention(q, real)
    assert torch.equal(a, b)


def test_scale_dtype_gqa_large_logits(dev):
    torch.manual_seed(3)
    pages, K, V = _paged([3], H=1)
    q = torch.randn(1, 1, 1, 64, dtype=torch.bfloat16, device=dev)
    _close(perform_streaming_attention(q, pages, scale=0.25), _eager(q, K, V, scale=0.25),
           torch.bfloat16)
    pages, K, V = _paged([6], H=4, kv_heads=2)
    q = torch.randn(1, 4, 1, 64, dtype=torch.bfloat16, device=dev)
    _close(perform_streaming_attention(q, pages), _eager(q, K, V), torch.bfloat16)
    pages, K, V = _paged([4, 4], dtype=torch.float16)
    q = torch.randn(1, 2, 1, 64, dtype=torch.float16, device=dev)
    out = perform_streaming_attention(q, pages)
    assert out.dtype == torch.float16
    _close(out, _eager(q, K, V), torch.float16)
    k = torch.full((1, 1, 8, 64), 100.0, dtype=torch.bfloat16, device=dev)
    v = torch.randn(1, 1, 8, 64, dtype=torch.bfloat16, device=dev)
    q = torch.full((1, 1, 1, 64), 100.0, dtype=torch.bfloat16, device=dev)
    out = perform_streaming_attention(q, [_page(k, v)])
    assert torch.isfinite(out).all()


def test_masks_softcap_and_batch_rows(dev):
    torch.manual_seed(1)
    pages, K, V = _paged([4, 4, 3])
    q = torch.randn(1, 2, 1, 64, dtype=torch.bfloat16, device=dev)
    mask = torch.zeros(1, 1, 1, 11, device=dev)
    mask[..., [0, 3, 4, 10]] = torch.finfo(torch.float32).min
    _close(perform_streaming_attention(q, pages, attention_mask=mask), _eager(q, K, V, mask=mask),
           torch.bfloat16)
    mask = torch.zeros(1, 1, 1, 11, device=dev)
    mask[..., :4] = torch.finfo(torch.float32).min      # first page fully masked
    _close(perform_streaming_attention(q, pages, attention_mask=mask), _eager(q, K, V, mask=mask),
           torch.bfloat16)
    _close(perform_streaming_attention(q, pages, softcap=50.0), _eager(q, K, V, softcap=50.0),
           torch.bfloat16)
    # several query rows over the same pages (batch dim broadcast, as in the reference)
    q4 = torch.randn(3, 2, 1, 64, dtype=torch.bfloat16, device=dev)
    _close(perform_streaming_attention(q4, pages), _eager(q4, K, V), torch.bfloat16)


def test_pool_pages_with_host_residency_match_all_gpu(dev):
    """The same cache with and without evictions gives the same attention, and
    the host-resident pages are counted as prefetched."""
    torch.manual_seed(7)
    H, D, P = 8, 128, 16
    results = []
    for watermark in (10 ** 12, 2 * 2 * H * P * D * 2):   # keep all / keep ~2 pages hot
        alloc = KVAllocator(1, H, D, page_size=P, dtype=torch.bfloat16)
        mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=watermark)
        g = torch.Generator().manual_seed(0)
        k = torch.randn(1, H, 300, D, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(1, H, 300, D, generator=g).to(torch.bfloat16).to(dev)
        mgr.append_prefill(0, k, v)
        for t in range(5):
            mgr.append_decode(0, k[:, :, t:t + 1], v[:, :, t:t + 1])
        q = torch.randn(1, 4 * H, 1, D, generator=g).to(torch.bfloat16).to(dev)
        reset_paging_stats()
        out = perform_streaming_attention(q, mgr.iterate_layer_pages(0))
        s = get_paging_stats()
        cold = sum(p.state == "CPU" for p in mgr.layers[0].pages)
        assert s["pages_prefetched"] == cold
        results.append((out, cold))
        ref = _eager(q, torch.cat([k, k[:, :, :5]], 2), torch.cat([v, v[:, :, :5]], 2))
        _close(out, ref, torch.bfloat16)
    assert results[0][1] == 0 and results[1][1] > 10
    assert torch.equal(results[0][0], results[1][0])


def test_cpu_pages_made_by_hand_with_cuda_query(dev):
    """Hand-made host pages (not pool slots) are copied in and counted."""
    torch.manual_seed(2)
    gpu_pages, K1, V1 = _paged([4], state="GPU")
    cpu_pages, K2, V2 = _paged([4], dev="cpu", state="CPU")
    q = torch.randn(1, 2, 1, 64, dtype=torch.bfloat16, device=dev)
    reset_paging_stats()
    out = perform_streaming_attention(q, gpu_pages + cpu_pages,
                                      attention_mask=torch.zeros(1, 1, 1, 8, device=dev))
    s = get_paging_stats()
    assert s["prefetch_calls"] == 1 and s["pages_prefetched"] == 1 and s["bytes_prefetched"] > 0
    _close(out, _eager(q, torch.cat([K1, K2.to(dev)], 2), torch.cat([V1, V2.to(dev)], 2)),
           torch.bfloat16)


@pytest.mark.parametrize("native", [False, True])
def test_dense_prefill_path_matches_page_walk(dev, monkeypatch, native):
    """A 64-token prefill chunk over 320 cached tokens: the device path
    (gather + library attention by default, the native paged kernel with
    HELM_B200_NATIVE_PREFILL=1 or a softcap) equals the fp32 page walk within
    the bf16 tolerance, with HELM's chunk-causal mask; with host-resident
    pages it declines (page walk used)."""
    from helm_b200.runtime.kv_cache import _prefill_over_pages
    from helm_b200.runtime.kv_offload import _prefill_dense_pages
    monkeypatch.setenv("HELM_B200_NATIVE_PREFILL", "1" if native else "0")
    torch.manual_seed(11)
    H, D, P, T, S = 2, 64, 16, 320, 64
    for watermark, expect_fast in ((10 ** 12, True), (2 * 2 * H * P * D * 2, False)):
        alloc = KVAllocator(1, H, D, page_size=P, dtype=torch.bfloat16)
        mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=watermark)
        k = torch.randn(1, H, T, D).to(torch.bfloat16).to(dev)
        v = torch.randn(1, H, T, D).to(torch.bfloat16).to(dev)
        mgr.append_prefill(0, k, v)
        q = torch.randn(1, 4 * H, S, D).to(torch.bfloat16).to(dev)
        past = T - S
        i = torch.arange(S, device=dev).view(S, 1)
        j = torch.arange(T, device=dev).view(1, T)
        mask = torch.where(j <= past + i, 0.0, torch.finfo(torch.bfloat16).min)
        mask = mask.to(torch.bfloat16).view(1, 1, S, T)
        for softcap in ((None, 30.0) if native else (None,)):
            fast = _prefill_dense_pages([mgr], q, 0, D ** -0.5, mask, softcap)
            ref = _prefill_over_pages(q, [mgr.iterate_layer_pages(0)], D ** -0.5, mask, softcap)
            if expect_fast:
                assert fast is not None
                _close(fast, ref, torch.bfloat16)
            else:
                assert fast is None


def test_dense_prefill_padding_mask_runs_on_the_kernel(dev, monkeypatch):
    """A later prefill chunk of a left-padded batch (HELM's chunk mask plus key
    padding, pipeline_runtime.py:96-112) runs on the native kernel with the
    padding as per-sequence first keys (gather + library attention is not
    called) and equals the fp32 page walk within the bf16 tolerance; a mask
    that leaves a query row without any key still takes the library path."""
    from helm_b200 import _capi
    from helm_b200.runtime.kv_cache import _prefill_over_pages
    from helm_b200.runtime.kv_offload import _prefill_dense_pages
    monkeypatch.delenv("HELM_B200_NATIVE_PREFILL", raising=False)
    torch.manual_seed(12)
    H, D, P, T, S = 2, 128, 16, 400, 96
    pads = [37, 0, 150]
    alloc = KVAllocator(1, H, D, page_size=P, dtype=torch.bfloat16)
    mgrs = []
    for _ in pads:
        m = KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12)
        m.append_prefill(0, torch.randn(1, H, T, D).to(torch.bfloat16).to(dev),
                         torch.randn(1, H, T, D).to(torch.bfloat16).to(dev))
        mgrs.append(m)
    q = torch.randn(len(pads), 4 * H, S, D).to(torch.bfloat16).to(dev)
    mn = torch.finfo(torch.bfloat16).min
    i = torch.arange(S, device=dev).view(S, 1)
    j = torch.arange(T, device=dev).view(1, T)
    causal = torch.where(j <= T - S + i, 0.0, mn)
    keep = (j.view(1, T) >= torch.tensor(pads, device=dev).view(-1, 1)).float()
    mask = (causal.view(1, 1, S, T) + ((1.0 - keep) * mn).view(-1, 1, 1, T)).to(torch.bfloat16)
    calls = []
    real_gather = _capi.gather_kv
    monkeypatch.setattr(_capi, "gather_kv", lambda *a, **k: calls.append(1) or real_gather(*a, **k))
    fast = _prefill_dense_pages(mgrs, q, 0, D ** -0.5, mask)
    assert fast is not None and not calls
    ref = _prefill_over_pages(q, [m.iterate_layer_pages(0) for m in mgrs], D ** -0.5, mask, None)
    _close(fast, ref, torch.bfloat16)
    lone = mask.clone()
    lone[2, 0, 0, :] = mn       # query row 0 of sequence 2 sees no key: library path
    _prefill_dense_pages(mgrs, q, 0, D ** -0.5, lone)
    assert calls


def test_gemma2_sliding_window_known_answers(dev):
    """The reference's analytic check of the Gemma-2 forward
    (tests/unit/runtime/test_kv_offload.py:367-413), restated at a head size the
    GPU path serves (64, bf16): q, k, v each pick one hidden component, so the
    last of three prompt tokens scores 10 against token 0 and 0 against tokens
    1 and 2.  With a window of 2 it must average v over tokens 1 and 2:
    (1 + 2) / 2 = 1.5 (the window ignored would give ~100).  One decode step
    after it (v = 4) must give (2 + 4) / 2 = 3.0 from the paged path."""
    import torch.nn as nn
    from helm_b200.runtime.kv_offload import _make_gemma2_forward
    D = 64
    attn = nn.Module()
    attn.q_proj = nn.Linear(3, D, bias=False)
    attn.k_proj = nn.Linear(3, D, bias=False)
    attn.v_proj = nn.Linear(3, D, bias=False)
    attn.o_proj = nn.Linear(D, 1, bias=False)
    with torch.no_grad():
        for lin in (attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj):
            lin.weight.zero_()
        attn.q_proj.weight[0, 0] = 1.0
        attn.k_proj.weight[0, 1] = 1.0
        attn.v_proj.weight[0, 2] = 1.0
        attn.o_proj.weight[0, 0] = 1.0
    attn = attn.to(dev, torch.bfloat16)
    attn.head_dim, attn.layer_idx, attn.scaling = D, 0, 1.0
    attn.attn_logit_softcapping, attn.sliding_window = None, 2
    alloc = KVAllocator(1, 1, D, page_size=16, dtype=torch.bfloat16)
    kvcms = [KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12)]
    forward = _make_gemma2_forward(kvcms)
    h = torch.tensor([[[1.0, 10.0, 100.0], [1.0, 0.0, 1.0], [1.0, 0.0, 2.0]]],
                     dtype=torch.bfloat16, device=dev)
    lo = torch.finfo(torch.bfloat16).min
    causal = torch.triu(torch.full((3, 3), lo, device=dev), diagonal=1)
    causal = causal.to(torch.bfloat16)[None, None]
    ones = torch.ones(1, 3, D, dtype=torch.bfloat16, device=dev)   # RoPE at angle 0
    out, _ = forward(attn, h, (ones, torch.zeros_like(ones)), attention_mask=causal,
                     cache_position=torch.arange(3, device=dev))
    assert abs(out[0, 2, 0].item() - 1.5) < 1e-2
    h4 = torch.tensor([[[1.0, 0.0, 4.0]]], dtype=torch.bfloat16, device=dev)
    one = torch.ones(1, 1, D, dtype=torch.bfloat16, device=dev)
    out4, _ = forward(attn, h4, (one, torch.zeros_like(one)),
                      attention_mask=torch.zeros(1, 1, 1, 4, dtype=torch.bfloat16, device=dev),
                      cache_position=torch.tensor([3], device=dev))
    assert abs(out4[0, 0, 0].item() - 3.0) < 2e-2
