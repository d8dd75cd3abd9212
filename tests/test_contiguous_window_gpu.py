"""The all-GPU decode window (KVCacheManager.build_contiguous and friends)
against the reference's contiguous path, run by tests/golden/make_golden.py
(tests/golden/contiguous.npz).

HELM's inference front end enables the contiguous path on all-GPU plans
(cont_capacity = max_input_tokens + 512, helm/runtime/inference.py:729-731);
_decode_batched then writes decode tokens to per-layer buffers until
cont_seq_len reaches the capacity and migrates them to pages
(helm/runtime/kv_offload.py:115-142, kv_cache.py:269-354).  Here the window is
a reservation of page-pool slots read by the paged kernel.  Checked, through
_decode_batched exactly as the reference calls it (2 layers, batch 2, 37-token
prefill, capacity 64, 35 decode steps: 27 in the window, the migration, 8 on
pages):
  * every step's attention output against the reference's
    (bf16: |d| <= 1e-2 + 1e-2 |ref|) and against this library's own page path
    without a window (same bound);
  * use_contiguous / cont_seq_len / cont_prefill_len after every step: equal;
  * final page placement (page ids, start and used tokens, tier): equal.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "contiguous.npz")


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def _t(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _run(z, dev, window: bool):
    from helm_b200.runtime.kv_allocator import KVAllocator
    from helm_b200.runtime.kv_cache import KVCacheManager
    from helm_b200.runtime import kv_offload as ko
    L, B, Hq, Hkv, D, P, S, CAP, STEPS = (int(x) for x in z["meta"])
    alloc = KVAllocator(L, Hkv, D, page_size=P, dtype=torch.bfloat16)
    mgrs = [KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12) for _ in range(B)]
    if window:
        for m in mgrs:
            assert m.build_contiguous(num_layers=L, num_kv_heads=Hkv, head_dim=D, capacity=CAP,
                                      device=dev, dtype=torch.bfloat16)
    pre_k, pre_v = _t(z["pre_k"], dev), _t(z["pre_v"], dev)
    q, k, v = _t(z["q"], dev), _t(z["k"], dev), _t(z["v"], dev)
    for lid in range(L):
        ko._append_prefill_batched(mgrs, pre_k[lid], pre_v[lid], lid)
    outs, counters = [], []
    for st in range(STEPS):
        for lid in range(L):
            o = ko._decode_batched(mgrs, q[st, lid], k[st, lid], v[st, lid], lid, D ** -0.5)
            outs.append(o[:, :, 0].float().cpu())
        counters.append([int(mgrs[0].use_contiguous), mgrs[0].cont_seq_len,
                         mgrs[0].cont_prefill_len])
    torch.cuda.synchronize()
    placement = []
    for b, m in enumerate(mgrs):
        for lid in sorted(m.layers):
            for p in m.layers[lid].pages:
                placement.append([b, lid, p.page_id, p.start_token, p.used_tokens,
                                  p.capacity_tokens, 1 if p.state == "GPU" else 0])
    out = torch.stack(outs).view(STEPS, L, B, Hq, D).numpy()
    return out, np.array(counters), np.array(placement), mgrs


def test_window_matches_reference_contiguous_path():
    dev = _cuda()
    from helm_b200 import _capi
    from oracle.norm_rope import bf16_bits_to_f32
    z = np.load(GOLDEN)
    out, counters, placement, mgrs = _run(z, dev, window=True)
    ref = bf16_bits_to_f32(z["out"])
    bad = np.abs(out - ref) > 1e-2 + 1e-2 * np.abs(ref)
    assert not bad.any(), f"{bad.sum()} outputs off, first step {np.nonzero(bad)[0][0]}"
    np.testing.assert_array_equal(counters, z["counters"])
    np.testing.assert_array_equal(placement, z["placement"])
    assert not mgrs[0].use_contiguous and not mgrs[0]._window   # migrated and released
    assert _capi.device_status(dev) == 0


def test_window_outputs_equal_page_path():
    """The window phase reads the same tokens as the page path would."""
    dev = _cuda()
    z = np.load(GOLDEN)
    win, _, _, _ = _run(z, dev, window=True)
    pages, counters, _, _ = _run(z, dev, window=False)
    assert counters[:, 0].sum() == 0
    bad = np.abs(win - pages) > 1e-2 + 1e-2 * np.abs(pages)
    assert not bad.any()


def test_window_dense_accessors():
    """get_kv_contiguous / cont_K give every cached token of the layer in
    order (prefill pages, then the window), as the reference's buffers hold
    them; reset_contiguous re-arms a kept window."""
    dev = _cuda()
    from helm_b200.runtime.kv_allocator import KVAllocator
    from helm_b200.runtime.kv_cache import KVCacheManager
    from helm_b200.runtime import kv_offload as ko
    g = torch.Generator().manual_seed(5)
    H, D, P, S = 2, 64, 16, 21
    alloc = KVAllocator(1, H, D, page_size=P, dtype=torch.bfloat16)
    m = KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12)
    assert m.build_contiguous(num_layers=1, num_kv_heads=H, head_dim=D, capacity=48,
                              device=dev, dtype=torch.bfloat16)
    kp = torch.randn(1, H, S, D, generator=g).to(torch.bfloat16).to(dev)
    vp = torch.randn(1, H, S, D, generator=g).to(torch.bfloat16).to(dev)
    ko._append_prefill_batched([m], kp, vp, 0)
    ks, vs = [kp], [vp]
    for _ in range(20):
        kn = torch.randn(1, H, 1, D, generator=g).to(torch.bfloat16).to(dev)
        vn = torch.randn(1, H, 1, D, generator=g).to(torch.bfloat16).to(dev)
        m.write_decode_contiguous(0, kn, vn)
        ks.append(kn)
        vs.append(vn)
        K, V = m.get_kv_contiguous(0)
        assert torch.equal(K, torch.cat(ks, dim=2)) and torch.equal(V, torch.cat(vs, dim=2))
        m.advance_contiguous()
    assert len(m.layers[0].pages) == 2      # decode tokens stay out of the page list
    buf = m.cont_K[0]
    assert buf.shape == (1, H, 48, D)
    assert torch.equal(buf[:, :, :S + 20], torch.cat(ks, dim=2))
    assert torch.count_nonzero(buf[:, :, S + 20:]) == 0
    m.clear()
    m.reset_contiguous()
    assert m.use_contiguous and m.cont_seq_len == 0
    m.drop_contiguous()
    m.reset_contiguous()
    assert not m.use_contiguous
