"""Parity of the CUDA paged decode attention (through the C ABI) with the
reference's outputs (golden fixtures) and with the CPU oracle.

Tolerances (bf16 / fp16 model dtypes; fp32 accumulation everywhere):
  O   : |gpu - oracle_fp32| <= ATOL + RTOL * |oracle_fp32|
        bf16: ATOL 1e-2, RTOL 1e-2   fp16: ATOL 2e-3, RTOL 4e-3
        (the output is rounded to the model dtype and P is rounded to it for
        the tensor-core PV product)
  LSE : |gpu - oracle| <= 1e-3 * max(1, |oracle|)
"""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import norm_rope

pytestmark = pytest.mark.gpu

TOL = {"bfloat16": (1e-2, 1e-2), "float16": (2e-3, 4e-3)}


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def _tensor(bits, dtype, dev):
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16))
    return t.view(getattr(torch, dtype)).to(dev)


def _f32(bits, dtype):
    if dtype == "float16":
        return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)
    return norm_rope.bf16_bits_to_f32(bits)


def run_case(case, dev, ragged=None, hint=0):
    from helm_b200 import _capi
    dtype = case["dtype"]
    q = _tensor(case["q"], dtype, dev)
    pool = _tensor(case["pool"], dtype, dev)
    pt = torch.from_numpy(case["page_table"]).to(dev)
    used = case["page_used"]
    lens = used.sum(axis=1).astype(np.int32)
    ragged = (not case["dense"]) if ragged is None else ragged
    kw = {}
    if ragged:
        start = np.zeros_like(used)
        start[:, 1:] = np.cumsum(used, axis=1)[:, :-1]
        kw = dict(num_pages=torch.from_numpy(case["num_pages"]).to(dev),
                  page_used=torch.from_numpy(used).to(dev),
                  page_start=torch.from_numpy(start.astype(np.int32)).to(dev))
    mask = case.get("mask")
    mask_t = torch.from_numpy(mask).to(dev) if mask is not None else None
    lse = torch.empty(q.shape[0], q.shape[1], dtype=torch.float32, device=dev)
    out, _ = _capi.paged_decode_attention(
        q, pool, pt, torch.from_numpy(lens).to(dev), num_kv_heads=case["Hkv"],
        page_size=case["P"], scale=case["scale_f"], softcap=case["softcap_f"] or None,
        mask=mask_t, lse=lse, max_kv_len_hint=hint, **kw)
    torch.cuda.synchronize()
    assert _capi.device_status(dev) == 0
    return out.float().cpu().numpy(), lse.cpu().numpy()


def oracle_case(case, threads=1):
    return oracle.paged_attention(
        _f32(case["q"], case["dtype"]), case["pool"],
        oracle.DT_F16 if case["dtype"] == "float16" else oracle.DT_BF16,
        case["page_table"], case["num_pages"], case["page_used"], num_kv_heads=case["Hkv"],
        page_size=case["P"], scale=case["scale_f"], softcap=case["softcap_f"],
        mask=case.get("mask"), threads=threads)


def assert_close(got, ref, dtype, what=""):
    atol, rtol = TOL[dtype]
    err = np.abs(got - ref) - (atol + rtol * np.abs(ref))
    assert np.all(err <= 0), f"{what}: max excess {err.max():.3g}"


def test_golden_cases(attention_golden):
    dev = _cuda()
    for name, case in attention_golden.items():
        out, lse = run_case(case, dev)
        ref32, ref_lse = oracle_case(case)
        assert_close(out, ref32, case["dtype"], name)
        # and against the reference's own output in the model dtype
        assert_close(out, _f32(case["out"], case["dtype"]), case["dtype"], name + " (golden)")
        fin = np.isfinite(ref_lse)
        assert np.array_equal(fin, np.isfinite(lse)), name
        assert np.all(np.abs(lse[fin] - ref_lse[fin]) <= 1e-3 * np.maximum(1, np.abs(ref_lse[fin]))), name


def test_dense_cases_through_ragged_path(attention_golden):
    """The ragged page-list form gives the same answer as dense paging."""
    dev = _cuda()
    for name, case in attention_golden.items():
        if not case["dense"]:
            continue
        a, la = run_case(case, dev, ragged=False)
        b, lb = run_case(case, dev, ragged=True)
        np.testing.assert_array_equal(a, b, err_msg=name)
        np.testing.assert_array_equal(la, lb, err_msg=name)


def test_empty_outputs_are_zero(attention_golden):
    dev = _cuda()
    for name in ("no_pages", "zero_used_page"):
        out, lse = run_case(attention_golden[name], dev)
        assert np.all(out == 0) and np.all(np.isneginf(lse)), name


def _random_problem(B, Hq, Hkv, D, P, lens, pool_pages, dtype=torch.bfloat16, seed=0):
    g = torch.Generator().manual_seed(seed)
    maxp = max(1, max((L + P - 1) // P for L in lens))
    perm = torch.randperm(pool_pages, generator=g)
    pt = perm[:B * maxp].view(B, maxp).to(torch.int32)
    pool = torch.randn(pool_pages, 2, Hkv, P, D, generator=g).to(dtype)
    q = torch.randn(B, Hq, D, generator=g).to(dtype)
    return q, pool, pt, torch.tensor(lens, dtype=torch.int32)


def _oracle_random(q, pool, pt, lens, Hkv, P, scale, threads):
    nump, used = oracle.dense_page_lists(lens.numpy(), P, pt.shape[1])
    bits = pool.view(torch.int16).numpy().view(np.uint16)
    dt = oracle.DT_BF16 if q.dtype == torch.bfloat16 else oracle.DT_F16
    return oracle.paged_attention(q.float().numpy(), bits, dt, pt.numpy(), nump, used,
                                  num_kv_heads=Hkv, page_size=P, scale=scale, threads=threads)


@pytest.mark.parametrize("B,Hq,Hkv,P,lens", [
    (4, 32, 8, 16, [4096, 3000, 1, 17]),       # config-2 heads, ragged lengths
    (1, 16, 8, 64, [576]),                     # config-1 layer at 512+64 tokens
    (3, 40, 8, 64, [1000, 0, 64]),             # Qwen3-14B heads (GQA 5), an empty sequence
    (2, 40, 40, 16, [300, 2048]),              # Llama-2-13B MHA, 16-token pages
])
def test_random_shapes_vs_oracle(B, Hq, Hkv, P, lens):
    dev = _cuda()
    from helm_b200 import _capi
    D = 128
    pool_pages = sum((L + P - 1) // P for L in lens) + 7
    pool_pages = max(pool_pages, B * max(1, max((L + P - 1) // P for L in lens)))
    q, pool, pt, kl = _random_problem(B, Hq, Hkv, D, P, lens, pool_pages)
    scale = D ** -0.5
    lse = torch.empty(B, Hq, device=dev)
    out, _ = _capi.paged_decode_attention(q.to(dev), pool.to(dev), pt.to(dev), kl.to(dev),
                                          num_kv_heads=Hkv, page_size=P, scale=scale, lse=lse)
    ref, ref_lse = _oracle_random(q, pool, pt, kl, Hkv, P, scale, os.cpu_count() or 1)
    assert_close(out.float().cpu().numpy(), ref, "bfloat16")
    got_lse = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(fin, np.isfinite(got_lse))
    assert np.all(np.abs(got_lse[fin] - ref_lse[fin]) <= 1e-3 * np.maximum(1, np.abs(ref_lse[fin])))
    assert _capi.device_status(dev) == 0


def test_config2_full_size_properties():
    """Config 2 at full size (B=4, 32q/8kv, D=128, T=32768, 16-token pages in a
    16384-page pool): all four sequences match the oracle, and moving every
    page to other pool slots (same contents) gives bit-identical output."""
    dev = _cuda()
    from helm_b200 import _capi
    B, Hq, Hkv, D, P, T, POOL = 4, 32, 8, 128, 16, 32768, 16384
    q, pool, pt, kl = _random_problem(B, Hq, Hkv, D, P, [T] * B, POOL, seed=0)
    scale = D ** -0.5
    qd, pd, ptd, kld = q.to(dev), pool.to(dev), pt.to(dev), kl.to(dev)
    lse = torch.empty(B, Hq, device=dev)
    out, _ = _capi.paged_decode_attention(qd, pd, ptd, kld, num_kv_heads=Hkv, page_size=P,
                                          scale=scale, lse=lse)
    out = out.float().cpu()
    # the oracle over the whole batch (threaded C port, ~35 ms per call on 16 cores)
    ref, ref_lse = _oracle_random(q, pool, pt, kl, Hkv, P, scale, os.cpu_count() or 1)
    assert_close(out.numpy(), ref, "bfloat16", "config2")
    assert np.all(np.abs(lse.cpu().numpy() - ref_lse) <= 1e-3 * np.maximum(1, np.abs(ref_lse)))
    # relocation: new slots = old slots shifted by a permutation of the pool
    g = torch.Generator().manual_seed(5)
    perm = torch.randperm(POOL, generator=g).to(dev)
    pool2 = torch.empty_like(pd)
    pool2[perm.long()] = pd
    pt2 = perm[ptd.long()].to(torch.int32)
    out2, _ = _capi.paged_decode_attention(qd, pool2, pt2, kld, num_kv_heads=Hkv, page_size=P,
                                           scale=scale)
    assert torch.equal(out2.float().cpu(), out)
    assert _capi.device_status(dev) == 0


def test_grid_size_does_not_change_result():
    """Different split-KV decompositions (grid hints) agree to fp32 rounding."""
    dev = _cuda()
    from helm_b200 import _capi
    q, pool, pt, kl = _random_problem(2, 32, 8, 128, 16, [5000, 777], 800, seed=3)
    args = (q.to(dev), pool.to(dev), pt.to(dev), kl.to(dev))
    outs = []
    for hint in (0, 16, 5000, 100000):
        o, _ = _capi.paged_decode_attention(*args, num_kv_heads=8, page_size=16,
                                            scale=128 ** -0.5, max_kv_len_hint=hint)
        outs.append(o.float().cpu())
    for o in outs[1:]:
        assert torch.allclose(o, outs[0], atol=1e-2, rtol=1e-2)


def test_bad_page_entry_is_reported_not_faulted():
    """An out-of-range page-table entry is clamped and flagged in the device
    status word; the call completes."""
    dev = _cuda()
    from helm_b200 import _capi
    q, pool, pt, kl = _random_problem(1, 8, 2, 128, 16, [64], 8, seed=1)
    pt[0, 1] = 1000  # pool has 8 slots
    _capi.paged_decode_attention(q.to(dev), pool.to(dev), pt.to(dev), kl.to(dev),
                                 num_kv_heads=2, page_size=16, scale=0.1)
    st = _capi.device_status(dev)
    assert st & _capi.DEV_BAD_PAGE
    assert _capi.device_status(dev) == 0  # cleared by the previous read


def test_invalid_arguments_raise():
    dev = _cuda()
    from helm_b200 import _capi
    q, pool, pt, kl = _random_problem(1, 8, 2, 128, 16, [64], 8, seed=1)
    with pytest.raises(_capi.HelmError):  # 3 KV heads do not divide 8 query heads
        _capi.paged_decode_attention(q.to(dev), pool.to(dev), pt.to(dev), kl.to(dev),
                                     num_kv_heads=3, page_size=16, scale=0.1)
    with pytest.raises(_capi.HelmError):  # head_dim 96 unsupported
        q2 = torch.randn(1, 8, 96, dtype=torch.bfloat16, device=dev)
        pool2 = torch.randn(8, 2, 2, 16, 96, dtype=torch.bfloat16, device=dev)
        _capi.paged_decode_attention(q2, pool2, pt.to(dev), kl.to(dev), num_kv_heads=2,
                                     page_size=16, scale=0.1)


def _append_then_decode(steps, overlap, graph):
    """Per step: the fused append writes q_out and one K/V row per sequence,
    then decode attention reads both.  Returns the outputs of every step."""
    from helm_b200 import _capi
    dev = torch.device("cuda:0")
    B, Hq, Hkv, D, P, T0 = 2, 8, 2, 128, 16, 100
    g = torch.Generator().manual_seed(11)
    npg = (T0 + steps) // P + 1
    pool = torch.randn(B * npg, 2, Hkv, P, D, generator=g).to(torch.bfloat16).to(dev)
    pt = torch.arange(B * npg, dtype=torch.int32).view(B, npg).to(dev)
    qs = torch.randn(steps, B, Hq, D, generator=g).to(torch.bfloat16).to(dev)
    ks = torch.randn(steps, B, Hkv, D, generator=g).to(torch.bfloat16).to(dev)
    vs = torch.randn(steps, B, Hkv, D, generator=g).to(torch.bfloat16).to(dev)
    cos = torch.rand(steps, B, D, generator=g).to(torch.bfloat16).to(dev)
    sin = torch.rand(steps, B, D, generator=g).to(torch.bfloat16).to(dev)
    rows = torch.stack([(pt[:, (T0 + s) // P].long() * P + (T0 + s) % P) for s in range(steps)])
    lens = torch.stack([torch.full((B,), T0 + s + 1, dtype=torch.int32, device=dev)
                        for s in range(steps)])
    q_out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device=dev)
    outs = torch.empty(steps, B, Hq, D, dtype=torch.bfloat16, device=dev)

    def run():
        for s in range(steps):
            _capi.kv_append(q=qs[s], k=ks[s], v=vs[s], q_out=q_out, cos=cos[s], sin=sin[s],
                            pool=pool, slot_rows=rows[s], page_size=P)
            _capi.paged_decode_attention(q_out, pool, pt, lens[s], num_kv_heads=Hkv, page_size=P,
                                         scale=D ** -0.5, out=outs[s], max_kv_len_hint=T0 + steps)

    with _capi.decode_overlap(overlap):
        if graph:
            run()        # warm-up outside capture (workspace), then reset the pool rows
            torch.cuda.synchronize()
            cg = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                with torch.cuda.graph(cg, stream=side):
                    run()
            torch.cuda.current_stream(dev).wait_stream(side)
            cg.replay()
        else:
            run()
    torch.cuda.synchronize()
    assert _capi.device_status(dev) == 0
    return outs.cpu()


def test_decode_overlap_sees_the_preceding_append():
    """Decode overlap places the decode kernel while the fused append that
    writes its query and newest K/V rows still runs; the results must equal
    those of plain stream order, bit for bit, eager and inside a CUDA graph."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    ref = _append_then_decode(6, overlap=False, graph=False)
    assert torch.equal(_append_then_decode(6, overlap=True, graph=False), ref)
    assert torch.equal(_append_then_decode(6, overlap=True, graph=True), ref)
