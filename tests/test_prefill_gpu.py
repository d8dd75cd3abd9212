"""Parity of the CUDA chunk-prefill attention (helm_paged_prefill_attention,
through the C ABI) with the CPU oracle, for each of its kernels: the tcgen05
kernel with two query tiles per CTA (default), the one-tile tcgen05 kernel
(HELM_B200_PREFILL_KERNEL=tc1) and the mma.sync one (=mma).

A prefill chunk is, row by row, the reference's streaming attention
(helm/runtime/kv_cache.py:469-555) for one query with the mask row of that
query: the oracle (pinned to the reference by the golden fixtures in
test_oracle.py) is called once per query position with mask[:, 0, s, :] plus
the causal limit.  The pool is filled with NaN before the pages are written,
so a stale row that leaked into a result would show up.

Tolerances (fp32 accumulation; output in the model dtype, P rounded to it for
the tensor-core P.V product):
  bf16: |gpu - oracle| <= 1e-2 + 1e-2 |oracle|
  fp16: |gpu - oracle| <= 2e-3 + 4e-3 |oracle|
"""
import numpy as np
import pytest
import torch

import oracle
from helm_b200 import _capi

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: (1e-2, 1e-2), torch.float16: (2e-3, 4e-3)}
ORACLE_DT = {torch.bfloat16: 2, torch.float16: 1}


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def _setup(dev, dtype, B, Hq, Hkv, D, P, lens, S, seed):
    g = torch.Generator().manual_seed(seed)
    maxp = max((l + P - 1) // P for l in lens)
    slots = B * maxp + 5
    pool = torch.full((slots, 2, Hkv, P, D), float("nan"), dtype=dtype)
    perm = torch.randperm(slots, generator=g)[:B * maxp].view(B, maxp).to(torch.int32)
    for b, L in enumerate(lens):
        kv = torch.randn(2, Hkv, L, D, generator=g).to(dtype)
        for j in range(0, L, P):
            n = min(P, L - j)
            pool[perm[b, j // P], :, :, :n] = kv[:, :, j:j + n]
    q = torch.randn(B, Hq, S, D, generator=g).to(dtype)
    return pool, perm, q, g


def _oracle(pool, perm, q, lens, P, Hkv, mask, causal, softcap, scale):
    """[B, Hq, S, D] fp32: the decode oracle once per query position."""
    B, Hq, S, D = q.shape
    T = max(lens)
    bits = pool.view(torch.int16).numpy().view(np.uint16)
    num_pages, page_used = oracle.dense_page_lists(lens, P, perm.shape[1])
    out = np.zeros((B, Hq, S, D), np.float32)
    for s in range(S):
        m = np.zeros((B, T), np.float32)
        if mask is not None:
            mm = mask[:, 0, s, :T].float().numpy()
            m += np.broadcast_to(mm, (B, T))
        if causal:
            for b, L in enumerate(lens):
                m[b, L - S + s + 1:] = -np.inf
        o, _ = oracle.paged_attention(q[:, :, s].float().numpy(), bits, ORACLE_DT[q.dtype],
                                      perm.numpy(), num_pages, page_used, num_kv_heads=Hkv,
                                      page_size=P, scale=scale, softcap=softcap, mask=m,
                                      threads=8)
        out[:, :, s] = o
    return out


def _chunk_mask(lens, S, dtype, pad=None):
    """HELM's chunk-prefill mask (pipeline_runtime.py:96-112): queries at
    [past, past+S) see keys <= their position, plus key padding."""
    B, T = len(lens), max(lens)
    mn = torch.finfo(dtype).min
    m = torch.full((B, 1, S, T), mn, dtype=dtype)
    for b, L in enumerate(lens):
        past = L - S
        for i in range(S):
            m[b, 0, i, :past + i + 1] = 0
        if pad and b in pad:
            m[b, 0, :, :pad[b]] = m[b, 0, :, :pad[b]] + mn
    return m


CASES = [
    # dtype, B, Hq, Hkv, D, P, lens, S, mask, causal, softcap
    (torch.bfloat16, 2, 8, 2, 128, 16, [300, 517], 40, "helm", False, 0.0),
    (torch.float16, 1, 4, 4, 64, 64, [130], 130, None, True, 0.0),
    (torch.bfloat16, 3, 16, 8, 128, 32, [64, 1000, 65], 33, "fp32", True, 30.0),
    (torch.bfloat16, 2, 8, 1, 64, 16, [50, 64], 50, None, True, 0.0),
    (torch.bfloat16, 1, 8, 8, 128, 64, [4096], 16, None, True, 0.0),
    (torch.float16, 2, 12, 4, 128, 16, [777, 129], 100, "helm", False, 0.0),
]


@pytest.fixture(params=["tc", "tc1", "mma"])
def kernel(request, monkeypatch):
    monkeypatch.setenv("HELM_B200_PREFILL_KERNEL", request.param)
    return request.param


@pytest.mark.parametrize("case", CASES, ids=[f"case{i}" for i in range(len(CASES))])
def test_prefill_kernel_matches_oracle(case, kernel):
    dev = _cuda()
    dtype, B, Hq, Hkv, D, P, lens, S, mask_kind, causal, softcap = case
    pool, perm, q, g = _setup(dev, dtype, B, Hq, Hkv, D, P, lens, S, seed=len(lens) * 7 + S)
    T = max(lens)
    mask = None
    if mask_kind == "helm":
        mask = _chunk_mask(lens, S, dtype, pad={0: 7})
    elif mask_kind == "fp32":
        mask = (torch.rand(1, 1, S, T, generator=g) * 2 - 1).float()
    scale = D ** -0.5
    out = _capi.paged_prefill_attention(
        q.to(dev), pool.to(dev), perm.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev),
        num_kv_heads=Hkv, page_size=P, scale=scale, max_kv_len=T,
        mask=None if mask is None else mask.to(dev), causal=causal, softcap=softcap)
    torch.cuda.synchronize()
    assert _capi.device_status(dev) == 0
    ref = _oracle(pool, perm, q, lens, P, Hkv, mask, causal, softcap, scale)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    atol, rtol = TOL[dtype]
    err = np.abs(got - ref)
    assert (err <= atol + rtol * np.abs(ref)).all(), err.max()


def test_prefill_rows_without_keys_are_zero(kernel):
    """A query row whose every key is masked with -inf gets zeros (the
    reference's running max stays -inf there); the other rows are unaffected."""
    dev = _cuda()
    dtype, Hq, Hkv, D, P, lens, S = torch.bfloat16, 4, 2, 128, 16, [200], 8
    pool, perm, q, _ = _setup(dev, dtype, 1, Hq, Hkv, D, P, lens, S, seed=3)
    mask = torch.zeros(1, 1, S, lens[0], dtype=torch.float32)
    mask[0, 0, 3] = -float("inf")
    out = _capi.paged_prefill_attention(
        q.to(dev), pool.to(dev), perm.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev),
        num_kv_heads=Hkv, page_size=P, scale=D ** -0.5, max_kv_len=lens[0], mask=mask.to(dev))
    got = out.float().cpu()
    assert torch.all(got[0, :, 3] == 0)
    mask[0, 0, 3] = 0
    ref = _oracle(pool, perm, q, lens, P, Hkv, mask, False, 0.0, D ** -0.5)
    keep = [s for s in range(S) if s != 3]
    err = (got[0, :, keep] - torch.from_numpy(ref)[0, :, keep]).abs()
    assert err.max() <= 1e-2 + 1e-2 * float(np.abs(ref).max())


PAD_CASES = [
    # dtype, Hq, Hkv, D, P, lens, S, left pads per sequence
    (torch.bfloat16, 8, 2, 128, 16, [700, 900, 333], 100, [70, 0, 200]),
    (torch.float16, 8, 8, 64, 64, [520, 515], 129, [64, 3]),
    (torch.bfloat16, 40, 8, 128, 64, [4096], 16, [1000]),   # split key range, empty splits
]


@pytest.mark.parametrize("case", PAD_CASES, ids=[f"pad{i}" for i in range(len(PAD_CASES))])
def test_prefill_key_starts_match_padding_mask(case, kernel):
    """HELM's chunk mask of a left-padded batch (causal + key padding,
    pipeline_runtime.py:96-112) given as causal=True and kv_starts = the pad
    lengths, with no mask read: the oracle with the full additive mask, and the
    kernel reading that mask, agree with it.  Starts fall inside tiles, on tile
    edges and at 0."""
    dev = _cuda()
    dtype, Hq, Hkv, D, P, lens, S, pads = case
    B, T = len(lens), max(lens)
    pool, perm, q, _ = _setup(dev, dtype, B, Hq, Hkv, D, P, lens, S, seed=sum(pads) + S)
    mask = _chunk_mask(lens, S, dtype, pad={b: p for b, p in enumerate(pads) if p})
    scale = D ** -0.5
    args = (q.to(dev), pool.to(dev), perm.to(dev),
            torch.tensor(lens, dtype=torch.int32, device=dev))
    kw = dict(num_kv_heads=Hkv, page_size=P, scale=scale, max_kv_len=T)
    got = _capi.paged_prefill_attention(
        *args, causal=True, kv_starts=torch.tensor(pads, dtype=torch.int32, device=dev), **kw)
    read = _capi.paged_prefill_attention(*args, mask=mask.to(dev), **kw)
    torch.cuda.synchronize()
    assert _capi.device_status(dev) == 0
    ref = _oracle(pool, perm, q, lens, P, Hkv, mask, False, 0.0, scale)
    g, r = got.float().cpu().numpy(), read.float().cpu().numpy()
    assert np.isfinite(g).all()
    atol, rtol = TOL[dtype]
    assert (np.abs(g - ref) <= atol + rtol * np.abs(ref)).all(), np.abs(g - ref).max()
    assert (np.abs(g - r) <= atol + rtol * np.abs(r)).all(), np.abs(g - r).max()


def test_prefill_output_layout_and_arguments(kernel):
    """The default output is a [B, Hq, S, D] view of a [B, S, Hq, D] buffer
    (what the attention forward reshapes next); a strided caller buffer is
    honoured; bad shapes are refused with a status, not a fault."""
    dev = _cuda()
    dtype, Hq, Hkv, D, P, lens, S = torch.bfloat16, 4, 2, 64, 16, [96], 32
    pool, perm, q, _ = _setup(dev, dtype, 1, Hq, Hkv, D, P, lens, S, seed=5)
    args = (q.to(dev), pool.to(dev), perm.to(dev), torch.tensor(lens, dtype=torch.int32,
                                                                   device=dev))
    kw = dict(num_kv_heads=Hkv, page_size=P, scale=D ** -0.5, max_kv_len=lens[0], causal=True)
    a = _capi.paged_prefill_attention(*args, **kw)
    assert a.shape == (1, Hq, S, D) and a.transpose(1, 2).is_contiguous()
    b = torch.empty(1, Hq, S, D, dtype=dtype, device=dev)
    _capi.paged_prefill_attention(*args, out=b, **kw)
    assert torch.equal(a, b)
    with pytest.raises(_capi.HelmError):
        _capi.paged_prefill_attention(*args, **{**kw, "page_size": 8})


def test_prefill_kernel_matches_reference_golden(prefill_golden, kernel):
    """Both kernels on the reference's own prefill-chunk outputs
    (tests/golden/prefill.npz, produced by running perform_streaming_attention
    with HELM's chunk masks): within the model-dtype tolerance of the
    reference's fp32 result."""
    dev = _cuda()
    for name, c in prefill_golden.items():
        dtype = torch.float16 if c["dtype"] == "float16" else torch.bfloat16
        bits = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(dtype)  # noqa: E731
        q, pool = bits(c["q"]), bits(c["pool"])
        lens = [int(x) for x in c["lens"]]
        mask = torch.from_numpy(c["mask"]).to(dtype)
        out = _capi.paged_prefill_attention(
            q.to(dev), pool.to(dev), torch.from_numpy(c["page_table"]).to(dev),
            torch.tensor(lens, dtype=torch.int32, device=dev), num_kv_heads=c["Hkv"],
            page_size=c["P"], scale=c["D"] ** -0.5, max_kv_len=max(lens), mask=mask.to(dev),
            softcap=c["softcap_f"])
        got = out.float().cpu().numpy()
        ref = c["out_fp32"]
        atol, rtol = TOL[dtype]
        assert np.isfinite(got).all(), name
        assert (np.abs(got - ref) <= atol + rtol * np.abs(ref)).all(), (name, np.abs(got - ref).max())
