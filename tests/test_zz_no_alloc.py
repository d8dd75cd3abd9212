"""The allocation-free decode attention entry point agrees with the regular one.

helm_paged_decode_attention_noalloc exists for callers that cannot allocate
device memory (a server that hands all of HBM to its own pool at start-up, or
a decode loop that must not stall on cudaFree's device-wide synchronisation).
It uses a fixed scratch array inside the library instead of a caller-provided
workspace.  This test calls it through the C ABI twice in a row, with two
different shapes (so the second call reuses scratch the first one dirtied),
and checks each result against helm_paged_decode_attention on the same inputs:
the two run the same kernel with the same grid, so O and LSE must be
bit-identical.  It also checks that a shape needing more than the fixed
scratch is refused before any launch.

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import numpy as np
import pytest
import torch

from helm_b200 import _capi

pytestmark = pytest.mark.gpu


def _problem(B, Hq, Hkv, D, P, lens, seed):
    g = torch.Generator().manual_seed(seed)
    maxp = max(1, max((L + P - 1) // P for L in lens))
    pool_pages = B * maxp + 5
    perm = torch.randperm(pool_pages, generator=g)
    pt = perm[:B * maxp].view(B, maxp).to(torch.int32)
    pool = torch.randn(pool_pages, 2, Hkv, P, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    return q, pool, pt, torch.tensor(lens, dtype=torch.int32)


def _noalloc(q, pool, pt, kl, Hkv, P, scale):
    B, Hq, D = q.shape
    out = torch.empty_like(q)
    lse = torch.empty(B, Hq, dtype=torch.float32, device=q.device)
    rc = _capi.lib().helm_paged_decode_attention_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), pool.data_ptr(), pool.shape[0],
        pt.data_ptr(), pt.stride(0), pt.shape[1], kl.data_ptr(), None, None, None,
        None, 0, 0, out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(),
        B, Hq, Hkv, D, P, _capi.DTYPE_BF16, scale, 0.0, 0,
        torch.cuda.current_stream(q.device).cuda_stream)
    assert rc == 0, _capi.lib().helm_status_string(rc)
    return out, lse


def _check(dev, B, Hq, Hkv, P, lens, seed):
    D = 128
    scale = D ** -0.5
    q, pool, pt, kl = (t.to(dev) for t in _problem(B, Hq, Hkv, D, P, lens, seed))
    got, got_lse = _noalloc(q, pool, pt, kl, Hkv, P, scale)
    lse_ref = torch.empty(B, Hq, dtype=torch.float32, device=dev)
    ref, _ = _capi.paged_decode_attention(q, pool, pt, kl, num_kv_heads=Hkv, page_size=P,
                                          scale=scale, lse=lse_ref)
    torch.cuda.synchronize(dev)
    assert _capi.device_status(dev) == 0
    # same kernel, grid and inputs (the kernel uses no atomics): bit-identical,
    # so a stale value or an overlap in the reused scratch would show
    assert torch.equal(got, ref)
    gl, rl = got_lse.cpu().numpy(), lse_ref.cpu().numpy()
    fin = np.isfinite(rl)
    assert np.array_equal(fin, np.isfinite(gl))
    assert np.array_equal(gl[fin], rl[fin])


def test_noalloc_matches_regular_entry_point_twice_in_a_row():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda:0")
    # first call: many pairs, long ragged lengths, an empty sequence
    _check(dev, B=4, Hq=32, Hkv=8, P=16, lens=[4096, 3000, 0, 17], seed=11)
    # second call: another shape, reusing the scratch the first call wrote
    _check(dev, B=2, Hq=16, Hkv=8, P=64, lens=[700, 2049], seed=12)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda:0")
    B, Hq, Hkv, D = 2048, 64, 8, 128
    need = _capi.decode_workspace_bytes(dev, B, Hq, Hkv, D)
    assert need > 8 << 20
    q = torch.zeros(1, Hq, D, dtype=torch.bfloat16, device=dev)
    rc = _capi.lib().helm_paged_decode_attention_noalloc(
        q.data_ptr(), 0, D, q.data_ptr(), 1, q.data_ptr(), 0, 1, q.data_ptr(), None, None, None,
        None, 0, 0, q.data_ptr(), 0, D, None, B, Hq, Hkv, D, 16, _capi.DTYPE_BF16, 1.0, 0.0, 0,
        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 4  # HELM_ERR_WORKSPACE, refused before any launch
