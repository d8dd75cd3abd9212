"""helm_decode_gemv_allreduce on one GPU (world 1: the exchange buffer is this
rank's own), called with the batch slices and shapes a tensor-parallel decode
step makes, one after another on one stream.

With one rank the all-reduce sum is this rank's partial, so every call must be
bit-identical to helm_decode_gemv with the same residual.  The exchange words
carry the call's epoch: the header's epoch must count the calls, and calls
whose grids or batch slices differ (16 rows, then 8, then 1 ...) must never
read a word left by an earlier call (a stale word would give a wrong sum, not
a timeout).
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def test_allreduce_gemv_one_rank_matches_plain_gemv_over_mixed_calls():
    dev = _cuda()
    from helm_b200 import _capi
    g = torch.Generator().manual_seed(3)
    N = 1536
    nbytes = _capi.decode_gemv_allreduce_bytes(N, 16, 1)
    buf = _capi.ipc_alloc(nbytes, dev)
    try:
        calls = 0
        # (batch, K): o_proj-like and down_proj-like widths, full and sliced batches
        for rep in range(3):
            for batch, K in ((16, 1024), (8, 2048), (8, 2048), (1, 1024), (3, 4096), (16, 512),
                             (2, 1024)):
                x = torch.randn(batch, K, generator=g).to(torch.bfloat16).to(dev)
                w = (torch.randn(N, K, generator=g) * 0.03).to(torch.bfloat16).to(dev)
                res = torch.randn(batch, N, generator=g).to(torch.bfloat16).to(dev)
                y_ar = res.clone()
                _capi.decode_gemv_allreduce([buf], 0, x, w, out=y_ar, residual=y_ar)
                y = res.clone()
                _capi.decode_gemv(x, w, out=y, residual=y)
                calls += 1
                torch.cuda.synchronize(dev)
                assert torch.equal(y_ar, y), (rep, batch, K)
        hdr_host = _read_words(buf, dev, 2)
        assert hdr_host[0] == calls and hdr_host[1] == 0
        assert _capi.device_status(dev) == 0
    finally:
        _capi.ipc_free(buf, dev)


def _read_words(ptr: int, dev, n: int):
    """n uint32 words at device address ptr (one helm_copy_pages copy of
    4 n bytes into a tensor)."""
    from helm_b200 import _capi
    out = torch.empty(n, dtype=torch.int32, device=dev)
    zero = (ctypes.c_int64 * 1)(0)
    with torch.cuda.device(dev):
        rc = _capi.lib().helm_copy_pages(out.data_ptr(), ptr, 4 * n, zero, zero, 1,
                                         torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0
    torch.cuda.synchronize(dev)
    return out.cpu().tolist()
