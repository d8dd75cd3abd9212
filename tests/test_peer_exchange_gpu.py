"""Peer-memory exchange + merge of sequence-split states on one GPU (GPU).

With one rank the kernel pushes to its own buffer, raises its own flags and
merges one state: the output is the input state (rounded to the output dtype)
on every call, so the per-CTA epochs and parity slots advance correctly.

Timeout: a second local buffer stands in for a rank that never arrives (no
one raises its flags).  The single launch must give up after its limit, set
HELM_DEV_TIMEOUT in the device status word and leave the context usable.
Several ranks over NVLink are covered in test_seq_parallel_gpu.py.
"""
import pytest
import torch

from helm_b200 import _capi

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


@pytest.mark.parametrize("rows,D,dtype", [(40, 128, torch.bfloat16), (640, 128, torch.float16),
                                          (3, 64, torch.float32)])
def test_single_rank_is_identity_over_calls(dev, rows, D, dtype):
    n = _capi.peer_exchange_bytes(rows, D, 1)
    buf = _capi.ipc_alloc(n, dev)
    try:
        for it in range(5):
            g = torch.Generator(device=dev).manual_seed(it)
            o = torch.randn(rows, D, device=dev, generator=g)
            lse = torch.randn(rows, device=dev, generator=g)
            lse[0] = float("-inf")            # an empty range: zero output, -inf LSE
            out = torch.empty(rows, D, dtype=dtype, device=dev)
            lse_out = torch.empty(rows, device=dev)
            _capi.seq_exchange_merge([buf], 0, o, lse, out, lse_out)
            torch.cuda.synchronize(dev)
            assert _capi.device_status(dev) == 0
            want = o.clone()
            want[0] = 0
            assert torch.equal(out, want.to(dtype))
            assert torch.equal(lse_out[1:], lse[1:]) and lse_out[0] == float("-inf")
    finally:
        _capi.ipc_free(buf, dev)


def test_missing_rank_times_out_with_status(dev):
    rows, D = 8, 128
    n = _capi.peer_exchange_bytes(rows, D, 2)
    bufs = [_capi.ipc_alloc(n, dev), _capi.ipc_alloc(n, dev)]
    try:
        o = torch.randn(rows, D, device=dev)
        lse = torch.randn(rows, device=dev)
        out = torch.empty(rows, D, dtype=torch.bfloat16, device=dev)
        _capi.seq_exchange_merge(bufs, 0, o, lse, out, timeout_s=0.2)
        torch.cuda.synchronize(dev)
        assert _capi.device_status(dev, reset=True) & _capi.DEV_TIMEOUT
        assert _capi.device_status(dev) == 0
        assert float(torch.ones(4, device=dev).sum()) == 4.0     # context still usable
    finally:
        for b in bufs:
            _capi.ipc_free(b, dev)
