"""Sequence split through the CUDA kernels (GPU).

* one GPU, R emulated ranks: the decode kernel's fp32 partial states over R
  page-aligned token ranges, packed as SeqSplitAttention packs them and merged
  by helm_merge_attention_states, equal the single-pass kernel (O within the
  bf16 tolerance of the attention tests, LSE within 1e-4);
* several GPUs (skipped with fewer than 2): real ranks over NCCL, each holding
  only its own range in its own HBM.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helm_b200 import _capi
from helm_b200.runtime.seq_parallel import SeqSplitAttention, split_ranges

pytestmark = pytest.mark.gpu


def _problem(B, Hq, Hkv, D, P, T, seed=0):
    g = torch.Generator().manual_seed(seed)
    npg = T // P
    slots = B * npg + 5
    perm = torch.randperm(slots, generator=g)
    pt = perm[:B * npg].view(B, npg).to(torch.int32)
    pool = torch.randn(slots, 2, Hkv, P, D, generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16)
    return q, pool, pt


def _local(pt, P, rng):
    """Page table and lengths of one rank's page-aligned token range."""
    a, b = rng
    sub = pt[:, a // P: -(-b // P)].contiguous()
    lens = torch.full((pt.shape[0],), b - a, dtype=torch.int32)
    return sub, lens


@pytest.mark.parametrize("R", [2, 4, 8])
def test_emulated_ranks_merge_to_single_pass(R):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda:0")
    B, Hq, Hkv, D, P, T = 1, 40, 8, 128, 16, 16384   # Qwen3-14B heads, 16k tokens
    q, pool, pt = _problem(B, Hq, Hkv, D, P, T)
    q, pool = q.to(dev), pool.to(dev)
    lse_ref = torch.empty(B, Hq, device=dev)
    ref, _ = _capi.paged_decode_attention(q, pool, pt.to(dev),
                                          torch.full((B,), T, dtype=torch.int32, device=dev),
                                          num_kv_heads=Hkv, page_size=P, scale=D ** -0.5,
                                          lse=lse_ref)
    rows = B * Hq
    parts = torch.empty(R, rows * (D + 1), dtype=torch.float32, device=dev)
    for r, rng in enumerate(split_ranges(T, P, R)):
        sub, lens = _local(pt, P, rng)
        _capi.paged_decode_attention(q, pool, sub.to(dev), lens.to(dev), num_kv_heads=Hkv,
                                     page_size=P, scale=D ** -0.5,
                                     out=parts[r, :rows * D].view(B, Hq, D),
                                     lse=parts[r, rows * D:].view(B, Hq))
    sp = SeqSplitAttention()
    sp.world = R
    out, lse = sp.merge(parts, rows, D, torch.bfloat16)
    torch.cuda.synchronize()
    assert _capi.device_status(dev) == 0
    got, want = out.view(B, Hq, D).float().cpu(), ref.float().cpu()
    assert torch.all((got - want).abs() <= 1e-2 + 1e-2 * want.abs())
    assert torch.allclose(lse.view(B, Hq).cpu(), lse_ref.cpu(), atol=1e-4, rtol=1e-5)


def _nccl_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        B, Hq, Hkv, D, P, T = 1, 40, 8, 128, 16, 16384
        q, pool, pt = _problem(B, Hq, Hkv, D, P, T)
        sub, lens = _local(pt, P, split_ranges(T, P, world)[rank])
        # this rank's pool holds only its own pages
        used = torch.unique(sub.flatten())
        remap = torch.full((pool.shape[0],), -1, dtype=torch.int64)
        remap[used.long()] = torch.arange(used.numel())
        local_pool = pool[used.long()].to(dev)
        local_pt = remap[sub.long()].to(torch.int32).to(dev)
        kw = dict(num_kv_heads=Hkv, page_size=P, scale=D ** -0.5)
        qs = [q] + [torch.randn(q.shape, generator=torch.Generator().manual_seed(50 + i))
                    .to(torch.bfloat16) for i in range(3)]
        nccl = SeqSplitAttention(exchange="nccl")
        p2p = SeqSplitAttention(exchange="p2p")
        res = {}
        for i, qi in enumerate(qs):          # eager: both exchanges, repeated calls
            for name, sp in (("nccl", nccl), ("p2p", p2p)):
                out, lse = sp.decode(qi.to(dev), local_pool, local_pt, lens.to(dev), **kw)
                res[f"{name}_out{i}"], res[f"{name}_lse{i}"] = out.float().cpu(), lse.cpu()
        # the p2p step captured in a CUDA graph and replayed with new queries
        q_static = qs[0].to(dev).clone()
        lens_d = lens.to(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            p2p.decode(q_static, local_pool, local_pt, lens_d, **kw)
            torch.cuda.synchronize(dev)
            dist.barrier()
            with torch.cuda.graph(graph, stream=side):
                g_out, g_lse = p2p.decode(q_static, local_pool, local_pt, lens_d, **kw)
        torch.cuda.current_stream(dev).wait_stream(side)
        for i, qi in enumerate(qs):
            q_static.copy_(qi.to(dev))
            graph.replay()
            res[f"graph_out{i}"], res[f"graph_lse{i}"] = g_out.float().cpu(), g_lse.cpu()
        torch.cuda.synchronize()
        assert _capi.device_status(dev) == 0
        del graph
        p2p.close()
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **{k: v.numpy() for k, v in res.items()})
    finally:
        dist.destroy_process_group()


def test_nccl_ranks_equal_single_gpu(tmp_path):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = min(n, 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_nccl_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    dev = torch.device("cuda:0")
    B, Hq, Hkv, D, P, T = 1, 40, 8, 128, 16, 16384
    q, pool, pt = _problem(B, Hq, Hkv, D, P, T)
    qs = [q] + [torch.randn(q.shape, generator=torch.Generator().manual_seed(50 + i))
                .to(torch.bfloat16) for i in range(3)]
    refs = []
    for qi in qs:
        lse_ref = torch.empty(B, Hq, device=dev)
        ref, _ = _capi.paged_decode_attention(qi.to(dev), pool.to(dev), pt.to(dev),
                                              torch.full((B,), T, dtype=torch.int32, device=dev),
                                              num_kv_heads=Hkv, page_size=P, scale=D ** -0.5,
                                              lse=lse_ref)
        refs.append((ref.float().cpu().numpy(), lse_ref.cpu().numpy()))
    for r in range(world):
        got = np.load(tmp_path / f"rank{r}.npz")
        for i, (want, want_lse) in enumerate(refs):
            for name in ("nccl", "p2p", "graph"):
                o = got[f"{name}_out{i}"]
                assert np.all(np.abs(o - want) <= 1e-2 + 1e-2 * np.abs(want)), (r, i, name)
                np.testing.assert_allclose(got[f"{name}_lse{i}"], want_lse, atol=1e-4, rtol=1e-5)
            # both exchanges merge the same fp32 states with the same formula
            np.testing.assert_array_equal(got[f"p2p_out{i}"], got[f"nccl_out{i}"])
            np.testing.assert_array_equal(got[f"graph_out{i}"], got[f"p2p_out{i}"])
