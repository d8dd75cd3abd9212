"""Tensor-parallel decode (helm_b200.runtime.tp_decode) against HF (GPU).

A tiny random-init Qwen3 (bf16) or Llama (fp16) model is sharded over the
ranks (KV heads, q/k/v and gate/up rows, o_proj and down_proj columns, vocab
of lm_head); the prompt is consumed token by token, then decoding is teacher
forced.  Logits (gathered over the vocab shards) must be at least as accurate
as HF's own low-precision path against an fp32 copy (the bar of the other
model-level tests).  Also: the step replayed as a CUDA graph equals the eager
step bit for bit.  With 2 GPUs the ranks are real processes whose row-parallel
projections all-reduce over NVLink inside helm_decode_gemv_allreduce.
"""
import copy
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helm_b200.runtime.tp_decode import TPDecodeModel, shard_hf_model
from helm_b200.synthetic import build_model, make_config
from test_model_gpu import _assert_logits_close, _hf_incremental

pytestmark = pytest.mark.gpu
S, N_STEPS = 40, 12


def _tiny(family, dtype, dev):
    cfg = make_config("tiny", family=family, layers=3, hidden=512, q_heads=8, kv_heads=4,
                      head_dim=64, intermediate=1024, vocab=512,
                      theta=1e6 if family == "qwen3" else 1e4)
    return build_model(cfg, seed=0, std=0.05, dtype=dtype, device=dev)


def _tokens():
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, 512, (1, S), generator=g), torch.randint(0, 512, (1, N_STEPS), generator=g)


@torch.no_grad()
def _tp_logits(model, prompt, forced, rank, world, group=None, graph=False):
    w = shard_hf_model(model, rank, world)
    tp = TPDecodeModel(w, batch=1, max_len=S + N_STEPS + 8, page_size=16, group=group)
    try:
        out = []
        for t in range(S):                       # the prompt, one token per step
            tp.ids.copy_(prompt[:, t:t + 1])
            tp.step()
        out.append(tp.full_logits())
        if graph:
            tp.capture()
        for s in range(N_STEPS - 1):
            tp.ids.copy_(forced[:, s:s + 1])
            if graph:
                tp.replay()
            else:
                tp.step()
            out.append(tp.full_logits())
        torch.cuda.synchronize()
        from helm_b200 import _capi
        assert _capi.device_status(tp.dev) == 0
        return torch.stack(out, 1)
    finally:
        tp.close()


@pytest.mark.parametrize("family,dtype", [("qwen3", torch.bfloat16), ("llama", torch.float16)])
def test_single_rank_matches_hf(family, dtype):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    dev = torch.device("cuda:0")
    model = _tiny(family, dtype, dev)
    prompt, forced = (t.to(dev) for t in _tokens())
    mine = _tp_logits(model, prompt, forced, 0, 1)
    ref = _hf_incremental(model, prompt, forced, N_STEPS)
    ref32 = _hf_incremental(copy.deepcopy(model).float(), prompt, forced, N_STEPS)
    _assert_logits_close(mine, ref, ref32, dtype)
    assert torch.equal(_tp_logits(model, prompt, forced, 0, 1, graph=True), mine)


def _worker(rank, world, port, out_dir, family):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    try:
        dtype = torch.bfloat16 if family == "qwen3" else torch.float16
        model = _tiny(family, dtype, dev)
        prompt, forced = (t.to(dev) for t in _tokens())
        eager = _tp_logits(model, prompt, forced, rank, world)
        graph = _tp_logits(model, prompt, forced, rank, world, graph=True)
        if rank == 0:
            np.save(os.path.join(out_dir, "eager.npy"), eager.cpu().numpy())
            np.save(os.path.join(out_dir, "graph.npy"), graph.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("family", ["qwen3", "llama"])
def test_two_ranks_match_hf(tmp_path, family):
    n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path), family), nprocs=2, join=True)
    dev = torch.device("cuda:0")
    dtype = torch.bfloat16 if family == "qwen3" else torch.float16
    model = _tiny(family, dtype, dev)
    prompt, forced = (t.to(dev) for t in _tokens())
    ref = _hf_incremental(model, prompt, forced, N_STEPS)
    ref32 = _hf_incremental(copy.deepcopy(model).float(), prompt, forced, N_STEPS)
    eager = torch.from_numpy(np.load(tmp_path / "eager.npy")).to(dev)
    graph = torch.from_numpy(np.load(tmp_path / "graph.npy")).to(dev)
    _assert_logits_close(eager, ref, ref32, dtype)
    assert torch.equal(graph, eager)
