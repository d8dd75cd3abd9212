"""Sequence-split decode (helm_b200.runtime.seq_decode): against HF on 2 GPUs,
and against the tensor-parallel model on one GPU.

A tiny random-init Qwen3 (bf16) or Llama (fp16) model is replicated on both
ranks; the prompt is consumed token by token (each token's K/V row lands on
the rank whose token range holds its position), then decoding is teacher
forced.  Per layer the ranks' partial attention states are merged over NVLink
by helm_seq_exchange_merge.  Logits must meet the bar of the other
model-level tests (at least as accurate as HF's own low-precision path
against an fp32 copy), be the same on both ranks, and the CUDA-graph replay
must equal the eager step bit for bit.
"""
import copy
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helm_b200.runtime.seq_decode import SeqSplitDecodeModel
from helm_b200.runtime.tp_decode import shard_hf_model
from test_model_gpu import _assert_logits_close, _hf_incremental
from test_tp_decode_gpu import N_STEPS, S, _tiny, _tokens

pytestmark = pytest.mark.gpu


@torch.no_grad()
def _seq_logits(model, prompt, forced, group=None, graph=False):
    w = shard_hf_model(model, 0, 1)             # the whole model on every rank
    sd = SeqSplitDecodeModel(w, batch=1, context_len=S, max_new=N_STEPS + 8, page_size=16,
                             group=group)
    try:
        sd.start(prompt[:, :1])
        out = []
        for t in range(S):                       # the prompt, one token per step
            sd.ids.copy_(prompt[:, t:t + 1])
            sd.step()
        out.append(sd.full_logits())
        if graph:
            sd.capture()
        for s in range(N_STEPS - 1):
            sd.ids.copy_(forced[:, s:s + 1])
            if graph:
                sd.replay()
            else:
                sd.step()
            out.append(sd.full_logits())
        torch.cuda.synchronize()
        from helm_b200 import _capi
        assert _capi.device_status(sd.dev) == 0
        return torch.stack(out, 1)
    finally:
        sd.close()


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
        eager = _seq_logits(model, prompt, forced)
        graph = _seq_logits(model, prompt, forced, graph=True)
        np.save(os.path.join(out_dir, f"eager{rank}.npy"), eager.cpu().numpy())
        np.save(os.path.join(out_dir, f"graph{rank}.npy"), graph.cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("family", ["qwen3", "llama"])
def test_two_ranks_sequence_split_match_hf(tmp_path, family):
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
    eager = [torch.from_numpy(np.load(tmp_path / f"eager{r}.npy")).to(dev) for r in range(2)]
    graph = [torch.from_numpy(np.load(tmp_path / f"graph{r}.npy")).to(dev) for r in range(2)]
    _assert_logits_close(eager[0], ref, ref32, dtype)
    assert torch.equal(eager[0], eager[1])       # every rank continues with the same state
    assert torch.equal(graph[0], eager[0]) and torch.equal(graph[1], eager[1])


@pytest.mark.parametrize("family,dtype", [("qwen3", torch.bfloat16), ("llama", torch.float16)])
def test_single_rank_equals_tensor_parallel_single_rank(family, dtype):
    """On one GPU the sequence split issues the same kernels in the same order
    as the tensor-parallel model: logits bit-identical, the prompt fed
    eagerly, the forced steps replayed as a CUDA graph."""
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from helm_b200 import _capi
    from helm_b200.runtime.tp_decode import TPDecodeModel
    dev = torch.device("cuda:0")
    model = _tiny(family, dtype, dev)
    prompt, forced = (t.to(dev) for t in _tokens())
    w = shard_hf_model(model, 0, 1)
    tp = TPDecodeModel(w, batch=1, max_len=S + N_STEPS + 8, page_size=16)
    sd = SeqSplitDecodeModel(w, batch=1, context_len=S, max_new=N_STEPS + 8, page_size=16)
    try:
        sd.start(prompt[:, :1])
        a, b = [], []
        for t in range(S):
            tp.ids.copy_(prompt[:, t:t + 1])
            tp.step()
            sd.ids.copy_(prompt[:, t:t + 1])
            sd.step()
        a.append(tp.full_logits())
        b.append(sd.full_logits())
        sd.capture()
        for s in range(N_STEPS - 1):
            tp.ids.copy_(forced[:, s:s + 1])
            tp.step()
            sd.ids.copy_(forced[:, s:s + 1])
            sd.replay()
            a.append(tp.full_logits())
            b.append(sd.full_logits())
        torch.cuda.synchronize()
        assert _capi.device_status(dev) == 0
        assert torch.equal(torch.stack(a), torch.stack(b))
    finally:
        tp.close()
        sd.close()
