"""Tensor-parallel sharding plan on CPU ranks (gloo, no GPU).

Two processes take shard_hf_model shards of the same tiny random-init Qwen3
model (fp32) and run a plain PyTorch restatement of the sharded decoder:
column-parallel q/k/v and gate/up over their heads / rows, attention over
their KV heads only, row-parallel o_proj and down_proj whose partial outputs
are all-reduced (gloo), vocab-parallel lm_head gathered.  The logits of a
short prompt must equal HF's unsharded forward: this pins which heads, rows
and columns each rank owns (the layout TPDecodeModel runs with its kernels).
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helm_b200.runtime.tp_decode import shard_hf_model
from helm_b200.synthetic import build_model, make_config


def _model():
    cfg = make_config("tiny", family="qwen3", layers=2, hidden=128, q_heads=8, kv_heads=4,
                      head_dim=32, intermediate=256, vocab=96, theta=1e6)
    return build_model(cfg, seed=0, std=0.05, dtype=torch.float32, device="cpu")


def _rms(x, w, eps):
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


def _rope(x, pos, theta, D):
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    f = pos.float().view(-1, 1) * inv.view(1, -1)
    emb = torch.cat([f, f], dim=-1)
    cos, sin = emb.cos(), emb.sin()                       # [S, D]
    rot = torch.cat([-x[..., D // 2:], x[..., :D // 2]], dim=-1)
    return x * cos + rot * sin


def _sharded_logits(w, ids, world):
    """Forward of one rank's shard over the whole prompt (causal)."""
    S = ids.shape[0]
    D = w.head_dim
    h = w.embed[ids]                                      # [S, H]
    pos = torch.arange(S)
    causal = torch.full((S, S), float("-inf")).triu(1)
    for L in w.layers:
        x = _rms(h, L.ln1, L.eps1)
        qkv = x @ L.wqkv.t()
        nq, nk = w.hq * D, w.hkv * D
        q = qkv[:, :nq].view(S, w.hq, D)
        k = qkv[:, nq:nq + nk].view(S, w.hkv, D)
        v = qkv[:, nq + nk:].view(S, w.hkv, D)
        q, k = _rms(q, L.q_norm, L.qk_eps), _rms(k, L.k_norm, L.qk_eps)
        q = _rope(q.transpose(0, 1), pos, w.theta, D)     # [hq, S, D]
        k = _rope(k.transpose(0, 1), pos, w.theta, D)
        v = v.transpose(0, 1)
        G = w.hq // w.hkv
        k, v = k.repeat_interleave(G, 0), v.repeat_interleave(G, 0)
        att = torch.softmax(q @ k.transpose(1, 2) * D ** -0.5 + causal, dim=-1) @ v
        part = att.transpose(0, 1).reshape(S, -1) @ L.wo.t()
        dist.all_reduce(part)                             # row-parallel o_proj
        h = h + part
        x = _rms(h, L.ln2, L.eps2)
        act = torch.nn.functional.silu(x @ L.wg.t()) * (x @ L.wu.t())
        part = act @ L.wd.t()
        dist.all_reduce(part)                             # row-parallel down_proj
        h = h + part
    loc = _rms(h, w.final_norm, w.final_eps) @ w.lm_head.t()
    parts = [torch.empty_like(loc) for _ in range(world)]
    dist.all_gather(parts, loc)                           # vocab-parallel lm_head
    return torch.cat(parts, dim=-1)


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _model()
        ids = torch.randint(0, 96, (12,), generator=torch.Generator().manual_seed(3))
        with torch.no_grad():
            logits = _sharded_logits(shard_hf_model(model, rank, world), ids, world)
        np.save(os.path.join(out_dir, f"tp{rank}.npy"), logits.numpy())
    finally:
        dist.destroy_process_group()


def test_two_cpu_ranks_equal_unsharded_model(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    model = _model()
    ids = torch.randint(0, 96, (12,), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        ref = model(input_ids=ids.view(1, -1), use_cache=False).logits[0].numpy()
    for r in range(2):
        np.testing.assert_allclose(np.load(tmp_path / f"tp{r}.npy"), ref, rtol=2e-4, atol=2e-4)


def test_gemv_staging_limit():
    from helm_b200 import _capi
    assert _capi.gemv_max_batch(1024) == 16
    assert _capi.gemv_max_batch(5120) == 16
    assert _capi.gemv_max_batch(6912) == 8
    assert _capi.gemv_max_batch(17408) == 4
