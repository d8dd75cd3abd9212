"""Host-side check of the model-level sequence split (runtime/seq_decode.py)
on CPU ranks (gloo).  The library's kernels are replaced by plain torch /
oracle restatements of their contracts (test infrastructure only: the GEMV
with fused RMSNorm / SwiGLU / residual, the fused append with its row -1
skip, paged decode attention with fp32 partial O + LSE, and the exchange as
an all-gather plus the oracle's merge), so that what runs is the model's own
orchestration: which rank writes each token, how many of its tokens each
rank attends, and how the partial states are combined.  Two ranks feeding a
prompt token by token must give the logits of one rank holding everything.
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import merge as oracle_merge

ARCH = dict(hidden=64, layers=2, q_heads=4, kv_heads=2, head_dim=16, intermediate=96, vocab=50,
            qk_norm=True, theta=1e4)
CTX, NEW, P = 40, 6, 16


def _rms(x, w, eps):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _rope(x, cos, sin):  # x [N, H, D]; cos/sin [N, D] (rotate-half convention)
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos.float().unsqueeze(1) + rot * sin.float().unsqueeze(1)


def _install_fakes(monkeypatch=None):
    from helm_b200 import _capi
    from helm_b200.runtime import seq_decode

    def decode_gemv(x, w, *, out, norm_w=None, eps=1e-6, w2=None, residual=None, stream=None):
        xx = _rms(x, norm_w, eps) if norm_w is not None else x.float()
        y = xx @ w.float().t()
        if w2 is not None:
            y = torch.nn.functional.silu(y) * (xx @ w2.float().t())
        if residual is not None:
            y = residual.float() + y
        out.copy_(y.to(out.dtype))
        return out

    def kv_append(*, k, v, pool, slot_rows, page_size, q=None, q_out=None, q_norm_w=None,
                  k_norm_w=None, eps=1e-6, cos=None, sin=None, k_out=None, v_out=None,
                  stream=None):
        qq = _rms(q, q_norm_w, eps) if q_norm_w is not None else q.float()
        kk = _rms(k, k_norm_w, eps) if k_norm_w is not None else k.float()
        q_out.copy_(_rope(qq, cos, sin).to(q_out.dtype))
        kk = _rope(kk, cos, sin)
        for t, row in enumerate(slot_rows.tolist()):
            if row < 0:
                continue
            slot, r = divmod(row, page_size)
            pool[slot, 0, :, r] = kk[t].to(pool.dtype)
            pool[slot, 1, :, r] = v[t].to(pool.dtype)

    def paged_decode_attention(q, pool, page_table, kv_lens, *, num_kv_heads, page_size, scale,
                               out=None, lse=None, max_kv_len_hint=0, **kw):
        B, Hq, D = q.shape
        G = Hq // num_kv_heads
        for b in range(B):
            n = int(kv_lens[b])
            if n == 0:
                out[b].zero_()
                if lse is not None:
                    lse[b].fill_(-float("inf"))
                continue
            idx = torch.arange(n)
            slots = page_table[b, idx // page_size].long()
            K = pool[slots, 0, :, idx % page_size].float()        # [n, Hkv, D]
            V = pool[slots, 1, :, idx % page_size].float()
            for h in range(Hq):
                s = K[:, h // G] @ q[b, h].float() * scale
                m = s.max()
                p = torch.exp(s - m)
                out[b, h] = ((p @ V[:, h // G]) / p.sum()).to(out.dtype)
                if lse is not None:
                    lse[b, h] = m + torch.log(p.sum())
        return out, lse

    class FakeExchange:
        def __init__(self, rows, head_dim, device, group=None):
            self.world = dist.get_world_size(group) if dist.is_initialized() else 1
            self.group = group

        def merge(self, o_part, lse_part, out, lse_out=None, stream=None):
            packed = torch.cat([o_part.reshape(-1), lse_part.reshape(-1)]).float()
            parts = [torch.empty_like(packed) for _ in range(self.world)]
            dist.all_gather(parts, packed, group=self.group)
            rows, D = o_part.shape
            o = np.stack([p[:rows * D].view(rows, D).numpy() for p in parts])
            l = np.stack([p[rows * D:].numpy() for p in parts])
            mo, _ = oracle_merge.merge_states(o, l)
            out.copy_(torch.from_numpy(np.asarray(mo, np.float32)).view_as(out).to(out.dtype))

        def close(self):
            pass

    _capi.decode_gemv = decode_gemv
    _capi.kv_append = kv_append
    _capi.paged_decode_attention = paged_decode_attention
    _capi.gemv_max_batch = lambda k, elem=2: 16
    seq_decode.PeerExchange = FakeExchange


def _run(rank, world, out_dir):
    _install_fakes()
    from helm_b200.runtime.seq_decode import SeqSplitDecodeModel
    from helm_b200.runtime.tp_decode import synthetic_shard
    w = synthetic_shard(ARCH, 0, 1, torch.float32, torch.device("cpu"), std=0.2)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, ARCH["vocab"], (2, CTX), generator=g)
    forced = torch.randint(0, ARCH["vocab"], (2, NEW), generator=g)
    sd = SeqSplitDecodeModel(w, batch=2, context_len=CTX, max_new=NEW + 2, page_size=P)
    sd.start(prompt[:, :1])
    logits = []
    for t in range(CTX):
        sd.ids.copy_(prompt[:, t:t + 1])
        sd.step()
    logits.append(sd.full_logits().clone())
    for s in range(NEW - 1):
        sd.ids.copy_(forced[:, s:s + 1])
        sd.step()
        logits.append(sd.full_logits().clone())
    torch.save(torch.stack(logits, 1), os.path.join(out_dir, f"logits_w{world}_r{rank}.pt"))


def _worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        _run(rank, world, out_dir)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_cpu_ranks_equal_one_rank(tmp_path):
    mp.spawn(_worker, args=(1, _free_port(), str(tmp_path)), nprocs=1, join=True)
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    one = torch.load(tmp_path / "logits_w1_r0.pt")
    a = torch.load(tmp_path / "logits_w2_r0.pt")
    b = torch.load(tmp_path / "logits_w2_r1.pt")
    assert torch.equal(a, b)                          # every rank carries the same state
    torch.testing.assert_close(a, one, rtol=1e-4, atol=1e-4)
    assert one.abs().max() > 0.1                      # the check is not vacuous
