"""Tensor-parallel decode of a Qwen3 / Llama-architecture model across the GPUs
of one node (one process per GPU).

HELM runs on one GPU (its planner declares multi-GPU but does not implement
it, compiler/optimization/strategy_selector.py:86-90).  Here rank r of N holds:

  * KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads: its own page pool,
    fused append and paged decode attention for those heads only (KV-head
    sharding: attention needs no exchange);
  * column slices of q/k/v and gate/up (their output rows) and row slices of
    o_proj and down_proj (their input columns); the row-parallel projections
    run as helm_decode_gemv_allreduce, which sums the ranks' partials over
    NVLink and adds the residual in the same kernel;
  * a vocab slice of lm_head; greedy argmax = local argmax + one all-gather of
    (value, index) pairs over the process group;
  * replicated embeddings and norms.

Every rank therefore reads 1/N of the layer weights and of the K/V cache per
step.  The decode step is captured as one CUDA graph; lengths, rows, positions
and the next token advance on the device, so a step needs no host work.  The
K/V layout is static (dense page tables, all pages resident): the model-level
multi-GPU form of the decode hot path, without the single-GPU offload policy.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch
import torch.distributed as dist

from .. import _capi


@dataclass
class TPLayer:
    ln1: torch.Tensor
    eps1: float
    wqkv: torch.Tensor          # [(hq + 2 hkv) * D, H]  this rank's heads
    q_norm: Optional[torch.Tensor]
    k_norm: Optional[torch.Tensor]
    qk_eps: float
    wo: torch.Tensor            # [H, hq * D]            input columns of this rank's heads
    ln2: torch.Tensor
    eps2: float
    wg: torch.Tensor            # [I / N, H]
    wu: torch.Tensor            # [I / N, H]
    wd: torch.Tensor            # [H, I / N]


@dataclass
class TPWeights:
    """One rank's shard of a decoder-only model."""
    embed: torch.Tensor         # [V, H] replicated
    final_norm: torch.Tensor
    final_eps: float
    lm_head: torch.Tensor       # [V / N, H] rows [r V/N, (r+1) V/N)
    vocab: int
    hq: int                     # query heads on this rank
    hkv: int                    # KV heads on this rank
    head_dim: int
    theta: float
    layers: List[TPLayer] = field(default_factory=list)


def _split(n: int, world: int, rank: int):
    if n % world:
        raise ValueError(f"{n} does not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


@torch.no_grad()
def shard_hf_model(model, rank: int, world: int) -> TPWeights:
    """This rank's shard of an HF Qwen3 / Llama causal LM (copies the slices)."""
    cfg = model.config
    inner = model.model
    Hq, Hkv = cfg.num_attention_heads, getattr(cfg, "num_key_value_heads", cfg.num_attention_heads)
    D = getattr(cfg, "head_dim", None) or cfg.hidden_size // Hq
    G = Hq // Hkv
    k0, k1 = _split(Hkv, world, rank)
    q0, q1 = k0 * G, k1 * G
    v0, v1 = _split(cfg.vocab_size, world, rank)
    layers = []
    for layer in inner.layers:
        a, m = layer.self_attn, layer.mlp
        wq = a.q_proj.weight[q0 * D:q1 * D]
        wk = a.k_proj.weight[k0 * D:k1 * D]
        wv = a.v_proj.weight[k0 * D:k1 * D]
        i0, i1 = _split(m.gate_proj.weight.shape[0], world, rank)
        qn, kn = getattr(a, "q_norm", None), getattr(a, "k_norm", None)
        layers.append(TPLayer(
            ln1=layer.input_layernorm.weight.clone(),
            eps1=float(layer.input_layernorm.variance_epsilon),
            wqkv=torch.cat([wq, wk, wv]).contiguous(),
            q_norm=None if qn is None else qn.weight.clone(),
            k_norm=None if kn is None else kn.weight.clone(),
            qk_eps=float(qn.variance_epsilon) if qn is not None else 1e-6,
            wo=a.o_proj.weight[:, q0 * D:q1 * D].contiguous(),
            ln2=layer.post_attention_layernorm.weight.clone(),
            eps2=float(layer.post_attention_layernorm.variance_epsilon),
            wg=m.gate_proj.weight[i0:i1].contiguous(), wu=m.up_proj.weight[i0:i1].contiguous(),
            wd=m.down_proj.weight[:, i0:i1].contiguous()))
    theta = float(getattr(cfg, "rope_theta", None) or cfg.rope_parameters["rope_theta"])
    return TPWeights(embed=inner.embed_tokens.weight.clone(), final_norm=inner.norm.weight.clone(),
                     final_eps=float(inner.norm.variance_epsilon),
                     lm_head=model.lm_head.weight[v0:v1].contiguous(), vocab=cfg.vocab_size,
                     hq=q1 - q0, hkv=k1 - k0, head_dim=D, theta=theta, layers=layers)


@torch.no_grad()
def synthetic_shard(arch: dict, rank: int, world: int, dtype, device, seed: int = 0,
                    std: float = 0.02) -> TPWeights:
    """This rank's shard of a random-init model of the given shape, drawn
    directly per shard (N(0, std), norms 1): the whole model never exists."""
    H, L, Hq, Hkv, D = arch["hidden"], arch["layers"], arch["q_heads"], arch["kv_heads"], arch["head_dim"]
    I, V = arch["intermediate"], arch["vocab"]
    G = Hq // Hkv
    k0, k1 = _split(Hkv, world, rank)
    hq, hkv = (k1 - k0) * G, k1 - k0
    i0, i1 = _split(I, world, rank)
    v0, v1 = _split(V, world, rank)
    gen = torch.Generator(device=device).manual_seed(seed * 1000 + rank)

    def rnd(*shape):
        return (torch.randn(*shape, generator=gen, device=device) * std).to(dtype)

    ones = lambda n: torch.ones(n, dtype=dtype, device=device)  # noqa: E731
    layers = []
    for _ in range(L):
        layers.append(TPLayer(
            ln1=ones(H), eps1=1e-6, wqkv=rnd((hq + 2 * hkv) * D, H),
            q_norm=ones(D) if arch["qk_norm"] else None, k_norm=ones(D) if arch["qk_norm"] else None,
            qk_eps=1e-6, wo=rnd(H, hq * D), ln2=ones(H), eps2=1e-6,
            wg=rnd(i1 - i0, H), wu=rnd(i1 - i0, H), wd=rnd(H, i1 - i0)))
    embed = (torch.randn(V, H, generator=torch.Generator(device=device).manual_seed(seed),
                         device=device) * std).to(dtype)
    return TPWeights(embed=embed, final_norm=ones(H), final_eps=1e-6, lm_head=rnd(v1 - v0, H),
                     vocab=V, hq=hq, hkv=hkv, head_dim=D, theta=arch["theta"], layers=layers)


class _PeerBuffers:
    """One zeroed exchange buffer per rank, mapped into every rank (CUDA IPC)."""

    def __init__(self, nbytes: int, device, group, rank: int, world: int):
        self.device, self.group, self.rank, self.world = device, group, rank, world
        self.local = _capi.ipc_alloc(nbytes, device)
        handles = [None] * world
        if world > 1:
            dist.all_gather_object(handles, _capi.ipc_get_handle(self.local, device), group=group)
        self.ptrs = [self.local if r == rank else _capi.ipc_open(handles[r], device)
                     for r in range(world)]
        if world > 1:
            dist.barrier(group=group)

    def close(self):
        if self.ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                _capi.ipc_close(p, self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        _capi.ipc_free(self.local, self.device)
        self.ptrs = None


class TPDecodeModel:
    """Greedy decode of B sequences with this rank's TPWeights.

    fill_kv() (synthetic context) or decode steps fed with prompt tokens
    (step(..., forced)) build the cache; step() advances every sequence by one
    token; capture()/replay() run the step as a CUDA graph.
    """

    def __init__(self, w: TPWeights, batch: int, max_len: int, page_size: int = 16,
                 group: Optional[dist.ProcessGroup] = None):
        self.w = w
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dev = w.embed.device
        self.dtype = w.embed.dtype
        self.embed_elem = w.embed.element_size()
        self.B, self.P, self.D = batch, page_size, w.head_dim
        self.L = len(w.layers)
        self.H = w.embed.shape[1]
        self.maxp = -(-max_len // page_size)
        self.max_len = max_len
        dev, L, B = self.dev, self.L, batch
        # pool[slot][kv][head][token][dim]; layer l, sequence b, page i -> slot (l*B + b)*maxp + i
        self.pool = torch.empty(L * B * self.maxp, 2, w.hkv, page_size, w.head_dim, dtype=self.dtype,
                                device=dev)
        base = torch.arange(L * B, dtype=torch.int32, device=dev).view(L, B, 1) * self.maxp
        self.tables = (base + torch.arange(self.maxp, dtype=torch.int32, device=dev)).contiguous()
        self.lens = torch.zeros(B, dtype=torch.int32, device=dev)      # tokens cached
        self.ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.h = torch.empty(B, self.H, dtype=self.dtype, device=dev)
        n_qkv = w.layers[0].wqkv.shape[0]
        self.qkv = torch.empty(B, n_qkv, dtype=self.dtype, device=dev)
        self.q_out = torch.empty(B, w.hq, w.head_dim, dtype=self.dtype, device=dev)
        self.attn = torch.empty(B, w.hq, w.head_dim, dtype=self.dtype, device=dev)
        self.act = torch.empty(B, w.layers[0].wg.shape[0], dtype=self.dtype, device=dev)
        self.logits = torch.empty(B, w.lm_head.shape[0], dtype=self.dtype, device=dev)
        self.pick = torch.empty(self.world, B, 2, dtype=torch.float32, device=dev)
        self.inv_freq = 1.0 / (w.theta ** (torch.arange(0, w.head_dim, 2, dtype=torch.float32,
                                                        device=dev) / w.head_dim))
        self.peers = None
        if self.world > 1:
            nbytes = _capi.decode_gemv_allreduce_bytes(self.H, B, self.world)
            self.peers = _PeerBuffers(nbytes, dev, group, self.rank, self.world)
        self.graph = None

    # ------------------------------------------------------------------ state --
    @torch.no_grad()
    def fill_kv(self, length: int, seed: int = 0) -> None:
        """Synthetic context of `length` tokens per sequence (N(0,1) K/V)."""
        if length >= self.max_len:
            raise ValueError("context does not fit max_len")
        g = torch.Generator(device=self.dev).manual_seed(seed * 7919 + self.rank)
        self.pool.normal_(generator=g)
        self.lens.fill_(length)

    def close(self) -> None:
        self.graph = None
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    # ------------------------------------------------------------------- step --
    def _slices(self, k: int):
        """Batch slices whose inputs helm_decode_gemv can stage (batch x k)."""
        n = _capi.gemv_max_batch(k, self.embed_elem)
        return [(b, min(self.B, b + n)) for b in range(0, self.B, n)]

    def _gemv(self, x, w, out, norm_w=None, eps=1e-6, w2=None):
        for b0, b1 in self._slices(x.shape[1]):
            _capi.decode_gemv(x[b0:b1], w, out=out[b0:b1], norm_w=norm_w, eps=eps, w2=w2)

    def _row_proj(self, x, w, out):
        """out = out + (row-parallel) W x, all-reduced over the ranks."""
        for b0, b1 in self._slices(x.shape[1]):
            if self.peers is None:
                _capi.decode_gemv(x[b0:b1], w, out=out[b0:b1], residual=out[b0:b1])
            else:
                _capi.decode_gemv_allreduce(self.peers.ptrs, self.rank, x[b0:b1], w,
                                            out=out[b0:b1], residual=out[b0:b1])

    @torch.no_grad()
    def step(self, forced: Optional[torch.Tensor] = None) -> None:
        """One decode step: the token in self.ids is appended at position
        lens and attended; self.ids becomes the greedy next token (or, when
        `forced` [B, 1] is given, that token; the argmax stays in self.next)."""
        w, B, D, P = self.w, self.B, self.D, self.P
        h = self.h
        torch.index_select(w.embed, 0, self.ids.view(-1), out=h)
        pos = self.lens.to(torch.float32).view(B, 1)
        freqs = pos * self.inv_freq.view(1, -1)
        emb = torch.cat([freqs, freqs], dim=-1)
        cos, sin = emb.cos().to(self.dtype), emb.sin().to(self.dtype)
        page = (self.lens // P).long()
        r_in = (self.lens % P).long()
        slot = self.tables[:, torch.arange(B, device=self.dev), page].long()      # [L, B]
        rows = (slot * P + r_in.view(1, B)).contiguous()
        lens1 = self.lens + 1
        scale = D ** -0.5
        for l, lw in enumerate(w.layers):
            self._gemv(h, lw.wqkv, self.qkv, norm_w=lw.ln1, eps=lw.eps1)
            nq, nk = w.hq * D, w.hkv * D
            q = self.qkv[:, :nq].view(B, w.hq, D)
            k = self.qkv[:, nq:nq + nk].view(B, w.hkv, D)
            v = self.qkv[:, nq + nk:].view(B, w.hkv, D)
            _capi.kv_append(q=q, k=k, v=v, q_out=self.q_out, q_norm_w=lw.q_norm,
                            k_norm_w=lw.k_norm, eps=lw.qk_eps, cos=cos, sin=sin, pool=self.pool,
                            slot_rows=rows[l], page_size=P)
            _capi.paged_decode_attention(self.q_out, self.pool, self.tables[l], lens1,
                                         num_kv_heads=w.hkv, page_size=P, scale=scale,
                                         out=self.attn, max_kv_len_hint=self.max_len)
            self._row_proj(self.attn.view(B, w.hq * D), lw.wo, h)
            self._gemv(h, lw.wg, self.act, norm_w=lw.ln2, eps=lw.eps2, w2=lw.wu)
            self._row_proj(self.act, lw.wd, h)
        self._gemv(h, w.lm_head, self.logits, norm_w=w.final_norm, eps=w.final_eps)
        # greedy pick over the vocab shards: (max value, global index) per rank
        val, idx = self.logits.float().max(dim=-1)
        local = torch.stack([val, (idx + self.rank * w.lm_head.shape[0]).float()], dim=-1)
        if self.world > 1:
            dist.all_gather_into_tensor(self.pick.view(-1), local.view(-1).contiguous(),
                                        group=self.group)
            best = self.pick[:, :, 0].argmax(dim=0)          # first rank wins ties
            nxt = self.pick[best, torch.arange(B, device=self.dev), 1]
        else:
            nxt = local[:, 1]
        self.next = nxt.long().view(B, 1)
        self.lens.copy_(lens1)
        self.ids.copy_(self.next if forced is None else forced)

    def capture(self) -> None:
        """Captures step() (argmax feeding the next step) as a CUDA graph."""
        self.graph = None
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        saved = (self.lens.clone(), self.ids.clone())
        with torch.cuda.stream(side), _capi.decode_overlap():
            with torch.cuda.graph(g, stream=side):
                self.step()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        self.lens.copy_(saved[0])
        self.ids.copy_(saved[1])
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def full_logits(self) -> torch.Tensor:
        """Logits of the last step over the whole vocabulary [B, V] (fp32)."""
        loc = self.logits.float()
        if self.world == 1:
            return loc
        out = torch.empty((self.world,) + tuple(loc.shape), dtype=loc.dtype, device=self.dev)
        dist.all_gather_into_tensor(out, loc.contiguous(), group=self.group)
        return out.permute(1, 0, 2).reshape(self.B, -1)
