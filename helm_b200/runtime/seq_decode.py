"""Sequence-split decode of a Qwen3 / Llama-architecture model across the GPUs
of one node (one process per GPU): the multi-GPU form of HELM's long-context
decode that BASELINE configs[3] names (K/V of a 131072-token context split by
token range, partial attention states merged over NVLink).

HELM itself runs on one GPU (compiler/optimization/strategy_selector.py:86-90).
Here every rank holds the whole model (replicated weights) and, for every
layer, the pages of one contiguous, page-aligned token range of the context
(seq_parallel.split_ranges); a token's K/V row goes to the rank whose range
holds its position, and every position past the context to the last rank.
Per layer:

  helm_decode_gemv        input RMSNorm + q/k/v (whole model, every rank)
  helm_kv_append          QK-RMSNorm + RoPE; the K/V row is written only by
                          its owner (the others pass row -1, a skip)
  paged decode attention  over this rank's range: fp32 partial O + LSE
  helm_seq_exchange_merge partial states pushed to every rank over NVLink and
                          merged in rank order (the same result everywhere)
  helm_decode_gemv x3     o_proj + residual, RMSNorm + gate/up + SwiGLU,
                          down_proj + residual

and the final norm + lm_head + argmax, computed identically on every rank, so
there is no other collective.  Compared with tensor parallelism
(tp_decode.py) every rank reads all the weights per step; the K/V bytes are
what the split divides.  K/V pages are static (all resident).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from .. import _capi
from .seq_parallel import PeerExchange, split_ranges
from .tp_decode import TPWeights


def token_rows(pos: torch.Tensor, rng, tail: bool, cap: int, tables: torch.Tensor, P: int):
    """This rank's share of the tokens at positions pos [B]: the pool row of
    each layer's K/V write, rows [L, B] (-1 where another rank owns the
    position), and how many of this rank's tokens each query attends,
    lens [B] int32.  rng = (a, b) is the rank's token range; the last rank
    (tail) also owns every position past it, up to cap tokens."""
    a, b = rng
    li = pos.long() - a
    if tail:
        own = li >= 0
        lens = (li + 1).clamp(min=0)
    else:
        own = (li >= 0) & (li < b - a)
        lens = (li + 1).clamp(min=0, max=b - a)
    lic = li.clamp(min=0, max=cap - 1)
    idx = torch.arange(pos.shape[0], device=pos.device)
    slot = tables[:, idx, lic // P].long()                                   # [L, B]
    rows = torch.where(own.view(1, -1), slot * P + (lic % P).view(1, -1),
                       torch.full_like(slot, -1)).contiguous()
    return rows, lens.to(torch.int32)


class SeqSplitDecodeModel:
    """Greedy decode of B sequences whose `context_len`-token contexts are
    split by token range over the ranks of `group`.

    `w` must be the whole model on every rank (synthetic_shard(arch, 0, 1, ...)
    with the same seed everywhere, or shard_hf_model(model, 0, 1)).  fill_kv()
    fills the context synthetically; step() advances every sequence by one
    token; capture() / replay() run the step as a CUDA graph.
    """

    def __init__(self, w: TPWeights, batch: int, context_len: int, max_new: int,
                 page_size: int = 16, group: Optional[dist.ProcessGroup] = None):
        if w.lm_head.shape[0] != w.vocab:
            raise ValueError("sequence-split decode needs the whole model on every rank")
        self.w = w
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.dev = w.embed.device
        self.dtype = w.embed.dtype
        self.B, self.P, self.D = batch, page_size, w.head_dim
        self.L = len(w.layers)
        self.H = w.embed.shape[1]
        self.context_len = context_len
        self.range = split_ranges(context_len, page_size, self.world)[self.rank]
        self.tail = self.rank == self.world - 1
        own = self.range[1] - self.range[0]
        self.cap = own + (max_new if self.tail else 0)     # tokens this rank may hold
        self.maxp = max(1, -(-self.cap // page_size))
        dev, L, B = self.dev, self.L, batch
        # pool[slot][kv][head][token][dim]; layer l, sequence b, page i -> slot (l*B + b)*maxp + i
        self.pool = torch.empty(L * B * self.maxp, 2, w.hkv, page_size, w.head_dim,
                                dtype=self.dtype, device=dev)
        base = torch.arange(L * B, dtype=torch.int32, device=dev).view(L, B, 1) * self.maxp
        self.tables = (base + torch.arange(self.maxp, dtype=torch.int32, device=dev)).contiguous()
        # global position of the token in self.ids: context_len after fill_kv(), 0 after
        # start() for a context built by feeding its tokens
        self.pos = torch.full((B,), context_len, dtype=torch.int32, device=dev)
        self.ids = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.next = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.h = torch.empty(B, self.H, dtype=self.dtype, device=dev)
        self.qkv = torch.empty(B, w.layers[0].wqkv.shape[0], dtype=self.dtype, device=dev)
        self.q_out = torch.empty(B, w.hq, w.head_dim, dtype=self.dtype, device=dev)
        self.o_part = torch.empty(B, w.hq, w.head_dim, dtype=torch.float32, device=dev)
        self.lse_part = torch.empty(B, w.hq, dtype=torch.float32, device=dev)
        self.attn = torch.empty(B, w.hq, w.head_dim, dtype=self.dtype, device=dev)
        self.act = torch.empty(B, w.layers[0].wg.shape[0], dtype=self.dtype, device=dev)
        self.logits = torch.empty(B, w.vocab, dtype=self.dtype, device=dev)
        self.inv_freq = 1.0 / (w.theta ** (torch.arange(0, w.head_dim, 2, dtype=torch.float32,
                                                        device=dev) / w.head_dim))
        self.exchange = (PeerExchange(B * w.hq, w.head_dim, dev, group)
                         if self.world > 1 else None)
        self.graph = None

    # ------------------------------------------------------------------ state --
    @torch.no_grad()
    def fill_kv(self, length: Optional[int] = None, seed: int = 0) -> None:
        """Synthetic context (N(0,1) K/V) over this rank's token range."""
        if length is not None and length != self.context_len:
            raise ValueError("the context length is fixed when the ranges are built")
        g = torch.Generator(device=self.dev).manual_seed(seed * 7919 + self.rank)
        self.pool.normal_(generator=g)
        self.pos.fill_(self.context_len)

    def start(self, ids: torch.Tensor) -> None:
        """An empty cache whose first token is ids [B, 1] at position 0; feed
        the rest of the context with step(forced=next prompt token)."""
        self.pos.zero_()
        self.ids.copy_(ids)

    def close(self) -> None:
        self.graph = None
        if self.exchange is not None:
            self.exchange.close()
            self.exchange = None

    # ------------------------------------------------------------------- step --
    def _gemv(self, x, w, out, norm_w=None, eps=1e-6, w2=None, residual=None):
        """helm_decode_gemv over batch slices whose inputs fit its staging."""
        n = _capi.gemv_max_batch(x.shape[1], x.element_size())
        for b0 in range(0, self.B, n):
            b1 = min(self.B, b0 + n)
            _capi.decode_gemv(x[b0:b1], w, out=out[b0:b1], norm_w=norm_w, eps=eps, w2=w2,
                              residual=None if residual is None else residual[b0:b1])

    @torch.no_grad()
    def step(self, forced: Optional[torch.Tensor] = None) -> None:
        """One decode step: the token in self.ids (position self.pos) is
        appended on the rank whose range holds that position (the last rank
        past the context) and attended over every rank's range; self.ids
        becomes the greedy next token (or `forced` [B, 1]; the argmax stays in
        self.next)."""
        w, B, D, P = self.w, self.B, self.D, self.P
        h = self.h
        torch.index_select(w.embed, 0, self.ids.view(-1), out=h)
        freqs = self.pos.to(torch.float32).view(B, 1) * self.inv_freq.view(1, -1)
        emb = torch.cat([freqs, freqs], dim=-1)
        cos, sin = emb.cos().to(self.dtype), emb.sin().to(self.dtype)
        rows, lens_attn = token_rows(self.pos, self.range, self.tail, self.cap,
                                     self.tables, P)
        scale = D ** -0.5
        nq, nk = w.hq * D, w.hkv * D
        for l, lw in enumerate(w.layers):
            self._gemv(h, lw.wqkv, self.qkv, norm_w=lw.ln1, eps=lw.eps1)
            q = self.qkv[:, :nq].view(B, w.hq, D)
            k = self.qkv[:, nq:nq + nk].view(B, w.hkv, D)
            v = self.qkv[:, nq + nk:].view(B, w.hkv, D)
            _capi.kv_append(q=q, k=k, v=v, q_out=self.q_out, q_norm_w=lw.q_norm,
                            k_norm_w=lw.k_norm, eps=lw.qk_eps, cos=cos, sin=sin, pool=self.pool,
                            slot_rows=rows[l], page_size=P)
            if self.exchange is None:
                _capi.paged_decode_attention(self.q_out, self.pool, self.tables[l], lens_attn,
                                             num_kv_heads=w.hkv, page_size=P, scale=scale,
                                             out=self.attn, max_kv_len_hint=self.context_len)
            else:
                _capi.paged_decode_attention(self.q_out, self.pool, self.tables[l], lens_attn,
                                             num_kv_heads=w.hkv, page_size=P, scale=scale,
                                             out=self.o_part, lse=self.lse_part,
                                             max_kv_len_hint=self.maxp * P)
                self.exchange.merge(self.o_part.view(B * w.hq, D), self.lse_part.view(-1),
                                    self.attn.view(B * w.hq, D))
            self._gemv(self.attn.view(B, nq), lw.wo, h, residual=h)
            self._gemv(h, lw.wg, self.act, norm_w=lw.ln2, eps=lw.eps2, w2=lw.wu)
            self._gemv(self.act, lw.wd, h, residual=h)
        self._gemv(h, w.lm_head, self.logits, norm_w=w.final_norm, eps=w.final_eps)
        self.next.copy_(self.logits.float().argmax(dim=-1, keepdim=True))
        self.pos.add_(1)
        self.ids.copy_(self.next if forced is None else forced)

    def capture(self) -> None:
        """Captures step() (argmax feeding the next step) as a CUDA graph."""
        self.graph = None
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        saved = (self.pos.clone(), self.ids.clone())
        with torch.cuda.stream(side), _capi.decode_overlap():
            with torch.cuda.graph(g, stream=side):
                self.step()
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        self.pos.copy_(saved[0])
        self.ids.copy_(saved[1])
        self.graph = g

    def replay(self) -> None:
        self.graph.replay()

    def full_logits(self) -> torch.Tensor:
        """Logits of the last step [B, V] (fp32; the same on every rank)."""
        return self.logits.float()
