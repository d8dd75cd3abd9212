"""Decode step of a whole causal LM as a short chain of fused kernels.

HELM's GPU stage runs the decoder layers as eager HF modules with the
attention forward patched (helm/runtime/kv_offload.py:349-519, executed from
compiler/executor.py:420); at decode time each layer is then ~25 launches of
small library GEMMs and element-wise ops, and at batch 1 those launches set
the step time.  FusedDecodeStage computes the same step (same weights, same
rounding points as the eager modules) with seven launches per layer:

  helm_decode_gemv   input RMSNorm + concatenated q/k/v projection
  helm_kv_append     QK-RMSNorm + RoPE + K/V rows into the page pool
  paged decode       attention over the layer's pages (+ its merge kernel)
  helm_decode_gemv   o_proj + residual add
  helm_decode_gemv   post-attention RMSNorm + gate/up projection + SiLU * up
  helm_decode_gemv   down_proj + residual add

and one more GEMV for the final norm + lm_head.  It serves Qwen3 (QK-norm)
and Llama-style layers without projection biases; the page-table state comes
from the GraphDecoder step context (rows, lengths, tables, cold-page staging).
"""
from __future__ import annotations

import torch

from .. import _capi


class _LayerWeights:
    __slots__ = ("ln1", "eps1", "wqkv", "nq", "nk", "q_norm", "k_norm", "qk_eps", "wo", "ln2",
                 "eps2", "wg", "wu", "wd")


def _fuse_qkv(attn) -> torch.Tensor:
    """One [Nq + 2 Nk, H] weight for q/k/v; the module parameters become views
    of it (no second copy of the weights)."""
    fused = getattr(attn, "_helm_wqkv", None)
    if fused is not None:
        return fused
    q, k, v = attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight
    w = torch.cat([q.data, k.data, v.data], dim=0).contiguous()
    nq, nk = q.shape[0], k.shape[0]
    attn.q_proj.weight.data = w[:nq]
    attn.k_proj.weight.data = w[nq:nq + nk]
    attn.v_proj.weight.data = w[nq + nk:]
    attn._helm_wqkv = w
    return w


class FusedDecodeStage:
    """Decode step (q_len = 1) of an HF Qwen3 / Llama causal LM on one GPU."""

    def __init__(self, model, max_batch: int):
        cfg = model.config
        inner = model.model
        self.model = model
        self.H = cfg.hidden_size
        self.Hq = cfg.num_attention_heads
        self.Hkv = getattr(cfg, "num_key_value_heads", self.Hq)
        self.D = getattr(cfg, "head_dim", None) or self.H // self.Hq
        self.dtype = next(model.parameters()).dtype
        self.dev = next(model.parameters()).device
        self.embed = inner.embed_tokens.weight
        self.rotary = inner.rotary_emb
        self.final_norm = inner.norm.weight
        self.final_eps = float(getattr(inner.norm, "variance_epsilon", getattr(inner.norm, "eps", 1e-6)))
        self.lm_head = model.lm_head.weight
        if getattr(model.lm_head, "bias", None) is not None:
            raise NotImplementedError("lm_head bias")
        self.layers = []
        for layer in inner.layers:
            attn, mlp = layer.self_attn, layer.mlp
            for lin in (attn.q_proj, attn.k_proj, attn.v_proj, attn.o_proj, mlp.gate_proj,
                        mlp.up_proj, mlp.down_proj):
                if lin.bias is not None:
                    raise NotImplementedError("projection biases are not fused")
            w = _LayerWeights()
            w.ln1 = layer.input_layernorm.weight
            w.eps1 = float(layer.input_layernorm.variance_epsilon)
            w.wqkv = _fuse_qkv(attn)
            w.nq, w.nk = attn.q_proj.weight.shape[0], attn.k_proj.weight.shape[0]
            qn, kn = getattr(attn, "q_norm", None), getattr(attn, "k_norm", None)
            w.q_norm = None if qn is None else qn.weight
            w.k_norm = None if kn is None else kn.weight
            if (qn is not None and qn.weight.shape[0] != self.D) or \
                    (kn is not None and kn.weight.shape[0] != self.D):
                raise NotImplementedError("only per-head QK-norm is fused")
            w.qk_eps = float(qn.variance_epsilon) if qn is not None else 1e-6
            w.wo = attn.o_proj.weight
            w.ln2 = layer.post_attention_layernorm.weight
            w.eps2 = float(layer.post_attention_layernorm.variance_epsilon)
            w.wg, w.wu, w.wd = mlp.gate_proj.weight, mlp.up_proj.weight, mlp.down_proj.weight
            self.layers.append(w)
        B = max_batch
        n_qkv = self.layers[0].wqkv.shape[0]
        inter = self.layers[0].wg.shape[0]
        self.h = torch.empty(B, self.H, dtype=self.dtype, device=self.dev)
        self.qkv = torch.empty(B, n_qkv, dtype=self.dtype, device=self.dev)
        self.act = torch.empty(B, inter, dtype=self.dtype, device=self.dev)

    @staticmethod
    def _gemv(x, w, out, **kw):
        """helm_decode_gemv over batch slices whose inputs fit its staging."""
        n = _capi.gemv_max_batch(x.shape[1], x.element_size())
        res = kw.pop("residual", None)
        for b0 in range(0, x.shape[0], n):
            b1 = min(x.shape[0], b0 + n)
            _capi.decode_gemv(x[b0:b1], w, out=out[b0:b1],
                              residual=None if res is None else res[b0:b1], **kw)

    @torch.no_grad()
    def step(self, ids: torch.Tensor, pos: torch.Tensor, logits: torch.Tensor, ctx) -> None:
        """ids, pos [B, 1] (device); writes logits [B, vocab].  ctx: the
        GraphDecoder step context (pool, rows, tables, lengths, staging)."""
        B, D, Hq = ids.shape[0], self.D, self.Hq
        h, qkv, act = self.h[:B], self.qkv[:B], self.act[:B]
        torch.index_select(self.embed, 0, ids.view(-1), out=h)
        cos, sin = self.rotary(h.view(B, 1, self.H), pos)
        cos, sin = cos.reshape(B, D), sin.reshape(B, D)
        pool = ctx.pool.storage
        for l, w in enumerate(self.layers):
            self._gemv(h, w.wqkv, qkv, norm_w=w.ln1, eps=w.eps1)
            q = qkv[:, :w.nq].view(B, Hq, D)
            k = qkv[:, w.nq:w.nq + w.nk].view(B, -1, D)
            v = qkv[:, w.nq + w.nk:].view(B, -1, D)
            _capi.kv_append(q=q, k=k, v=v, q_out=ctx.q_out[l], q_norm_w=w.q_norm,
                            k_norm_w=w.k_norm, eps=w.qk_eps, cos=cos, sin=sin, pool=pool,
                            slot_rows=ctx.rows[l], page_size=ctx.P)
            ctx.before_attention(l)
            _capi.paged_decode_attention(ctx.q_out[l], pool, ctx.tables[l], ctx.lens[l],
                                         num_kv_heads=k.shape[1], page_size=ctx.P,
                                         scale=D ** -0.5, out=ctx.attn_out[l],
                                         max_kv_len_hint=ctx.max_len)
            ctx.after_attention(l)
            self._gemv(ctx.attn_out[l].view(B, Hq * D), w.wo, h, residual=h)
            self._gemv(h, w.wg, act, w2=w.wu, norm_w=w.ln2, eps=w.eps2)
            self._gemv(act, w.wd, h, residual=h)
        self._gemv(h, self.lm_head, logits, norm_w=self.final_norm, eps=self.final_eps)
