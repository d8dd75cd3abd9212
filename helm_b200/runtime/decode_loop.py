"""Greedy generation over a model whose GPU attention runs on the paged cache.

Restates the caller of the hot path, HELM's PipelineRuntime
(helm/runtime/pipeline_runtime.py:63-338), for an unpartitioned HF causal LM
on one device: chunked prefill (HELM_PREFILL_CHUNK, default 512) with
chunk-causal additive masks, then one token per step with a [B, 1, 1, T]
key-padding mask, argmax decoding, eos/pad handling, and a reset of the KV
offload manager before every request.  The masks are handed to HF as prepared 4-D
additive masks, which it passes through unchanged, so every decoder layer and
its patched attention see exactly HELM's masks.
"""
from __future__ import annotations

import os
from typing import Optional

import torch


class DecodeLoop:
    def __init__(self, model, kv_offload_mgr=None, dtype: Optional[torch.dtype] = None):
        self.model = model
        self.kv_offload_mgr = kv_offload_mgr
        self.dtype = dtype or next(model.parameters()).dtype

    # masks (pipeline_runtime.py:63-113)
    def _position_ids(self, attention_mask):
        positions = attention_mask.cumsum(dim=1) - 1
        return positions.clamp_min(0) * attention_mask

    def _chunk_mask(self, past: int, chunk: int, device, attention_mask):
        total = past + chunk
        lo = torch.finfo(self.dtype).min
        q_idx = torch.arange(chunk, device=device).view(chunk, 1)
        k_idx = torch.arange(total, device=device).view(1, total)
        mask = torch.where(k_idx <= past + q_idx, torch.zeros((), device=device, dtype=self.dtype),
                           torch.full((), lo, device=device, dtype=self.dtype))[None, None]
        if attention_mask is not None:
            pad = (1.0 - attention_mask[:, :total].to(device=device, dtype=self.dtype)) * lo
            mask = mask + pad[:, None, None, :]
        return mask

    def _decode_mask(self, total: int, device, attention_mask):
        if attention_mask is None:
            return torch.zeros((1, 1, 1, total), device=device, dtype=self.dtype)
        lo = torch.finfo(self.dtype).min
        pad = (1.0 - attention_mask.to(device=device, dtype=self.dtype)) * lo
        return pad[:, None, None, :]

    def _forward(self, input_ids, mask, position_ids):
        # a prepared 4-D additive mask is passed through unchanged by HF
        out = self.model(input_ids=input_ids, attention_mask=mask, position_ids=position_ids,
                         use_cache=False, logits_to_keep=1)
        return out.logits[:, -1, :]

    @staticmethod
    def _chunk_size(seq_len: int) -> int:
        raw = os.environ.get("HELM_PREFILL_CHUNK", "512")
        try:
            chunk = int(raw)
        except ValueError:
            chunk = 512
        return 0 if chunk <= 0 or seq_len <= chunk else chunk

    @torch.no_grad()
    def prefill(self, input_ids, attention_mask=None):
        device = input_ids.device
        S = input_ids.shape[1]
        am = torch.ones_like(input_ids) if attention_mask is None else attention_mask.long()
        pos = self._position_ids(am)
        chunk = self._chunk_size(S) or S
        logits = None
        past = 0
        while past < S:
            n = min(chunk, S - past)
            logits = self._forward(input_ids[:, past:past + n],
                                   self._chunk_mask(past, n, device, am),
                                   pos[:, past:past + n])
            past += n
        return logits

    @torch.no_grad()
    def generate(self, input_ids, max_new_tokens: int = 8, attention_mask=None,
                 eos_token_id=None, pad_token_id=None, forced_tokens=None, keep_logits=False):
        """Greedy tokens [B, n].  forced_tokens [B, >= n] (optional) feeds those
        tokens instead of the argmax (teacher forcing) while still returning the
        argmax of every step; keep_logits also returns each step's logits."""
        if self.kv_offload_mgr is not None:
            self.kv_offload_mgr.reset()
        B, S = input_ids.shape
        am = torch.ones_like(input_ids) if attention_mask is None else attention_mask.long()
        prompt_lengths = am.sum(dim=1)
        logits = self.prefill(input_ids, am)
        out_tokens, all_logits = [], []
        finished = torch.zeros(B, dtype=torch.bool, device=logits.device)
        terminal = pad_token_id if pad_token_id is not None else eos_token_id
        dec_am = am.to(logits.device)
        positions = prompt_lengths.to(logits.device).clone()
        for step in range(max_new_tokens):
            if keep_logits:
                all_logits.append(logits.float())
            nxt = torch.argmax(logits, dim=-1, keepdim=True)
            if finished.any() and terminal is not None:
                nxt = nxt.clone()
                nxt[finished] = terminal
            out_tokens.append(nxt)
            if eos_token_id is not None:
                finished = finished | (nxt.squeeze(-1) == eos_token_id)
            if bool(finished.all()) or step + 1 >= max_new_tokens:
                break
            feed = nxt if forced_tokens is None else forced_tokens[:, step:step + 1].to(nxt.device)
            active = ~finished
            dec_am = torch.cat([dec_am, active.unsqueeze(1).to(dec_am.dtype)], dim=1)
            logits = self._forward(feed, self._decode_mask(S + step + 1, feed.device, dec_am),
                                   positions.unsqueeze(1))
            positions = positions + active.to(positions.dtype)
        toks = torch.cat(out_tokens, dim=1)
        return (toks, all_logits) if keep_logits else toks
