"""Decode attention across the GPUs of one node: sequence split and KV-head sharding.

HELM runs on one GPU (its planner declares multi-GPU but does not implement
it, compiler/optimization/strategy_selector.py:86-90); this module adds the two
multi-GPU forms of its decode attention:

Sequence split (long contexts).  Rank r of N holds a contiguous, page-aligned
token range of every sequence in its own page pool.  Each decode step it
computes the partial attention state of its range with the paged decode
kernel (O in fp32 and LSE); one native kernel then pushes the state to every
rank over NVLink (CUDA IPC mappings of per-rank exchange buffers), waits for
the other ranks' states and merges them (PeerExchange).  The NCCL form --
all-gather of the packed states, then the merge kernel -- is kept for
process groups without peer mappings (and gloo on CPU).  The merge is

    M = max_r LSE_r,  O = sum_r e^(LSE_r - M) O_r / sum_r e^(LSE_r - M)

which is the running-max rescale of the reference's streaming attention
(helm/runtime/kv_cache.py:523-529) taken across devices.  New tokens are
appended on the rank that holds the tail of the sequence.

KV-head sharding.  Rank r owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query
heads; attention needs no exchange (a model gathers or reduces afterwards,
e.g. the all-reduce after a row-parallel o_proj).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .. import _capi


def split_ranges(total_tokens: int, page_size: int, world: int) -> list:
    """Contiguous page-aligned [start, end) token ranges, one per rank, as even
    as whole pages allow; the last rank also takes the partial tail page."""
    pages = -(-total_tokens // page_size) if total_tokens > 0 else 0
    bounds = [(pages * r) // world for r in range(world + 1)]
    return [(min(bounds[r] * page_size, total_tokens), min(bounds[r + 1] * page_size, total_tokens))
            for r in range(world)]


def head_range(num_kv_heads: int, num_q_heads: int, rank: int, world: int):
    """(kv head range, q head range) owned by `rank` under KV-head sharding."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV heads do not split over {world} ranks")
    per = num_kv_heads // world
    group = num_q_heads // num_kv_heads
    kv = (rank * per, (rank + 1) * per)
    return kv, (kv[0] * group, kv[1] * group)


class PeerExchange:
    """Per-rank exchange buffers mapped into every rank (CUDA IPC), for
    helm_seq_exchange_merge.  Collective: every rank of `group` constructs it
    with the same rows / head_dim and calls merge() the same number of times."""

    def __init__(self, rows: int, head_dim: int, device: torch.device,
                 group: Optional[dist.ProcessGroup] = None, timeout_s: float = 5.0):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.rows, self.head_dim, self.device = rows, head_dim, torch.device(device)
        self.timeout_s = timeout_s
        self.nbytes = _capi.peer_exchange_bytes(rows, head_dim, self.world)
        self.local = _capi.ipc_alloc(self.nbytes, self.device)
        handles = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, _capi.ipc_get_handle(self.local, self.device),
                                   group=group)
        self.ptrs = [self.local if r == self.rank else _capi.ipc_open(handles[r], self.device)
                     for r in range(self.world)]
        if self.world > 1:
            dist.barrier(group=group)

    def merge(self, o_part: torch.Tensor, lse_part: torch.Tensor, out: torch.Tensor,
              lse_out: Optional[torch.Tensor] = None, stream=None) -> None:
        _capi.seq_exchange_merge(self.ptrs, self.rank, o_part, lse_part, out, lse_out,
                                 timeout_s=self.timeout_s, stream=stream)

    def reset(self) -> None:
        """Re-zeroes this rank's buffer (all ranks, e.g. after a timeout)."""
        torch.cuda.synchronize(self.device)
        _capi.ipc_zero(self.local, self.nbytes, self.device)
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)

    def close(self) -> None:
        if self.ptrs is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)     # no rank still writes into a buffer
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                _capi.ipc_close(p, self.device)
        if self.world > 1:
            dist.barrier(group=self.group)     # every mapping of this buffer is closed
        _capi.ipc_free(self.local, self.device)
        self.ptrs = None


class SeqSplitAttention:
    """Merged decode attention over a sequence split across the ranks of `group`.

    partial_fn(q, rows_out_fp32, lse_out) computes this rank's state into the
    given buffers; the default is the paged decode kernel over this rank's
    pool (see decode()).  gather and merge use NCCL and the native merge
    kernel on GPUs; other process groups (gloo, for host-side tests) take the
    same packed-buffer path with their own collective.
    """

    def __init__(self, group: Optional[dist.ProcessGroup] = None,
                 merge_fn: Optional[Callable] = None, exchange: str = "p2p"):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.merge_fn = merge_fn or _capi.merge_attention_states
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.exchange_kind = exchange
        self._peers: dict = {}

    def peer_exchange(self, rows: int, head_dim: int, device) -> PeerExchange:
        key = (rows, head_dim, torch.device(device))
        px = self._peers.get(key)
        if px is None:
            px = self._peers[key] = PeerExchange(rows, head_dim, device, self.group)
        return px

    def close(self) -> None:
        for px in self._peers.values():
            px.close()
        self._peers.clear()

    def exchange(self, part: torch.Tensor) -> torch.Tensor:
        """All-gathers this rank's packed state [rows*(D+1)] -> [world, rows*(D+1)]."""
        if self.world == 1:
            return part.unsqueeze(0)
        out = torch.empty((self.world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
        if part.device.type == "cuda":
            dist.all_gather_into_tensor(out, part, group=self.group)
        else:
            dist.all_gather(list(out.unbind(0)), part, group=self.group)
        return out

    def merge(self, gathered: torch.Tensor, rows: int, D: int, out_dtype: torch.dtype):
        """gathered [world, rows*D + rows] fp32 -> (O [rows, D], LSE [rows])."""
        o_parts = gathered[:, :rows * D].view(self.world, rows, D)
        lse_parts = gathered[:, rows * D:]
        return self.merge_fn(o_parts, lse_parts, out_dtype)

    def decode(self, q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor,
               kv_lens: torch.Tensor, *, num_kv_heads: int, page_size: int, scale: float,
               mask: Optional[torch.Tensor] = None, softcap: Optional[float] = None,
               max_kv_len_hint: int = 0):
        """q [B, Hq, D] on every rank (same values); pool / page_table / kv_lens
        describe this rank's token range.  Returns (O [B, Hq, D] in q.dtype,
        LSE fp32 [B, Hq]) of attention over all ranks' ranges."""
        B, Hq, D = q.shape
        rows = B * Hq
        if self.world == 1 and q.device.type == "cuda":   # nothing to exchange
            lse = torch.empty(B, Hq, dtype=torch.float32, device=q.device)
            out, _ = _capi.paged_decode_attention(q, pool, page_table, kv_lens,
                                                  num_kv_heads=num_kv_heads, page_size=page_size,
                                                  scale=scale, softcap=softcap, mask=mask, lse=lse,
                                                  max_kv_len_hint=max_kv_len_hint)
            return out, lse
        part = torch.empty(rows * (D + 1), dtype=torch.float32, device=q.device)
        o_local = part[:rows * D].view(B, Hq, D)
        lse_local = part[rows * D:].view(B, Hq)
        _capi.paged_decode_attention(q, pool, page_table, kv_lens, num_kv_heads=num_kv_heads,
                                     page_size=page_size, scale=scale, softcap=softcap, mask=mask,
                                     out=o_local, lse=lse_local, max_kv_len_hint=max_kv_len_hint)
        if self.exchange_kind == "p2p" and q.device.type == "cuda" and self.world > 1:
            out = torch.empty(B, Hq, D, dtype=q.dtype, device=q.device)
            lse = torch.empty(B, Hq, dtype=torch.float32, device=q.device)
            self.peer_exchange(rows, D, q.device).merge(o_local.view(rows, D), lse_local.view(rows),
                                                        out, lse)
            return out, lse
        gathered = self.exchange(part)
        out, lse = self.merge(gathered, rows, D, q.dtype)
        return out.view(B, Hq, D), lse.view(B, Hq)


def head_sharded_decode(q_local: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor,
                        kv_lens: torch.Tensor, *, num_kv_heads_local: int, page_size: int,
                        scale: float, group: Optional[dist.ProcessGroup] = None,
                        gather: bool = False, mask: Optional[torch.Tensor] = None):
    """KV-head-sharded decode attention: q_local [B, Hq/N, D] and this rank's
    pool of Hkv/N heads.  With gather=True the outputs of all ranks are
    all-gathered along the head axis ([B, Hq, D])."""
    out, _ = _capi.paged_decode_attention(q_local, pool, page_table, kv_lens,
                                          num_kv_heads=num_kv_heads_local, page_size=page_size,
                                          scale=scale, mask=mask)
    if not gather or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return out
    world = dist.get_world_size(group)
    full = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device=out.device)
    dist.all_gather_into_tensor(full, out.contiguous(), group=group)
    B, h, D = out.shape
    return full.permute(1, 0, 2, 3).reshape(B, world * h, D)
