"""Generates the golden fixtures in tests/golden/ by running the HELM reference.

    PYTHONPATH=<helm checkout> python tests/golden/make_golden.py [--ref <helm checkout>]
        [--only attention|placement|norm_rope|prefill]

Everything here executes the reference's own code on seeded inputs and stores
inputs plus the reference's outputs:

  attention.npz   perform_streaming_attention (helm/runtime/kv_cache.py:405)
                  on paged inputs shaped like the reference's own tests
                  (tests/unit/runtime/test_streaming_attention.py) and on
                  head_dim 64/128 pools with 16/64-token pages
  placement.json  KVAllocator + KVCacheManager page placement / eviction
                  (kv_allocator.py, kv_cache.py:88-265) for scripted appends;
                  GPU-tier semantics come from giving the reference's page
                  tensors a 'cuda' device label (the policy only reads
                  .device.type), so no GPU is needed
  norm_rope.npz   transformers' Qwen3RMSNorm + apply_rotary_pos_emb as called
                  by the reference's Qwen3 attention patch (kv_offload.py:368-373)
  prefill.npz     perform_streaming_attention with q_len > 1: a prefill chunk
                  (the last S positions of each sequence, already in the
                  pages) under HELM's chunk-prefill mask
                  (pipeline_runtime.py:96-112), as _stream_prefill_batched
                  calls it (kv_offload.py:206-227)
  contiguous.npz  _decode_batched on the all-GPU contiguous path and its
                  migration to pages (kv_offload.py:115-142)
  config1_pipeline.npz
                  BASELINE configs[0] (Qwen3-0.6B architecture, seed-0
                  weights, 512-token prompt, 64 greedy steps) through the
                  reference's compile -> StageRuntimeExecutor ->
                  KVOffloadManager -> PipelineRuntime path, fp32 on the CPU

The fixtures are committed; this script is only needed to regenerate them.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _bits(t: torch.Tensor) -> np.ndarray:
    """bf16/fp16 tensor -> raw uint16 bits; fp32 -> float32."""
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy().astype(np.float32)


# ----------------------------------------------------------------- attention --
def _attention_cases():
    """(name, spec) pairs.  spec: Hq, Hkv, D, P, dtype, page sizes per batch item
    (list of lists of used tokens), scale, softcap, mask kind, q/k scaling."""
    c = []
    # shapes of the reference's own tests, lifted to kernel-supported head dims
    c.append(("single_page", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[4]])))
    c.append(("two_pages", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[4, 3]])))
    c.append(("three_pages_ragged", dict(Hq=1, Hkv=1, D=64, P=16, pages=[[3, 5, 2]])))
    c.append(("no_pages", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[]])))
    c.append(("zero_used_page", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[0]])))
    c.append(("empty_then_real", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[0, 4]])))
    c.append(("custom_scale", dict(Hq=1, Hkv=1, D=64, P=16, pages=[[3]], scale=0.25)))
    c.append(("gqa", dict(Hq=4, Hkv=2, D=64, P=16, pages=[[6]])))
    c.append(("gqa_multi_page", dict(Hq=4, Hkv=2, D=64, P=16, pages=[[4, 3]])))
    c.append(("large_logits", dict(Hq=1, Hkv=1, D=64, P=16, pages=[[8]], large=True)))
    c.append(("zero_mask", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[3, 5, 2]], mask="zero")))
    c.append(("padding_mask", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[4, 4, 3]],
                                   mask="pad:0,3,4,10")))
    c.append(("fully_masked_page", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[4, 4]],
                                        mask="pad:0,1,2,3")))
    c.append(("softcap", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[3, 5]], softcap=50.0)))
    c.append(("gqa_mask", dict(Hq=4, Hkv=2, D=64, P=16, pages=[[4, 3]], mask="pad:1")))
    c.append(("fp16_mask", dict(Hq=2, Hkv=2, D=64, P=16, pages=[[4, 4]], mask="zero",
                                dtype="float16")))
    # dense paging at the kernel's production shapes (small T)
    c.append(("dense_bf16_d128_p16", dict(Hq=8, Hkv=2, D=128, P=16, dense=[100, 37])))
    c.append(("dense_bf16_d128_p64_gqa4", dict(Hq=8, Hkv=2, D=128, P=64, dense=[70, 20])))
    c.append(("dense_fp16_mha", dict(Hq=4, Hkv=4, D=128, P=16, dense=[50], dtype="float16")))
    c.append(("dense_bf16_gqa5", dict(Hq=10, Hkv=2, D=128, P=16, dense=[77])))
    c.append(("dense_bf16_gqa16_d64", dict(Hq=16, Hkv=1, D=64, P=16, dense=[45])))
    c.append(("dense_bf16_d256", dict(Hq=4, Hkv=2, D=256, P=16, dense=[40])))
    c.append(("dense_bf16_mask_softcap", dict(Hq=8, Hkv=2, D=128, P=16, dense=[70, 33],
                                              mask="pad:5,16,17,31", softcap=30.0)))
    c.append(("dense_bf16_page8", dict(Hq=4, Hkv=2, D=128, P=8, dense=[27])))
    c.append(("dense_bf16_page24", dict(Hq=4, Hkv=2, D=128, P=24, dense=[61])))
    return c


def make_attention(ref, out_path: str):
    from helm.runtime.kv_cache import KVPage, perform_streaming_attention
    gen = torch.Generator().manual_seed(1234)
    arrays = {}
    names = []
    for name, s in _attention_cases():
        dtype = getattr(torch, s.get("dtype", "bfloat16"))
        Hq, Hkv, D, P = s["Hq"], s["Hkv"], s["D"], s["P"]
        if "dense" in s:
            lens = s["dense"]
            pages = [[min(P, L - i * P) for i in range(math.ceil(L / P))] for L in lens]
        else:
            pages = s["pages"]
        B = len(pages)
        maxp = max(1, max(len(p) for p in pages))
        n_used = sum(len(p) for p in pages)
        slots = n_used + 1
        perm = torch.randperm(slots, generator=gen)
        pool = torch.randn(slots, 2, Hkv, P, D, generator=gen).to(dtype)
        q = torch.randn(B, Hq, D, generator=gen).to(dtype)
        if s.get("large"):
            q = torch.full((B, Hq, D), 100.0).to(dtype)
            pool[:, 0] = 100.0
        page_table = np.zeros((B, maxp), np.int32)
        page_used = np.zeros((B, maxp), np.int32)
        num_pages = np.array([len(p) for p in pages], np.int32)
        k = 0
        for b, plist in enumerate(pages):
            for i, used in enumerate(plist):
                page_table[b, i] = int(perm[k])
                page_used[b, i] = used
                k += 1
        T = max(1, max(sum(p) for p in pages))
        mask = None
        mk = s.get("mask")
        if mk is not None:
            mask = torch.zeros(B, T)
            if mk.startswith("pad:"):
                for idx in mk[4:].split(","):
                    mask[:, int(idx)] = torch.finfo(torch.float32).min
        scale = s.get("scale")
        softcap = s.get("softcap")
        outs, outs32 = [], []
        for b in range(B):
            plist = []
            for i in range(int(num_pages[b])):
                slot = int(page_table[b, i])
                plist.append(KVPage(page_id=i, layer_id=0, start_token=0,
                                    used_tokens=int(page_used[b, i]), capacity_tokens=P,
                                    k_tensor=pool[slot, 0].unsqueeze(0),
                                    v_tensor=pool[slot, 1].unsqueeze(0),
                                    device=torch.device("cpu"), state="CPU"))
            qb = q[b:b + 1].unsqueeze(2)  # [1, Hq, 1, D]
            mb = None if mask is None else mask[b:b + 1].view(1, 1, 1, T)
            mb_t = None if mb is None else mb[..., :sum(int(u) for u in page_used[b])]
            o = perform_streaming_attention(qb, plist, scale=scale, attention_mask=mb_t,
                                            softcap=softcap)
            outs.append(o.view(Hq, D))
            # the same computation in fp32 (inputs are exact in fp32)
            plist32 = []
            for p in plist:
                plist32.append(KVPage(page_id=p.page_id, layer_id=0, start_token=0,
                                      used_tokens=p.used_tokens, capacity_tokens=P,
                                      k_tensor=p.k_tensor.float(), v_tensor=p.v_tensor.float(),
                                      device=p.device, state="CPU"))
            o32 = perform_streaming_attention(qb.float(), plist32, scale=scale,
                                              attention_mask=mb_t, softcap=softcap)
            outs32.append(o32.view(Hq, D))
        pre = name + "/"
        arrays[pre + "q"] = _bits(q)
        arrays[pre + "pool"] = _bits(pool)
        arrays[pre + "page_table"] = page_table
        arrays[pre + "page_used"] = page_used
        arrays[pre + "num_pages"] = num_pages
        arrays[pre + "out"] = _bits(torch.stack(outs))
        arrays[pre + "out_fp32"] = torch.stack(outs32).numpy()
        if mask is not None:
            arrays[pre + "mask"] = mask.numpy()
        arrays[pre + "meta"] = np.array([Hq, Hkv, D, P, 1 if "dense" in s else 0,
                                         0 if dtype == torch.bfloat16 else 1], np.int64)
        arrays[pre + "scale"] = np.array([scale if scale is not None else 1.0 / math.sqrt(D)],
                                         np.float64)
        arrays[pre + "softcap"] = np.array([softcap or 0.0], np.float64)
        names.append(name)
    arrays["names"] = np.array(names)
    np.savez_compressed(out_path, **arrays)


# ----------------------------------------------------------------- placement --
def _scenarios():
    sc = []

    def mk(name, L, H, D, P, elt, batch, wm, ops):
        sc.append(dict(name=name, num_layers=L, num_kv_heads=H, head_dim=D, page_size=P,
                       elem_bytes=elt, batch=batch, watermark_per_item=wm, ops=ops))

    def snapped(ops):
        out = []
        for op in ops:
            out.append(op)
            out.append(["snap"])
        return out

    # CPU tier only, as tests/unit/runtime/test_kv_cache.py drives it
    mk("cpu_prefill_decode", 4, 2, 8, 4, 4, 1, 0, snapped(
        [["prefill", 0, 0, 9, "cpu"], ["decode", 0, 0, "cpu"], ["decode", 0, 0, "cpu"],
         ["decode", 0, 0, "cpu"], ["decode", 0, 0, "cpu"], ["prefill", 0, 3, 2, "cpu"],
         ["evict", 0, 99999], ["clear", 0], ["prefill", 0, 1, 5, "cpu"]]))
    # GPU tier, zero watermark: evict everything evictable after every append
    mk("gpu_zero_watermark", 2, 2, 8, 4, 4, 1, 0, snapped(
        [["prefill", 0, 0, 8, "cuda"], ["evict", 0, 999999], ["decode", 0, 0, "cuda"],
         ["decode", 0, 0, "cuda"], ["decode", 0, 0, "cuda"], ["decode", 0, 0, "cuda"],
         ["decode", 0, 0, "cuda"], ["prefill", 0, 1, 10, "cuda"], ["clear", 0],
         ["prefill", 0, 0, 6, "cuda"]]))
    # high watermark then an explicit eviction (test_evict_pages_increments_counters)
    mk("gpu_explicit_evict", 2, 2, 8, 4, 4, 1, 10 ** 12, snapped(
        [["prefill", 0, 0, 8, "cuda"], ["evict", 0, 999999], ["decode", 0, 0, "cuda"]]))
    # strict '>' watermark: exactly two full non-tail pages fit
    page_b = 2 * 2 * 4 * 8 * 2
    mk("gpu_watermark_boundary", 2, 2, 8, 4, 2, 1, 2 * page_b, snapped(
        [["prefill", 0, 0, 12, "cuda"], ["decode", 0, 0, "cuda"], ["prefill", 0, 1, 12, "cuda"],
         ["decode", 0, 1, "cuda"], ["decode", 0, 0, "cuda"], ["decode", 0, 0, "cuda"],
         ["decode", 0, 0, "cuda"], ["decode", 0, 0, "cuda"]]))
    # global oldest-first across layers, decode interleaved per layer
    ops = [["prefill", 0, lid, 10 + 3 * lid, "cuda"] for lid in range(3)]
    for step in range(9):
        for lid in range(3):
            ops.append(["decode", 0, lid, "cuda"])
    mk("gpu_multilayer_oldest_first", 3, 2, 8, 4, 2, 1, 3 * page_b, snapped(ops))
    # batch items sharing one allocator, per-item watermark split, pool reuse
    ops = []
    for item in range(3):
        ops.append(["prefill", item, 0, 7 + 2 * item, "cuda"])
        ops.append(["prefill", item, 1, 7 + 2 * item, "cuda"])
    for step in range(6):
        for item in range(3):
            for lid in range(2):
                ops.append(["decode", item, lid, "cuda"])
    ops += [["clear", 1], ["prefill", 1, 0, 9, "cuda"], ["clear", 0], ["clear", 2],
            ["prefill", 2, 1, 5, "cuda"]]
    mk("gpu_batch_shared_allocator", 2, 2, 8, 4, 2, 3, max((4 * page_b) // 3, 1), snapped(ops))
    # chunked prefill leaves a partially filled page in the middle
    mk("gpu_chunked_prefill_ragged", 1, 2, 8, 4, 2, 1, page_b, snapped(
        [["prefill", 0, 0, 6, "cuda"], ["prefill", 0, 0, 6, "cuda"], ["decode", 0, 0, "cuda"],
         ["decode", 0, 0, "cuda"], ["decode", 0, 0, "cuda"], ["evict", 0, 10 ** 9]]))
    # decode without residency enforcement, then a later enforcing append
    mk("gpu_skip_residency", 1, 2, 8, 4, 2, 1, 0, snapped(
        [["decode_skip", 0, 0, "cuda"] for _ in range(9)] + [["decode", 0, 0, "cuda"]]))
    # Qwen3-0.6B-shaped cache (28 layers, 8 KV heads, D 128, page 64, bf16):
    # default KVOffloadConfig watermark -> no eviction at 512+64 tokens
    L, H, D, P = 28, 8, 128, 64
    default_wm = 512 * 2 * H * D * 2 * L
    ops = [["prefill", 0, lid, 512, "cuda"] for lid in range(L)] + [["snap"]]
    for step in range(64):
        for lid in range(L):
            ops.append(["decode", 0, lid, "cuda"])
    ops.append(["snap"])
    mk("qwen3_0p6b_default_watermark", L, H, D, P, 2, 1, default_wm, ops)
    # same cache with the forced 1024-byte watermark of test_kv_eviction_e2e
    ops = [["prefill", 0, lid, 512, "cuda"] for lid in range(L)] + [["snap"]]
    for step in range(64):
        for lid in range(L):
            ops.append(["decode", 0, lid, "cuda"])
        if step in (0, 63):
            ops.append(["snap"])
    mk("qwen3_0p6b_forced_watermark", L, H, D, P, 2, 1, 1024, ops)
    return sc


class _FakeCudaTensor(torch.Tensor):
    """A CPU tensor whose .device reads 'cuda:0' (the policy's only GPU test)."""

    @property
    def device(self):
        return torch.device("cuda:0")


def _fake_cuda_torch():
    """A stand-in for the torch module inside the reference's kv modules:
    tensors requested on a CUDA device are made on the CPU and labelled
    'cuda', so the GPU-tier policy runs without a GPU."""
    real_empty, real_zeros = torch.empty, torch.zeros

    def on_fake_cuda(fn, a, kw):
        dev = kw.get("device")
        if dev is not None and torch.device(dev).type == "cuda":
            kw["device"] = "cpu"
            return fn(*a, **kw).as_subclass(_FakeCudaTensor)
        return fn(*a, **kw)

    class TorchShim:
        def __getattr__(self, n):
            return getattr(torch, n)

        def empty(self, *a, **kw):
            return on_fake_cuda(real_empty, a, kw)

        def zeros(self, *a, **kw):
            return on_fake_cuda(real_zeros, a, kw)

    return TorchShim()


def make_placement(ref, out_path: str):
    import helm.runtime.kv_allocator as ka
    import helm.runtime.kv_cache as kc

    FakeCudaTensor = _FakeCudaTensor
    ka.torch = _fake_cuda_torch()
    results = []
    for sc in _scenarios():
        dtype = {4: torch.float32, 2: torch.bfloat16}[sc["elem_bytes"]]
        alloc = ka.KVAllocator(sc["num_layers"], sc["num_kv_heads"], sc["head_dim"],
                               page_size=sc["page_size"], dtype=dtype)
        kc.reset_paging_stats()
        mgrs = [kc.KVCacheManager(alloc, gpu_high_watermark_bytes=sc["watermark_per_item"])
                for _ in range(sc["batch"])]
        H, D = sc["num_kv_heads"], sc["head_dim"]

        def kv(n, dev):
            t = torch.zeros(1, H, n, D, dtype=dtype)
            return t.as_subclass(FakeCudaTensor) if dev == "cuda" else t

        snaps = []
        for op in sc["ops"]:
            kind = op[0]
            if kind == "prefill":
                t = kv(op[3], op[4])
                mgrs[op[1]].append_prefill(op[2], t, t)
            elif kind in ("decode", "decode_skip"):
                t = kv(1, op[3])
                mgrs[op[1]].append_decode(op[2], t, t, skip_residency=(kind == "decode_skip"))
            elif kind == "evict":
                mgrs[op[1]].evict_pages(op[2])
            elif kind == "clear":
                mgrs[op[1]].clear()
            elif kind == "snap":
                items = []
                for m in mgrs:
                    layers = []
                    for lid in sorted(m.layers):
                        lay = m.layers[lid]
                        layers.append([lid, lay.total_tokens,
                                       None if lay.tail_page is None else lay.tail_page.page_id,
                                       [[p.page_id, p.layer_id, p.start_token, p.used_tokens,
                                         p.capacity_tokens, p.state, p.device.type]
                                        for p in lay.pages]])
                    items.append(layers)
                snaps.append({"items": items,
                              "alloc": {"gpu_total": alloc.gpu_total_pages,
                                        "cpu_total": alloc.cpu_total_pages,
                                        "gpu_free": [p.page_id for p in alloc.gpu_free_pool],
                                        "cpu_free": [p.page_id for p in alloc.cpu_free_pool]},
                              "stats": kc.get_paging_stats()})
        results.append(dict(scenario=sc, snapshots=snaps))
    with open(out_path, "w") as f:
        json.dump(results, f, separators=(",", ":"))


# ----------------------------------------------------------------- norm/rope --
def make_norm_rope(ref, out_path: str):
    from transformers.models.qwen3.configuration_qwen3 import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3RMSNorm, Qwen3RotaryEmbedding,
                                                          apply_rotary_pos_emb)
    gen = torch.Generator().manual_seed(7)
    arrays = {}
    for dtype_name, theta, N, Hq, Hkv in (("bfloat16", 1e6, 5, 16, 8),
                                          ("bfloat16", 1e6, 3, 32, 8),
                                          ("float16", 1e4, 4, 8, 8)):
        dtype = getattr(torch, dtype_name)
        D = 128
        cfg = Qwen3Config(hidden_size=Hq * D, num_attention_heads=Hq, num_key_value_heads=Hkv,
                          head_dim=D, rope_theta=theta, max_position_embeddings=140000)
        rot = Qwen3RotaryEmbedding(cfg)
        qn = Qwen3RMSNorm(D, eps=1e-6).to(dtype)
        kn = Qwen3RMSNorm(D, eps=1e-6).to(dtype)
        with torch.no_grad():
            qn.weight.copy_(1.0 + 0.1 * torch.randn(D, generator=gen))
            kn.weight.copy_(1.0 + 0.1 * torch.randn(D, generator=gen))
        q = (torch.randn(1, N, Hq, D, generator=gen) * 3).to(dtype)
        k = (torch.randn(1, N, Hkv, D, generator=gen) * 3).to(dtype)
        pos = torch.tensor([[0, 1, 511, 4097, 131071][:N]])
        x = torch.zeros(1, N, Hq * D, dtype=dtype)
        cos, sin = rot(x, pos)
        with torch.no_grad():
            qo = qn(q).transpose(1, 2)
            ko = kn(k).transpose(1, 2)
            qo, ko = apply_rotary_pos_emb(qo, ko, cos, sin)
        tag = f"{dtype_name}_h{Hq}"
        arrays[tag + "/q"] = _bits(q[0])
        arrays[tag + "/k"] = _bits(k[0])
        arrays[tag + "/qw"] = _bits(qn.weight.detach())
        arrays[tag + "/kw"] = _bits(kn.weight.detach())
        arrays[tag + "/cos"] = _bits(cos[0])
        arrays[tag + "/sin"] = _bits(sin[0])
        arrays[tag + "/pos"] = pos[0].numpy()
        arrays[tag + "/theta"] = np.array([theta])
        arrays[tag + "/q_out"] = _bits(qo[0].transpose(0, 1))   # [N, Hq, D]
        arrays[tag + "/k_out"] = _bits(ko[0].transpose(0, 1))
    np.savez_compressed(out_path, **arrays)


# ------------------------------------------------------------------- prefill --
def _chunk_mask(lens, S, T, dtype, pad=None):
    """HELM's chunk-prefill mask, built the way PipelineRuntime builds it
    (pipeline_runtime.py:96-112): a query at position past + i sees keys
    <= past + i; key padding adds finfo.min on padded keys."""
    min_val = torch.finfo(dtype).min
    B = len(lens)
    masks = []
    for b in range(B):
        past = lens[b] - S
        q_idx = torch.arange(S).view(S, 1)
        k_idx = torch.arange(T).view(1, T)
        m = torch.where(k_idx <= past + q_idx, torch.zeros((), dtype=dtype),
                        torch.full((), min_val, dtype=dtype))
        if pad and b in pad:
            keys = torch.ones(T, dtype=dtype)
            keys[:pad[b]] = 0
            m = m + ((1.0 - keys) * min_val).view(1, T)
        masks.append(m)
    return torch.stack(masks).view(B, 1, S, T)


def _prefill_cases():
    c = []
    c.append(("chunk_causal_bf16_d128_p16",
              dict(Hq=8, Hkv=2, D=128, P=16, lens=[200], S=40)))
    c.append(("chunk_padded_bf16_d64_p16",
              dict(Hq=4, Hkv=4, D=64, P=16, lens=[150, 150], S=30, pad={0: 5})))
    c.append(("chunk_softcap_fp16_d128_p64",
              dict(Hq=4, Hkv=2, D=128, P=64, lens=[130], S=33, softcap=30.0,
                   dtype="float16")))
    c.append(("first_chunk_gqa8_d64_p32",
              dict(Hq=8, Hkv=1, D=64, P=32, lens=[100], S=100)))
    return c


def make_prefill(ref, out_path: str):
    from helm.runtime.kv_cache import KVPage, perform_streaming_attention
    gen = torch.Generator().manual_seed(4321)
    arrays = {}
    names = []
    for name, s in _prefill_cases():
        dtype = getattr(torch, s.get("dtype", "bfloat16"))
        Hq, Hkv, D, P, S = s["Hq"], s["Hkv"], s["D"], s["P"], s["S"]
        lens = s["lens"]
        B, T = len(lens), max(lens)
        maxp = max(math.ceil(L / P) for L in lens)
        slots = B * maxp + 1
        perm = torch.randperm(slots, generator=gen)
        pool = torch.randn(slots, 2, Hkv, P, D, generator=gen).to(dtype)
        q = torch.randn(B, Hq, S, D, generator=gen).to(dtype)
        page_table = np.zeros((B, maxp), np.int32)
        for b in range(B):
            for i in range(math.ceil(lens[b] / P)):
                page_table[b, i] = int(perm[b * maxp + i])
        mask = _chunk_mask(lens, S, T, dtype, s.get("pad"))
        softcap = s.get("softcap")
        outs, outs32 = [], []
        for b in range(B):
            for fp32 in (False, True):
                plist = []
                for i in range(math.ceil(lens[b] / P)):
                    slot = int(page_table[b, i])
                    k, v = pool[slot, 0].unsqueeze(0), pool[slot, 1].unsqueeze(0)
                    if fp32:
                        k, v = k.float(), v.float()
                    plist.append(KVPage(page_id=i, layer_id=0, start_token=i * P,
                                        used_tokens=min(P, lens[b] - i * P), capacity_tokens=P,
                                        k_tensor=k, v_tensor=v, device=torch.device("cpu"),
                                        state="CPU"))
                qb = q[b:b + 1].float() if fp32 else q[b:b + 1]
                o = perform_streaming_attention(qb, plist, scale=None,
                                                attention_mask=mask[b:b + 1, :, :, :lens[b]],
                                                softcap=softcap)
                (outs32 if fp32 else outs).append(o[0])
        pre = name + "/"
        arrays[pre + "q"] = _bits(q)
        arrays[pre + "pool"] = _bits(pool)
        arrays[pre + "page_table"] = page_table
        arrays[pre + "lens"] = np.array(lens, np.int32)
        arrays[pre + "mask"] = mask.float().numpy()
        arrays[pre + "out"] = _bits(torch.stack(outs))
        arrays[pre + "out_fp32"] = torch.stack(outs32).numpy()
        arrays[pre + "meta"] = np.array([Hq, Hkv, D, P, S, 0 if dtype == torch.bfloat16 else 1],
                                        np.int64)
        arrays[pre + "softcap"] = np.array([softcap or 0.0], np.float64)
        names.append(name)
    arrays["names"] = np.array(names)
    np.savez_compressed(out_path, **arrays)


# ---------------------------------------------------------------- contiguous --
def make_contiguous(ref, out_path: str):
    """The all-GPU contiguous path of _decode_batched (kv_offload.py:115-142)
    as HELM's inference front end enables it (cont_capacity set,
    inference.py:729-731): one prefill of 37 tokens, then decode steps; the
    first 27 go to the contiguous buffers, at cont_capacity = 64 the decode
    tokens migrate to pages (kv_cache.py:317-335) and the rest run on pages.
    GPU-tier placement via 'cuda'-labelled CPU tensors, as in placement.json.
    Stores inputs, every step's attention output, the counters after every
    step and the final page placement."""
    import helm.runtime.kv_allocator as ka
    import helm.runtime.kv_cache as kc
    import helm.runtime.kv_offload as ko
    shim = _fake_cuda_torch()
    ka.torch = shim
    kc.torch = shim
    L, B, Hq, Hkv, D, P, S, CAP, STEPS = 2, 2, 4, 2, 64, 16, 37, 64, 35
    dtype = torch.bfloat16
    gen = torch.Generator().manual_seed(2024)
    pre_k = torch.randn(L, B, Hkv, S, D, generator=gen).to(dtype)
    pre_v = torch.randn(L, B, Hkv, S, D, generator=gen).to(dtype)
    qs = torch.randn(STEPS, L, B, Hq, 1, D, generator=gen).to(dtype)
    ks = torch.randn(STEPS, L, B, Hkv, 1, D, generator=gen).to(dtype)
    vs = torch.randn(STEPS, L, B, Hkv, 1, D, generator=gen).to(dtype)
    alloc = ka.KVAllocator(L, Hkv, D, page_size=P, dtype=dtype)
    kc.reset_paging_stats()
    mgrs = [kc.KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12) for _ in range(B)]
    for m in mgrs:
        assert m.build_contiguous(num_layers=L, num_kv_heads=Hkv, head_dim=D, capacity=CAP,
                                  device=torch.device("cuda:0"), dtype=dtype)
    fake = (lambda t: t.clone().as_subclass(_FakeCudaTensor))
    for lid in range(L):
        ko._append_prefill_batched(mgrs, fake(pre_k[lid]), fake(pre_v[lid]), lid)
    outs, counters = [], []
    scale = D ** -0.5
    for st in range(STEPS):
        for lid in range(L):
            o = ko._decode_batched(mgrs, fake(qs[st, lid]), fake(ks[st, lid]),
                                   fake(vs[st, lid]), lid, scale)
            outs.append(torch.Tensor(o).as_subclass(torch.Tensor)[:, :, 0].clone())
        counters.append([int(mgrs[0].use_contiguous), mgrs[0].cont_seq_len,
                         mgrs[0].cont_prefill_len])
    placement = []
    for b, m in enumerate(mgrs):
        for lid in sorted(m.layers):
            for p in m.layers[lid].pages:
                placement.append([b, lid, p.page_id, p.start_token, p.used_tokens,
                                  p.capacity_tokens, 1 if p.state == "GPU" else 0])
    np.savez_compressed(
        out_path, pre_k=_bits(pre_k), pre_v=_bits(pre_v), q=_bits(qs), k=_bits(ks), v=_bits(vs),
        out=_bits(torch.stack(outs).view(STEPS, L, B, Hq, D)),
        counters=np.array(counters, np.int64), placement=np.array(placement, np.int64),
        meta=np.array([L, B, Hq, Hkv, D, P, S, CAP, STEPS], np.int64))


# ------------------------------------------------------------------- config 1 --
def make_config1(ref, out_path: str):
    """BASELINE configs[0] through the reference's own pipeline, as its
    execute_stagewise mode runs it (helm/_pipeline.py:530-573): the
    Qwen3-0.6B architecture with seed-0 N(0, 0.02) weights (helm_b200.synthetic,
    rounded to bf16 so that the GPU run loads the same model), in fp32 on the
    CPU, a 512-token random prompt, FX capture -> compile_graph with a manual
    all-CPU plan -> DecodeTracer -> StageRuntimeExecutor -> KVOffloadManager
    (default config: 64-token pages) -> PipelineRuntime.generate, 64 greedy
    steps.  Stores the tokens, the full logits of the first step and the
    top-32 logits of every step."""
    import tempfile
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    import helm.kernels as hk
    from helm._pipeline import capture_decode_fx_graph, capture_fx_graph
    from helm.compiler.compiler import HelmCompileOptions, compile_graph
    from helm.compiler.importers.decode_tracer import DecodeTracer
    from helm.runtime.executor import StageRuntimeExecutor
    from helm.runtime.kv_offload import KVOffloadConfig, KVOffloadManager
    from helm.runtime.pipeline_runtime import PipelineRuntime
    from helm_b200.synthetic import build_model, make_config
    hk._load_error = "not built: fp32 weights take torch's linear"   # no JIT build
    torch.set_num_threads(os.cpu_count() or 1)
    S, STEPS = 512, 64
    cfg = make_config("qwen3-0.6b")
    model = build_model(cfg, seed=0, std=0.02, dtype=torch.bfloat16, device="cpu").float()
    ids = torch.randint(0, cfg.vocab_size, (1, S), generator=torch.Generator().manual_seed(0))
    mask_dtype = torch.float16
    causal = torch.triu(torch.full((S, S), torch.finfo(mask_dtype).min, dtype=mask_dtype),
                        diagonal=1)[None, None]
    dummy = (ids, causal, torch.arange(S).unsqueeze(0), torch.arange(S))
    L = cfg.num_hidden_layers

    def options(kind):
        return HelmCompileOptions(
            mode="both", objective="decode_latency", plan_mode="manual",
            cpu_layers=f"0:{L - 1}", gpu_layers=None, lower_stages=True, graph_kind=kind,
            model_name="qwen3-0.6b-random", kv_offload=True,
            workload={"batch_size": 1, "prefill_seq_len": S, "decode_context_len": S,
                      "decode_tokens": STEPS, "dtype_size": 2})
    with tempfile.TemporaryDirectory() as run_dir:
        gm = capture_fx_graph(model, dummy, run_dir, allow_fallback=True,
                              trace_policy="explicit_leaf")
        pre = compile_graph(gm=gm, example_inputs=dummy, model=model, tokenizer=None,
                            options=options("prefill"), artifacts_dir=run_dir)
        dd = DecodeTracer.build_dummy_inputs(device="cpu", batch_size=1, dtype=mask_dtype)
        dgm = capture_decode_fx_graph(model, dd, run_dir)
        dec = compile_graph(gm=dgm, example_inputs=dd, model=model, tokenizer=None,
                            options=options("decode"), partition_plan_override=pre.partition_plan,
                            artifacts_dir=os.path.join(run_dir, "decode"))
        mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model))
        pexec, dexec = StageRuntimeExecutor(pre.stage_graphs), StageRuntimeExecutor(dec.stage_graphs)
        mgr.patch_module_roots(*(st.module for st in pexec.stages),
                               *(st.module for st in dexec.stages))
        rt = PipelineRuntime(pexec, dexec, tokenizer=None, dtype=mask_dtype, kv_offload_mgr=mgr)
        seen = []
        select, step = rt._select_next_token_logits, rt.decode_step

        def select_rec(logits, lengths):
            out = select(logits, lengths)
            seen.append(out[0].float().clone())
            return out

        def step_rec(*a, **kw):
            out = step(*a, **kw)
            seen.append(out[0, -1].float().clone())
            return out
        rt._select_next_token_logits, rt.decode_step = select_rec, step_rec
        toks = rt.generate(ids, STEPS)
    logits = torch.stack(seen[:STEPS])                       # [64, vocab]
    top = torch.topk(logits, 32, dim=-1)
    assert torch.equal(top.indices[:, 0], toks[0]), "argmax of the recorded logits"
    np.savez_compressed(out_path, prompt=ids[0].numpy(), tokens=toks[0].numpy(),
                        logits0=logits[0].numpy(), top_ids=top.indices.numpy(),
                        top_vals=top.values.numpy())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("HELM_REFERENCE"),
                    help="HELM checkout to run (default: $HELM_REFERENCE)")
    ap.add_argument("--only", choices=["attention", "placement", "norm_rope", "prefill",
                                       "contiguous", "config1"],
                    default=None)
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the HELM checkout with --ref or HELM_REFERENCE")
    sys.path.insert(0, args.ref)
    import helm  # noqa: F401  (fails loudly when the reference is absent)
    torch.manual_seed(0)
    makers = {"attention": (make_attention, "attention.npz"),
              "placement": (make_placement, "placement.json"),
              "norm_rope": (make_norm_rope, "norm_rope.npz"),
              "prefill": (make_prefill, "prefill.npz"),
              "contiguous": (make_contiguous, "contiguous.npz"),
              "config1": (make_config1, "config1_pipeline.npz")}
    for key, (fn, fname) in makers.items():
        if args.only is None or args.only == key:
            fn(args.ref, os.path.join(HERE, fname))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
