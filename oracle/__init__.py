"""ORACLE — test infrastructure only.

CPU restatements of HELM's paged-KV decode path, used to CHECK the CUDA
product path (tests, __graft_entry__.smoke) and as the timed CPU baseline of
bench.py.  Nothing in helm_b200/ imports this package.

  paged_attention.c   perform_streaming_attention math (kv_cache.py:405-662), C + pthreads
  placement.py        KVAllocator / KVCacheManager placement and eviction policy
                      (kv_allocator.py:6-163, kv_cache.py:88-265), metadata only
  norm_rope.py        Qwen3 QK-RMSNorm + rotate_half RoPE with eager bf16 rounding
  merge.py            (O, LSE) merge over disjoint key ranges

Pinning: tests/golden/ holds fixtures produced by running the reference itself
(tests/golden/make_golden.py); tests/test_oracle.py checks every restatement
here against them.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
_BUILD_DIR = os.path.join(_DIR, "_build")
_LIB_PATH = os.path.join(_BUILD_DIR, "liboracle.so")
_SRC = os.path.join(_DIR, "paged_attention.c")

DT_F32, DT_F16, DT_BF16 = 0, 1, 2
_lib = None


def build(force: bool = False) -> str:
    """Compiles the C restatement (gcc, x86-64-v3) into oracle/_build/."""
    if not force and os.path.exists(_LIB_PATH) and \
            os.path.getmtime(_LIB_PATH) >= os.path.getmtime(_SRC):
        return _LIB_PATH
    os.makedirs(_BUILD_DIR, exist_ok=True)
    tmp = _LIB_PATH + ".tmp"
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fPIC", "-shared", "-pthread", "-o", tmp, _SRC,
           "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(_LIB_PATH)
        P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        lib.oracle_paged_attention.restype = I
        lib.oracle_paged_attention.argtypes = [P, I, I, I, I, P, I, I, P, I64, P, P, P, I64, F, F,
                                               P, P, I]
        _lib = lib
    return _lib


def _np_ptr(a):
    return None if a is None else a.ctypes.data


def paged_attention(q: np.ndarray, pool: np.ndarray, pool_dtype: int, page_table: np.ndarray,
                    num_pages: np.ndarray, page_used: np.ndarray, *, num_kv_heads: int,
                    page_size: int, scale: float, softcap: float = 0.0,
                    mask: np.ndarray | None = None, threads: int = 1):
    """Decode attention over a page pool, fp32.

    q float32 [B, Hq, D]; pool [slots, 2, Hkv, P, D] as float32 (DT_F32) or as the
    raw uint16 bits of fp16/bf16; page_table / page_used int32 [B, maxp];
    num_pages int32 [B]; mask float32 [B, T] or None.
    Returns (out float32 [B, Hq, D], lse float32 [B, Hq]).
    """
    q = np.ascontiguousarray(q, dtype=np.float32)
    B, Hq, D = q.shape
    pool = np.ascontiguousarray(pool)
    page_table = np.ascontiguousarray(page_table, dtype=np.int32)
    page_used = np.ascontiguousarray(page_used, dtype=np.int32)
    num_pages = np.ascontiguousarray(num_pages, dtype=np.int32)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
    out = np.zeros((B, Hq, D), np.float32)
    lse = np.zeros((B, Hq), np.float32)
    rc = _load().oracle_paged_attention(
        _np_ptr(q), B, Hq, num_kv_heads, D, _np_ptr(pool), pool_dtype, page_size,
        _np_ptr(page_table), page_table.shape[1], _np_ptr(num_pages), _np_ptr(page_used),
        _np_ptr(mask), mask.shape[1] if mask is not None else 0, float(scale), float(softcap),
        _np_ptr(out), _np_ptr(lse), int(threads))
    if rc != 0:
        raise ValueError("oracle_paged_attention: invalid arguments")
    return out, lse


def dense_page_lists(kv_lens, page_size: int, max_pages: int):
    """(num_pages, page_used) for dense paging: every page full but the last."""
    kv_lens = np.asarray(kv_lens, dtype=np.int64)
    B = kv_lens.shape[0]
    num_pages = ((kv_lens + page_size - 1) // page_size).astype(np.int32)
    page_used = np.zeros((B, max_pages), np.int32)
    for b in range(B):
        n = int(num_pages[b])
        if n:
            page_used[b, :n] = page_size
            page_used[b, n - 1] = int(kv_lens[b]) - (n - 1) * page_size
    return num_pages, page_used
