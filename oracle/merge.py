"""ORACLE — test infrastructure only.

Numpy restatement of merging attention states computed over disjoint key
ranges, the cross-partition form of the running-max rescale of
perform_streaming_attention (helm/runtime/kv_cache.py:523-529):

    M = max_r lse_r,   w_r = exp(lse_r - M)
    O = sum_r w_r O_r / sum_r w_r,   LSE = M + log(sum_r w_r)

A partition with lse = -inf (no keys) has weight 0.
"""
from __future__ import annotations

import numpy as np


def merge_states(o_parts: np.ndarray, lse_parts: np.ndarray):
    """o_parts [R, rows, D], lse_parts [R, rows] -> (O [rows, D], LSE [rows]), fp64 math."""
    o = np.asarray(o_parts, np.float64)
    lse = np.asarray(lse_parts, np.float64)
    M = np.max(lse, axis=0)
    m_use = np.where(np.isneginf(M), 0.0, M)
    w = np.exp(lse - m_use[None])
    L = w.sum(axis=0)
    out = np.where(L[:, None] > 0, (w[..., None] * o).sum(axis=0) / np.where(L > 0, L, 1)[:, None],
                   0.0)
    lse_out = np.where(L > 0, M + np.log(np.where(L > 0, L, 1)), -np.inf)
    return out.astype(np.float32), lse_out.astype(np.float32)
