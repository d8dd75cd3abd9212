"""ORACLE — test infrastructure only.

Numpy restatement of the q/k processing of HELM's patched Qwen3 attention
forward (helm/runtime/kv_offload.py:368-373), which calls transformers'
Qwen3RMSNorm and apply_rotary_pos_emb (transformers 5.x,
models/qwen3/modeling_qwen3.py: Qwen3RMSNorm.forward, rotate_half,
apply_rotary_pos_emb).  Each eager op's rounding to the model dtype is
reproduced:

    var = mean(x_f32^2)                     (fp32)
    y   = dtype(x_f32 * rsqrt(var + eps))   (hidden_states.to(input_dtype))
    z   = dtype(w * y)                      (weight * hidden_states)
    out = dtype( dtype(z * cos) + dtype(rotate_half(z) * sin) )

Arrays are float32 holding values exactly representable in `dtype`.
"""
from __future__ import annotations

import numpy as np


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round-to-nearest-even of float32 values to bf16 or fp16, returned as float32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype != "bfloat16":
        raise ValueError(dtype)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    out[nan] = np.nan
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (round_to(x, "bfloat16").view(np.uint32) >> 16).astype(np.uint16)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    x = np.asarray(x, np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    y = round_to(x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))), dtype)
    return round_to(np.asarray(w, np.float32) * y, dtype)


def rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str) -> np.ndarray:
    """x [..., D]; cos/sin broadcastable to x (HF rotate_half convention)."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return round_to(round_to(x * cos, dtype) + round_to(rot * sin, dtype), dtype)


def rope_tables(positions: np.ndarray, head_dim: int, theta: float, dtype: str):
    """cos/sin [N, D] as HF's default rotary embedding makes them (fp32, then cast)."""
    inv_freq = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32)
                                / head_dim))
    inv_freq = inv_freq.astype(np.float32)
    freqs = np.asarray(positions, np.float32)[:, None] * inv_freq[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float32)
    return round_to(np.cos(emb), dtype), round_to(np.sin(emb), dtype)
