"""ctypes binding of libhelm_b200.so (the C ABI declared in include/helm_b200.h)
plus thin wrappers that take torch tensors and pass their raw pointers.

PyTorch is only the plumbing here: it owns device memory and streams.  Every
computation runs in the native library; when the library is missing these
functions raise instead of computing anything another way.
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

from . import build as _build

HELM_OK = 0
DTYPE_FP32, DTYPE_FP16, DTYPE_BF16 = 0, 1, 2
DEV_TIMEOUT, DEV_BAD_PAGE = 1, 2

_TORCH_TO_HELM = {torch.float32: DTYPE_FP32, torch.float16: DTYPE_FP16,
                  torch.bfloat16: DTYPE_BF16}

# name -> (restype, argtypes); must match include/helm_b200.h exactly.
_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
_SIGNATURES = {
    "helm_version": (_I, []),
    "helm_set_decode_overlap": (_I, [_I]),
    "helm_status_string": (ctypes.c_char_p, [_I]),
    "helm_last_cuda_error": (ctypes.c_char_p, []),
    "helm_get_device_status": (_I, [ctypes.POINTER(ctypes.c_uint), _I, _P]),
    "helm_paged_decode_workspace_bytes": (_I64, [_I, _I, _I, _I]),
    "helm_paged_decode_attention": (_I, [
        _P, _I64, _I64,            # q, strides
        _P, _I64,                  # pool, pool_pages
        _P, _I64, _I,              # page_table, pt_stride_b, max_pages
        _P, _P, _P, _P,            # kv_lens, num_pages, page_used, page_start
        _P, _I, _I64,              # mask, mask_dtype, mask_stride_b
        _P, _I64, _I64, _P,        # out, strides, lse
        _P, _I64,                  # workspace, bytes
        _I, _I, _I, _I, _I, _I, _I,  # batch, hq, hkv, head_dim, page_size, dtype, out_dtype
        _F, _F, _I, _P]),          # scale, softcap, max_kv_len_hint, stream
    "helm_paged_decode_attention_noalloc": (_I, [
        _P, _I64, _I64, _P, _I64, _P, _I64, _I, _P, _P, _P, _P,
        _P, _I, _I64, _P, _I64, _I64, _P,
        _I, _I, _I, _I, _I, _I, _F, _F, _I, _P]),
    "helm_kv_append": (_I, [
        _P, _I64, _I64, _P, _I64, _I64, _P, _I64, _I64,   # q, k, v
        _P, _P, _F,                                       # norm weights, eps
        _P, _P, _I64,                                     # cos, sin, stride
        _P, _I64, _I64, _P, _P,                           # q_out, k_out, v_out
        _P, _I64, _P,                                     # pool, pool_pages, slot_rows
        _I, _I, _I, _I, _I, _I, _P]),
    "helm_copy_pages": (_I, [_P, _P, _I64, _P, _P, _I64, _P]),
    "helm_gather_kv": (_I, [_P, _I64, _P, _I64, _I, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
    "helm_paged_prefill_workspace_bytes": (_I64, [_I, _I, _I, _I, _I, _I, _I]),
    "helm_paged_prefill_attention": (_I, [
        _P, _I64, _I64, _I64,      # q, strides (b, h, s)
        _P, _I64,                  # pool, pool_pages
        _P, _I64, _I,              # page_table, pt_stride_b, max_pages
        _P, _P,                    # kv_lens, kv_starts
        _P, _I, _I64, _I64,        # mask, mask_dtype, mask strides (b, q)
        _P, _I64, _I64, _I64,      # out, strides (b, h, s)
        _P, _I64,                  # workspace, bytes
        _I, _I, _I, _I, _I, _I,    # batch, q_len, hq, hkv, head_dim, page_size
        _I, _I, _F, _F, _I, _P]),  # dtype, causal, scale, softcap, max_kv_len, stream
    "helm_merge_attention_states": (_I, [_P, _I, _I64, _P, _I64, _I, _I64, _I, _P, _I, _P, _P]),
    "helm_decode_gemv": (_I, [_P, _I64, _P, _F, _P, _P, _I64, _I64, _P, _I64, _P, _I64, _I, _I,
                              _I, _P]),
    "helm_decode_gemv_allreduce": (_I, [_P, _I, _I, _P, _I64, _P, _I64, _I64, _P, _I64, _P,
                                        _I64, _I, _I, ctypes.c_uint64, _P]),
    "helm_decode_gemv_allreduce_bytes": (_I64, [_I64, _I, _I]),
    "helm_peer_exchange_bytes": (_I64, [_I64, _I, _I]),
    "helm_ipc_alloc": (_I, [_I64, ctypes.POINTER(_P)]),
    "helm_ipc_free": (_I, [_P]),
    "helm_ipc_zero": (_I, [_P, _I64, _P]),
    "helm_ipc_handle_bytes": (_I, []),
    "helm_ipc_get_handle": (_I, [_P, _P]),
    "helm_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "helm_ipc_close": (_I, [_P]),
    "helm_seq_exchange_merge": (_I, [_P, _I, _I, _P, _P, _I64, _I, _P, _I, _P,
                                     ctypes.c_uint64, _P]),
}

_lib = None
_lib_lock = threading.Lock()


class HelmError(RuntimeError):
    """A helm_b200 C-ABI call returned a non-zero status."""


def library_path() -> str:
    return _build.LIB_PATH


def lib() -> ctypes.CDLL:
    """Loads libhelm_b200.so (building it first if its sources changed and
    nvcc is available).  Raises if the library cannot be loaded."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is None:
            path = _build.LIB_PATH
            if _build.needs_build():
                try:
                    _build.build()
                except Exception as exc:  # noqa: BLE001 - re-raised below with context
                    if not os.path.exists(path):
                        raise HelmError(f"helm_b200 native library is not built and the build "
                                        f"failed: {exc}") from exc
            if not os.path.exists(path):
                raise HelmError(f"helm_b200 native library not found at {path}; "
                                f"run `python -m helm_b200.build`")
            handle = ctypes.CDLL(path)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def _check(rc: int, what: str) -> None:
    if rc != HELM_OK:
        L = lib()
        msg = L.helm_status_string(rc).decode()
        cuda = L.helm_last_cuda_error().decode()
        raise HelmError(f"{what}: {msg}" + (f" ({cuda})" if cuda and rc == 3 else ""))


def helm_dtype(dt: torch.dtype) -> int:
    try:
        return _TORCH_TO_HELM[dt]
    except KeyError:
        raise HelmError(f"unsupported dtype {dt}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream_handle(device: torch.device, stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream(device)
    return s.cuda_stream


def device_status(device: torch.device, reset: bool = True, stream=None) -> int:
    """Synchronises `stream` and returns the device status word (HELM_DEV_* bits).
    A non-zero word also zeroes the decode workspace."""
    out = ctypes.c_uint(0)
    with torch.cuda.device(device):
        _check(lib().helm_get_device_status(ctypes.byref(out), int(reset),
                                            _stream_handle(device, stream)),
               "helm_get_device_status")
    if out.value:
        reset_workspace(device)
    return out.value


# ------------------------------------------------------------------ workspace --
class _Workspace:
    """Per-device scratch of the decode kernel (fp32 split-KV partials; needs
    no initialisation).  Grows, never shrinks."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        return self.buf


_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.type, device.index)
    ws = _workspaces.get(key)
    if ws is None:
        ws = _workspaces[key] = _Workspace()
    return ws.get(device, nbytes)


def reset_workspace(device: torch.device) -> None:
    """Zeroes the workspace (nothing depends on it; kept for callers that
    clean up after an error)."""
    ws = _workspaces.get((device.type, device.index))
    if ws is not None and ws.buf is not None:
        ws.buf.zero_()


_ws_bytes_cache: dict = {}


def decode_workspace_bytes(device: torch.device, batch: int, hq: int, hkv: int, d: int) -> int:
    """Workspace bytes of a decode call (depends on the device's SM count: cached)."""
    key = (device.index, batch, hq, hkv, d)
    v = _ws_bytes_cache.get(key)
    if v is None:
        with torch.cuda.device(device):
            v = _ws_bytes_cache[key] = int(lib().helm_paged_decode_workspace_bytes(batch, hq, hkv,
                                                                                  d))
    return v


class _on_device:
    """torch.cuda.device(dev), skipped when dev is current already (the common
    case; entering the context costs several microseconds per call)."""
    __slots__ = ("dev", "ctx")

    def __init__(self, dev: torch.device):
        self.dev = dev
        self.ctx = None

    def __enter__(self):
        if torch.cuda.current_device() != self.dev.index:
            self.ctx = torch.cuda.device(self.dev)
            self.ctx.__enter__()
        return self

    def __exit__(self, *exc):
        if self.ctx is not None:
            self.ctx.__exit__(*exc)
        return False


# ------------------------------------------------------------------- wrappers --
def paged_decode_attention(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor,
                           kv_lens: torch.Tensor, *, num_kv_heads: int, page_size: int,
                           scale: float, softcap: Optional[float] = None,
                           mask: Optional[torch.Tensor] = None,
                           num_pages: Optional[torch.Tensor] = None,
                           page_used: Optional[torch.Tensor] = None,
                           page_start: Optional[torch.Tensor] = None,
                           out: Optional[torch.Tensor] = None,
                           lse: Optional[torch.Tensor] = None,
                           max_kv_len_hint: int = 0, stream=None):
    """Decode attention over a page pool.

    q [B, Hq, D] (dim stride 1); pool [slots, 2, Hkv, P, D]; page_table int32
    [B, max_pages]; kv_lens int32 [B]; mask additive [B, T] (or None).
    Returns (out [B, Hq, D] in q.dtype, lse fp32 [B, Hq] or None).
    """
    if q.device.type != "cuda":
        raise HelmError("paged_decode_attention runs on CUDA tensors only")
    B, Hq, D = q.shape
    if q.stride(2) != 1:
        raise HelmError("q must have a unit stride on the head dim")
    if pool.dtype != q.dtype:
        raise HelmError(f"KV pool dtype {pool.dtype} != query dtype {q.dtype}")
    if page_table.dtype != torch.int32 or kv_lens.dtype != torch.int32:
        raise HelmError("page_table and kv_lens must be int32")
    if page_table.stride(1) != 1:
        raise HelmError("page_table rows must be contiguous")
    dev = q.device
    if out is None:
        out = torch.empty(B, Hq, D, dtype=q.dtype, device=dev)
    if out.dtype not in (q.dtype, torch.float32) or out.stride(2) != 1:
        raise HelmError("out must be [B, Hq, D] in the query dtype or fp32, unit dim stride")
    ws_bytes = decode_workspace_bytes(dev, B, Hq, num_kv_heads, D)
    ws = _workspace(dev, ws_bytes)
    mask_ptr, mask_dt, mask_sb = None, 0, 0
    if mask is not None:
        if mask.stride(-1) != 1:
            mask = mask.contiguous()
        mask_ptr, mask_dt = mask.data_ptr(), helm_dtype(mask.dtype)
        mask_sb = mask.stride(0) if mask.shape[0] > 1 else 0
    with _on_device(dev):
        rc = lib().helm_paged_decode_attention(
            q.data_ptr(), q.stride(0), q.stride(1),
            pool.data_ptr(), pool.shape[0],
            page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
            kv_lens.data_ptr(), _ptr(num_pages), _ptr(page_used), _ptr(page_start),
            mask_ptr, mask_dt, mask_sb,
            out.data_ptr(), out.stride(0), out.stride(1), _ptr(lse),
            ws.data_ptr(), ws.numel(),
            B, Hq, num_kv_heads, D, page_size, helm_dtype(q.dtype), helm_dtype(out.dtype),
            float(scale), float(softcap or 0.0), int(max_kv_len_hint),
            _stream_handle(dev, stream))
    _check(rc, "helm_paged_decode_attention")
    return out, lse


def paged_prefill_attention(q: torch.Tensor, pool: torch.Tensor, page_table: torch.Tensor,
                            kv_lens: torch.Tensor, *, num_kv_heads: int, page_size: int,
                            scale: float, max_kv_len: int, mask: Optional[torch.Tensor] = None,
                            causal: bool = False, softcap: Optional[float] = None,
                            kv_starts: Optional[torch.Tensor] = None,
                            out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Chunk-prefill attention over a page pool (the chunk's K/V already in it).

    q [B, Hq, S, D] (any strides, unit dim stride); pool [slots, 2, Hkv, P, D];
    page_table int32 [B, max_pages]; kv_lens int32 [B] (query i of sequence b
    sits at position kv_lens[b] - S + i); mask additive [B or 1, 1, S, >= T]
    or None; kv_starts int32 [B] or None (sequence b's rows see keys from
    kv_starts[b] on: a left-padding mask as a key range); max_kv_len =
    max(kv_lens).  Returns out [B, Hq, S, D] in q.dtype, a view of a
    [B, S, Hq, D] buffer unless `out` is given.
    """
    if q.device.type != "cuda":
        raise HelmError("paged_prefill_attention runs on CUDA tensors only")
    B, Hq, S, D = q.shape
    if q.stride(3) != 1:
        raise HelmError("q must have a unit stride on the head dim")
    if pool.dtype != q.dtype:
        raise HelmError(f"KV pool dtype {pool.dtype} != query dtype {q.dtype}")
    if page_table.dtype != torch.int32 or kv_lens.dtype != torch.int32:
        raise HelmError("page_table and kv_lens must be int32")
    if page_table.stride(1) != 1:
        raise HelmError("page_table rows must be contiguous")
    if kv_starts is not None and (kv_starts.dtype != torch.int32 or kv_starts.numel() != B
                                  or not kv_starts.is_contiguous()):
        raise HelmError("kv_starts must be a contiguous int32 tensor of one entry per sequence")
    dev = q.device
    if out is None:
        out = torch.empty(B, S, Hq, D, dtype=q.dtype, device=dev).transpose(1, 2)
    if out.dtype != q.dtype or out.shape != q.shape or out.stride(3) != 1:
        raise HelmError("out must be [B, Hq, S, D] in the query dtype, unit dim stride")
    mask_ptr, mask_dt, mask_sb, mask_sq = None, 0, 0, 0
    if mask is not None:
        if mask.dim() != 4 or mask.shape[2] != S or mask.shape[3] < max_kv_len:
            raise HelmError("mask must be [B or 1, 1, S, >= max_kv_len]")
        if mask.stride(-1) != 1:
            mask = mask.contiguous()
        mask_ptr, mask_dt = mask.data_ptr(), helm_dtype(mask.dtype)
        mask_sb = mask.stride(0) if mask.shape[0] > 1 else 0
        mask_sq = mask.stride(2)
    dt = helm_dtype(q.dtype)
    with _on_device(dev):
        ws_bytes = int(lib().helm_paged_prefill_workspace_bytes(B, S, Hq, num_kv_heads, D, dt,
                                                                int(max_kv_len)))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        rc = lib().helm_paged_prefill_attention(
            q.data_ptr(), q.stride(0), q.stride(1), q.stride(2),
            pool.data_ptr(), pool.shape[0],
            page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
            kv_lens.data_ptr(), None if kv_starts is None else kv_starts.data_ptr(),
            mask_ptr, mask_dt, mask_sb, mask_sq,
            out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
            ws.data_ptr(), ws_bytes,
            B, S, Hq, num_kv_heads, D, page_size, dt, 1 if causal else 0,
            float(scale), float(softcap or 0.0), int(max_kv_len),
            _stream_handle(dev, stream))
    _check(rc, "helm_paged_prefill_attention")
    return out


def prefill_supported(dtype: torch.dtype, head_dim: int, page_size: int) -> bool:
    """Shapes helm_paged_prefill_attention serves (others return UNSUPPORTED)."""
    return (dtype in (torch.bfloat16, torch.float16) and head_dim in (64, 128)
            and page_size % 16 == 0)


def kv_append(*, k: torch.Tensor, v: torch.Tensor, pool: Optional[torch.Tensor],
              slot_rows: Optional[torch.Tensor], page_size: int,
              q: Optional[torch.Tensor] = None, q_out: Optional[torch.Tensor] = None,
              q_norm_w: Optional[torch.Tensor] = None, k_norm_w: Optional[torch.Tensor] = None,
              eps: float = 1e-6, cos: Optional[torch.Tensor] = None,
              sin: Optional[torch.Tensor] = None, k_out: Optional[torch.Tensor] = None,
              v_out: Optional[torch.Tensor] = None, stream=None) -> None:
    """Fused (QK-RMSNorm, RoPE, page write).  Token-major views:
    q [N, Hq, D], k/v [N, Hkv, D] (unit dim stride), cos/sin [N, D],
    slot_rows int64 [N] (pool row = slot*page_size + row, -1 = skip)."""
    N, Hkv, D = k.shape
    Hq = q.shape[1] if q is not None else 0
    dev = k.device
    for name, t in (("k", k), ("v", v), ("q", q), ("q_out", q_out)):
        if t is not None and t.stride(-1) != 1:
            raise HelmError(f"{name} must have a unit stride on the head dim")
    if cos is not None and cos.stride(-1) != 1:
        raise HelmError("cos/sin must have a unit stride on the head dim")
    if slot_rows is not None and slot_rows.dtype != torch.int64:
        raise HelmError("slot_rows must be int64")
    with _on_device(dev):
        rc = lib().helm_kv_append(
            _ptr(q), q.stride(0) if q is not None else 0, q.stride(1) if q is not None else 0,
            k.data_ptr(), k.stride(0), k.stride(1),
            v.data_ptr(), v.stride(0), v.stride(1),
            _ptr(q_norm_w), _ptr(k_norm_w), float(eps),
            _ptr(cos), _ptr(sin), cos.stride(0) if cos is not None else 0,
            _ptr(q_out), q_out.stride(0) if q_out is not None else 0,
            q_out.stride(1) if q_out is not None else 0,
            _ptr(k_out), _ptr(v_out),
            _ptr(pool), pool.shape[0] if pool is not None else 0, _ptr(slot_rows),
            N, Hq, Hkv, D, page_size, helm_dtype(k.dtype), _stream_handle(dev, stream))
    _check(rc, "helm_kv_append")


def copy_pages(dst_pool: torch.Tensor, src_pool: torch.Tensor, dst_slots, src_slots,
               device: torch.device, stream=None) -> None:
    """dst_pool[dst_slots[i]] = src_pool[src_slots[i]] on `stream` (copy engine)."""
    n = len(dst_slots)
    if n != len(src_slots):
        raise HelmError("slot lists differ in length")
    if n == 0:
        return
    page_bytes = dst_pool[0].numel() * dst_pool.element_size()
    if src_pool[0].numel() * src_pool.element_size() != page_bytes:
        raise HelmError("page size differs between pools")
    dst = (ctypes.c_int64 * n)(*dst_slots)
    src = (ctypes.c_int64 * n)(*src_slots)
    with torch.cuda.device(device):
        rc = lib().helm_copy_pages(dst_pool.data_ptr(), src_pool.data_ptr(), page_bytes,
                                   dst, src, n, _stream_handle(device, stream))
    _check(rc, "helm_copy_pages")


def gather_kv(pool: torch.Tensor, page_table: torch.Tensor, kv_lens: torch.Tensor, t_max: int,
              *, num_kv_heads: int, page_size: int, stream=None):
    """Dense K, V [B, Hkv, t_max, D] from the page pool (zero beyond kv_lens)."""
    B = page_table.shape[0]
    D = pool.shape[-1]
    dev = pool.device
    k = torch.empty(B, num_kv_heads, t_max, D, dtype=pool.dtype, device=dev)
    v = torch.empty_like(k)
    with _on_device(dev):
        rc = lib().helm_gather_kv(pool.data_ptr(), pool.shape[0], page_table.data_ptr(),
                                  page_table.stride(0), page_table.shape[1], kv_lens.data_ptr(),
                                  k.data_ptr(), v.data_ptr(), B, num_kv_heads, D, page_size,
                                  t_max, helm_dtype(pool.dtype), _stream_handle(dev, stream))
    _check(rc, "helm_gather_kv")
    return k, v


def merge_attention_states(o_parts: torch.Tensor, lse_parts: torch.Tensor,
                           out_dtype: torch.dtype, stream=None):
    """o_parts [R, ..., D] (rows contiguous within a part, any part stride),
    lse_parts fp32 [R, ...] -> (out [..., D] in out_dtype, lse fp32 [...])."""
    R = o_parts.shape[0]
    D = o_parts.shape[-1]
    rows = lse_parts[0].numel()
    if o_parts[0].numel() != rows * D or not o_parts[0].is_contiguous():
        raise HelmError("each part of o_parts must be a contiguous [rows, D] block")
    if lse_parts.dtype != torch.float32 or not lse_parts[0].is_contiguous():
        raise HelmError("lse_parts must be fp32 with contiguous parts")
    dev = o_parts.device
    out = torch.empty(o_parts.shape[1:], dtype=out_dtype, device=dev)
    lse = torch.empty(lse_parts.shape[1:], dtype=torch.float32, device=dev)
    with _on_device(dev):
        rc = lib().helm_merge_attention_states(
            o_parts.data_ptr(), helm_dtype(o_parts.dtype), o_parts.stride(0),
            lse_parts.data_ptr(), lse_parts.stride(0), R, rows, D,
            out.data_ptr(), helm_dtype(out_dtype), lse.data_ptr(), _stream_handle(dev, stream))
    _check(rc, "helm_merge_attention_states")
    return out, lse


# ── peer-memory exchange (sequence split) ─────────────────────────────────────
def peer_exchange_bytes(rows: int, head_dim: int, world: int) -> int:
    n = lib().helm_peer_exchange_bytes(rows, head_dim, world)
    if n < 0:
        raise HelmError(f"unsupported exchange geometry rows={rows} head_dim={head_dim} "
                        f"world={world}")
    return int(n)


def ipc_alloc(nbytes: int, device: torch.device) -> int:
    p = ctypes.c_void_p()
    with torch.cuda.device(device):
        _check(lib().helm_ipc_alloc(nbytes, ctypes.byref(p)), "helm_ipc_alloc")
    return int(p.value)


def ipc_free(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _check(lib().helm_ipc_free(ptr), "helm_ipc_free")


def ipc_zero(ptr: int, nbytes: int, device: torch.device, stream=None) -> None:
    with torch.cuda.device(device):
        _check(lib().helm_ipc_zero(ptr, nbytes, _stream_handle(device, stream)), "helm_ipc_zero")


def ipc_get_handle(ptr: int, device: torch.device) -> bytes:
    buf = ctypes.create_string_buffer(lib().helm_ipc_handle_bytes())
    with torch.cuda.device(device):
        _check(lib().helm_ipc_get_handle(ptr, buf), "helm_ipc_get_handle")
    return buf.raw


def ipc_open(handle: bytes, device: torch.device) -> int:
    p = ctypes.c_void_p()
    with torch.cuda.device(device):
        _check(lib().helm_ipc_open(handle, ctypes.byref(p)), "helm_ipc_open")
    return int(p.value)


def ipc_close(ptr: int, device: torch.device) -> None:
    with torch.cuda.device(device):
        _check(lib().helm_ipc_close(ptr), "helm_ipc_close")


def seq_exchange_merge(bufs: list, rank: int, o_part: torch.Tensor, lse_part: torch.Tensor,
                       out: torch.Tensor, lse_out: Optional[torch.Tensor] = None,
                       timeout_s: float = 5.0, stream=None) -> None:
    """Exchange + merge of partial states over peer memory: o_part fp32
    [rows, D], lse_part fp32 [rows] -> out [rows, D] (its dtype), lse_out."""
    D = o_part.shape[-1]
    rows = lse_part.numel()
    if o_part.dtype != torch.float32 or lse_part.dtype != torch.float32:
        raise HelmError("partial states must be fp32")
    if not (o_part.is_contiguous() and lse_part.is_contiguous() and out.is_contiguous()):
        raise HelmError("o_part, lse_part and out must be contiguous")
    if o_part.numel() != rows * D or out.numel() != rows * D:
        raise HelmError("o_part / out must hold rows * head_dim elements")
    if lse_out is not None and (lse_out.dtype != torch.float32 or lse_out.numel() != rows):
        raise HelmError("lse_out must be fp32 [rows]")
    dev = o_part.device
    arr = (ctypes.c_void_p * len(bufs))(*bufs)
    with _on_device(dev):
        rc = lib().helm_seq_exchange_merge(arr, rank, len(bufs), o_part.data_ptr(),
                                           lse_part.data_ptr(), rows, D, out.data_ptr(),
                                           helm_dtype(out.dtype), _ptr(lse_out),
                                           int(timeout_s * 1e9), _stream_handle(dev, stream))
    _check(rc, "helm_seq_exchange_merge")


def set_decode_overlap(enable: bool) -> bool:
    """Decode overlap for calls made from this thread (see include/helm_b200.h);
    returns the previous setting."""
    return bool(lib().helm_set_decode_overlap(1 if enable else 0))


class decode_overlap:
    """Context manager: decode overlap on (or off) inside the block."""

    def __init__(self, enable: bool = True):
        self.enable = enable
        self.prev = False

    def __enter__(self):
        self.prev = set_decode_overlap(self.enable)
        return self

    def __exit__(self, *exc):
        set_decode_overlap(self.prev)
        return False


def decode_gemv(x: torch.Tensor, w: torch.Tensor, *, out: torch.Tensor,
                norm_w: Optional[torch.Tensor] = None, eps: float = 1e-6,
                w2: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                stream=None) -> torch.Tensor:
    """out[b] = W . f(x[b]) with the fused RMSNorm / SwiGLU / residual of
    helm_decode_gemv.  x [B, K] (unit inner stride), w (and w2) [N, K]
    contiguous, out [B, N] (model dtype or fp32), residual [B, N] or None."""
    B, K = x.shape
    N = w.shape[0]
    if x.stride(1) != 1 or not w.is_contiguous() or (w2 is not None and not w2.is_contiguous()):
        raise HelmError("decode_gemv: x needs a unit inner stride, weights must be contiguous")
    if w.shape[1] != K or out.shape[0] != B or out.shape[1] != N or out.stride(1) != 1:
        raise HelmError("decode_gemv: shape mismatch")
    if residual is not None and (residual.shape != out.shape or residual.stride(1) != 1):
        raise HelmError("decode_gemv: residual must match out")
    dev = x.device
    with _on_device(dev):
        rc = lib().helm_decode_gemv(
            x.data_ptr(), x.stride(0), _ptr(norm_w), float(eps), w.data_ptr(), _ptr(w2), N, K,
            _ptr(residual), residual.stride(0) if residual is not None else 0,
            out.data_ptr(), out.stride(0), 1 if out.dtype == torch.float32 else 0, B,
            helm_dtype(x.dtype), _stream_handle(dev, stream))
    _check(rc, "helm_decode_gemv")
    return out


def decode_gemv_allreduce_bytes(n: int, batch: int, world: int) -> int:
    v = lib().helm_decode_gemv_allreduce_bytes(n, batch, world)
    if v < 0:
        raise HelmError("unsupported all-reduce geometry")
    return int(v)


def decode_gemv_allreduce(bufs: list, rank: int, x: torch.Tensor, w: torch.Tensor, *,
                          out: torch.Tensor, residual: Optional[torch.Tensor] = None,
                          timeout_s: float = 5.0, stream=None) -> torch.Tensor:
    """Row-parallel projection with its all-reduce: out[b] = residual[b] +
    sum over ranks of W_r x_r[b] (this rank's W_r [N, K_r], x_r [B, K_r]).
    bufs: every rank's exchange buffer mapped here (decode_gemv_allreduce_bytes)."""
    B, K = x.shape
    N = w.shape[0]
    if x.stride(1) != 1 or not w.is_contiguous() or w.shape[1] != K:
        raise HelmError("decode_gemv_allreduce: x [B, K] unit inner stride, w [N, K] contiguous")
    if out.shape != (B, N) or out.stride(1) != 1 or out.dtype != x.dtype:
        raise HelmError("decode_gemv_allreduce: out must be [B, N] in the model dtype")
    if residual is not None and (residual.shape != out.shape or residual.stride(1) != 1):
        raise HelmError("decode_gemv_allreduce: residual must match out")
    dev = x.device
    arr = (ctypes.c_void_p * len(bufs))(*bufs)
    with _on_device(dev):
        rc = lib().helm_decode_gemv_allreduce(
            arr, rank, len(bufs), x.data_ptr(), x.stride(0), w.data_ptr(), N, K, _ptr(residual),
            residual.stride(0) if residual is not None else 0, out.data_ptr(), out.stride(0), B,
            helm_dtype(x.dtype), int(timeout_s * 1e9), _stream_handle(dev, stream))
    _check(rc, "helm_decode_gemv_allreduce")
    return out


def gemv_max_batch(k: int, elem: int = 2) -> int:
    """Largest batch (<= 16) helm_decode_gemv stages for input width k: x of
    every batch row plus the weight-stream ring must fit in shared memory."""
    for nb in (16, 8, 4, 2, 1):
        threads = 512 if nb == 1 else 256
        ring = 128 if nb >= 8 or nb == 1 else 256
        stride = k if nb == 1 else k + 8
        static = 4 * (threads // 32) * 16 * nb * 2 + 1024
        nw = (k * elem + 127) // 128 * 128 if nb == 1 else 0   # prefetched norm weight
        if (nb * stride * elem + 127) // 128 * 128 + nw + threads * ring + static <= 224 * 1024:
            return nb
    raise HelmError(f"input width {k} too large for decode_gemv")
