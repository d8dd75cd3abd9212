"""helm_b200 — B200-native paged-KV decode path for HELM.

Drop-in replacements for HELM's ``helm.runtime.kv_allocator``,
``helm.runtime.kv_cache`` and ``helm.runtime.kv_offload`` live in
``helm_b200.runtime``; the CUDA work happens in the native library
``helm_b200/_lib/libhelm_b200.so`` (C ABI: include/helm_b200.h), reached
through ``helm_b200._capi``.
"""
__version__ = "0.1.0"
