"""Parity of the fused KV append kernel (csrc/kv_append.cu) through the C ABI.

The kernel replaces, in one launch per layer, the eager q_norm / k_norm /
apply_rotary_pos_emb of HELM's patched Qwen3 attention forward
(helm/runtime/kv_offload.py:368-373) and the page copy_ of
KVCacheManager.append_decode / append_prefill (helm/runtime/kv_cache.py:113-171);
for Llama (kv_offload.py:467-519) only RoPE and the page write.

Pins and tolerances:
  * HF's own Qwen3RMSNorm + apply_rotary_pos_emb outputs (tests/golden/norm_rope.npz,
    written by tests/golden/make_golden.py from transformers): Q and K within
    2 ulp of the model dtype, more than 99 % of elements bit-identical (for the
    RoPE outputs, 2 ulp of the larger of the result and its two rounded terms:
    the fp32 variance sum and rsqrt may land on the other side of a rounding
    boundary, and a one-ulp difference before RoPE stays one ulp of the terms).
  * The oracle restatement (oracle/norm_rope.py) at the head shapes of
    BASELINE configs 1 (Qwen3-0.6B: 16 q / 8 KV heads), 4 (Qwen3-14B: 40 / 8)
    and 5 (Llama-2-13B, fp16, no QK-norm, theta 1e4: 40 / 40), for decode rows
    (one token per sequence) and prefill rows (a chunk of consecutive
    positions), pages of 16 and 64 tokens: same 2 ulp / 99 % bar.
  * V is copied bit for bit.
  * Placement: the pool is filled with a NaN bit pattern first; each token's
    K and V rows land at exactly pool row slot * page_size + r of their head,
    and every other pool element keeps its NaN bits (no stray writes).
"""
import zlib

import numpy as np
import pytest
import torch

from oracle import norm_rope

pytestmark = pytest.mark.gpu

SENTINEL = 0x7FC1  # a NaN in both bf16 and fp16


def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


def _ulp_ok(got, ref, dtype, tag, mag=None):
    """|got - ref| <= 2 ulp of `mag` (default |ref|) in the model dtype, and more
    than 99 % of elements bit-identical.  For RoPE outputs `mag` is the size
    of the two rounded terms, |z cos| + |rotate_half(z) sin|: when they
    cancel, one ulp of difference in z (the fp32 variance sum or rsqrt landing
    on the other side of a rounding boundary) is many ulps of the result."""
    mag = np.abs(ref) if mag is None else np.maximum(np.abs(ref), mag)
    ulp = mag * (2 ** -7 if dtype == "bfloat16" else 2 ** -10) + 1e-6
    bad = np.abs(got - ref) > 2 * ulp
    assert not bad.any(), f"{tag}: {bad.sum()} elements beyond 2 ulp, max |d| " \
                          f"{np.abs(got - ref).max()}"
    exact = np.mean(got == ref)
    assert exact > 0.99, f"{tag}: only {exact:.4f} bit-identical"


def _rope_mag(z, cos, sin):
    """|z cos| + |rotate_half(z) sin| for z [N, H, D], cos/sin [N, D]."""
    half = z.shape[-1] // 2
    rot = np.concatenate([-z[..., half:], z[..., :half]], axis=-1)
    return np.abs(z * cos[:, None, :]) + np.abs(rot * sin[:, None, :])


def _bits_to_f32(bits, dtype):
    bits = np.asarray(bits, np.uint16)
    if dtype == "float16":
        return bits.view(np.float16).astype(np.float32)
    return norm_rope.bf16_bits_to_f32(bits)


def _to_dev(arr_f32, dtype, dev):
    return torch.from_numpy(np.ascontiguousarray(arr_f32, np.float32)).to(
        getattr(torch, dtype)).to(dev)


def _run_append(dev, dtype, q, k, v, qw, kw, cos, sin, slot_rows, pool_pages, page_size,
                with_kv_out=False, q_strided=False):
    """q [N, Hq, D], k/v [N, Hkv, D], cos/sin [N, D] float32 arrays holding
    dtype values; slot_rows int64 [N].  Returns (q_out, pool bits, k_out, v_out)."""
    from helm_b200 import _capi
    N, Hq, D = q.shape
    Hkv = k.shape[1]
    td = getattr(torch, dtype)
    if q_strided:
        # q, k and v as column blocks of one fused projection output [N, (Hq + 2 Hkv) * D],
        # the layout the decode stage's q/k/v GEMV writes
        qkv = torch.empty(N, (Hq + 2 * Hkv) * D, dtype=td, device=dev)
        qkv[:, :Hq * D] = _to_dev(q.reshape(N, -1), dtype, dev)
        qkv[:, Hq * D:(Hq + Hkv) * D] = _to_dev(k.reshape(N, -1), dtype, dev)
        qkv[:, (Hq + Hkv) * D:] = _to_dev(v.reshape(N, -1), dtype, dev)
        qt = qkv[:, :Hq * D].view(N, Hq, D)
        kt = qkv[:, Hq * D:(Hq + Hkv) * D].view(N, Hkv, D)
        vt = qkv[:, (Hq + Hkv) * D:].view(N, Hkv, D)
    else:
        qt, kt, vt = (_to_dev(a, dtype, dev) for a in (q, k, v))
    pool = torch.full((pool_pages, 2, Hkv, page_size, D), SENTINEL, dtype=torch.int16,
                      device=dev).view(td)
    q_out = torch.full((N, Hq, D), SENTINEL, dtype=torch.int16, device=dev).view(td)
    k_out = torch.empty(N, Hkv, D, dtype=td, device=dev) if with_kv_out else None
    v_out = torch.empty(N, Hkv, D, dtype=td, device=dev) if with_kv_out else None
    _capi.kv_append(q=qt, k=kt, v=vt, q_out=q_out,
                    q_norm_w=None if qw is None else _to_dev(qw, dtype, dev),
                    k_norm_w=None if kw is None else _to_dev(kw, dtype, dev),
                    eps=1e-6, cos=_to_dev(cos, dtype, dev), sin=_to_dev(sin, dtype, dev),
                    pool=pool, slot_rows=torch.from_numpy(np.asarray(slot_rows, np.int64)).to(dev),
                    page_size=page_size, k_out=k_out, v_out=v_out)
    torch.cuda.synchronize()
    assert _capi.device_status(dev) == 0
    qo = q_out.float().cpu().numpy()
    pool_bits = pool.view(torch.int16).cpu().numpy().view(np.uint16)
    ko = k_out.float().cpu().numpy() if with_kv_out else None
    vo = v_out.float().cpu().numpy() if with_kv_out else None
    return qo, pool_bits, ko, vo


def _check_pool(pool_bits, k_ref, v_in, slot_rows, page_size, dtype, tag, k_mag=None):
    """K rows within 2 ulp (of k_mag), V rows bit-exact, nothing else written."""
    N, Hkv, D = k_ref.shape
    written = np.zeros(pool_bits.shape, bool)
    k_got = np.zeros_like(k_ref)
    for t, row in enumerate(slot_rows):
        if row < 0:
            continue
        slot, r = divmod(int(row), page_size)
        written[slot, :, :, r, :] = True
        k_got[t] = _bits_to_f32(pool_bits[slot, 0, :, r, :], dtype)
        v_got = _bits_to_f32(pool_bits[slot, 1, :, r, :], dtype)
        assert np.array_equal(v_got.view(np.uint32), v_in[t].astype(np.float32).view(np.uint32)), \
            f"{tag}: V row of token {t} is not bit-identical"
    live = np.asarray(slot_rows) >= 0
    _ulp_ok(k_got[live], k_ref[live], dtype, tag + " K",
            None if k_mag is None else k_mag[live])
    assert np.all(pool_bits[~written] == SENTINEL), f"{tag}: pool written outside the target rows"


def _scattered_rows(rng, n, pool_pages, page_size, consecutive):
    """Pool rows for n tokens: consecutive positions fill pages in order (a
    prefill chunk, pages drawn from a permutation of the pool); otherwise one
    row in each of n distinct random pages (decode rows of n sequences)."""
    if consecutive:
        pages = rng.permutation(pool_pages)[: -(-n // page_size) + 1]
        first = int(rng.integers(0, page_size))  # the chunk starts mid-page
        idx = np.arange(n) + first
        return pages[idx // page_size] * page_size + idx % page_size
    pages = rng.permutation(pool_pages)[:n]
    return pages * page_size + rng.integers(0, page_size, size=n)


def test_append_matches_hf_golden(norm_rope_golden):
    """HF's Qwen3RMSNorm + apply_rotary_pos_emb outputs, with HF's own cos/sin."""
    dev = _cuda()
    z = norm_rope_golden
    rng = np.random.default_rng(7)
    for tag in sorted({k.split("/")[0] for k in z.files}):
        dtype = "float16" if tag.startswith("float16") else "bfloat16"
        conv = (lambda a: _bits_to_f32(a, dtype))
        q, k = conv(z[tag + "/q"]), conv(z[tag + "/k"])
        N, Hkv, D = k.shape
        v = norm_rope.round_to(rng.standard_normal((N, Hkv, D)).astype(np.float32), dtype)
        cos, sin = conv(z[tag + "/cos"]), conv(z[tag + "/sin"])
        q_mag = _rope_mag(norm_rope.rms_norm(q, conv(z[tag + "/qw"]), 1e-6, dtype), cos, sin)
        k_mag = _rope_mag(norm_rope.rms_norm(k, conv(z[tag + "/kw"]), 1e-6, dtype), cos, sin)
        for page_size in (16, 64):
            pool_pages = 2 * N + 3
            rows = _scattered_rows(rng, N, pool_pages, page_size, consecutive=False)
            qo, pool_bits, ko, vo = _run_append(
                dev, dtype, q, k, v, conv(z[tag + "/qw"]), conv(z[tag + "/kw"]),
                conv(z[tag + "/cos"]), conv(z[tag + "/sin"]), rows, pool_pages, page_size,
                with_kv_out=True)
            _ulp_ok(qo, conv(z[tag + "/q_out"]), dtype, f"{tag} P{page_size} Q", q_mag)
            _ulp_ok(ko, conv(z[tag + "/k_out"]), dtype, f"{tag} P{page_size} k_out", k_mag)
            assert np.array_equal(vo, v), tag
            _check_pool(pool_bits, conv(z[tag + "/k_out"]), v, rows, page_size, dtype,
                        f"{tag} P{page_size}", k_mag)


# (name, Hq, Hkv, D, dtype, theta, qk_norm)
SHAPES = [
    ("config1_qwen3_0.6b", 16, 8, 128, "bfloat16", 1e6, True),
    ("config4_qwen3_14b", 40, 8, 128, "bfloat16", 1e6, True),
    ("config5_llama2_13b", 40, 40, 128, "float16", 1e4, False),
    ("d256_no_norm", 8, 4, 256, "bfloat16", 1e4, False),
    ("d64_gqa", 8, 2, 64, "float16", 1e6, True),
]


@pytest.mark.parametrize("shape", SHAPES, ids=[s[0] for s in SHAPES])
@pytest.mark.parametrize("page_size", [16, 64])
@pytest.mark.parametrize("mode", ["decode", "prefill"])
def test_append_matches_oracle(shape, page_size, mode):
    dev = _cuda()
    name, Hq, Hkv, D, dtype, theta, qk_norm = shape
    rng = np.random.default_rng(zlib.crc32(f"{name}/{page_size}/{mode}".encode()))
    if mode == "decode":
        N = 16
        positions = rng.integers(0, 131072, size=N)
    else:
        N = 77
        positions = 4000 + np.arange(N)
    pool_pages = 64
    rows = _scattered_rows(rng, N, pool_pages, page_size, consecutive=(mode == "prefill"))
    r = (lambda *s: norm_rope.round_to(rng.standard_normal(s).astype(np.float32) * 0.7, dtype))
    q, k, v = r(N, Hq, D), r(N, Hkv, D), r(N, Hkv, D)
    qw = kw = None
    if qk_norm:
        qw = norm_rope.round_to(1.0 + 0.1 * rng.standard_normal(D).astype(np.float32), dtype)
        kw = norm_rope.round_to(1.0 + 0.1 * rng.standard_normal(D).astype(np.float32), dtype)
    cos, sin = norm_rope.rope_tables(positions, D, theta, dtype)
    qo, pool_bits, _, _ = _run_append(dev, dtype, q, k, v, qw, kw, cos, sin, rows, pool_pages,
                                      page_size, q_strided=(mode == "decode"))
    qn = norm_rope.rms_norm(q, qw, 1e-6, dtype) if qk_norm else q
    kn = norm_rope.rms_norm(k, kw, 1e-6, dtype) if qk_norm else k
    q_ref = norm_rope.rope(qn, cos[:, None, :], sin[:, None, :], dtype)
    k_ref = norm_rope.rope(kn, cos[:, None, :], sin[:, None, :], dtype)
    tag = f"{name} P{page_size} {mode}"
    _ulp_ok(qo, q_ref, dtype, tag + " Q", _rope_mag(qn, cos, sin))
    _check_pool(pool_bits, k_ref, v, rows, page_size, dtype, tag, _rope_mag(kn, cos, sin))


def test_append_skips_negative_rows_and_writes_nothing_else():
    """A slot row of -1 (a padded batch position) leaves the pool untouched
    while the other tokens are still written and q is still produced."""
    dev = _cuda()
    rng = np.random.default_rng(3)
    dtype, N, Hq, Hkv, D, P = "bfloat16", 6, 16, 8, 128, 16
    r = (lambda *s: norm_rope.round_to(rng.standard_normal(s).astype(np.float32), dtype))
    q, k, v = r(N, Hq, D), r(N, Hkv, D), r(N, Hkv, D)
    w = np.ones(D, np.float32)
    cos, sin = norm_rope.rope_tables(np.arange(N) * 1000, D, 1e6, dtype)
    rows = np.array([3 * P + 1, -1, 7 * P + 15, -1, 0, 9 * P + 8], np.int64)
    qo, pool_bits, _, _ = _run_append(dev, dtype, q, k, v, w, w, cos, sin, rows, 12, P)
    k_ref = norm_rope.rope(norm_rope.rms_norm(k, w, 1e-6, dtype), cos[:, None], sin[:, None],
                           dtype)
    q_ref = norm_rope.rope(norm_rope.rms_norm(q, w, 1e-6, dtype), cos[:, None], sin[:, None],
                           dtype)
    _ulp_ok(qo, q_ref, dtype, "padded Q",
            _rope_mag(norm_rope.rms_norm(q, w, 1e-6, dtype), cos, sin))
    _check_pool(pool_bits, k_ref, v, rows, P, dtype, "padded",
                _rope_mag(norm_rope.rms_norm(k, w, 1e-6, dtype), cos, sin))
