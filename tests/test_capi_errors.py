"""Error convention of the C ABI: bad arguments come back as the documented int
status before anything touches a device (no GPU needed).  Pointers here are
placeholders that the library validates but never dereferences on a refused
call."""
import ctypes

from helm_b200 import _capi

OK, INVALID, UNSUPPORTED, WORKSPACE, ALIGN = 0, 1, 2, 4, 5
BF16 = _capi.DTYPE_BF16
P16 = 0x10000  # 16-byte-aligned placeholder address (never dereferenced)


def _decode(**kw):
    a = dict(q=P16, q_sb=4096, q_sh=128, pool=P16, pool_pages=64, pt=P16, pt_sb=19, max_pages=19,
             lens=P16, num_pages=None, page_used=None, page_start=None, mask=None, mask_dtype=0,
             mask_sb=0, out=P16, out_sb=4096, out_sh=128, lse=None, ws=0x100000, ws_bytes=1 << 30,
             batch=2, hq=32, hkv=8, d=128, page=16, dtype=BF16, out_dtype=BF16)
    a.update(kw)
    return _capi.lib().helm_paged_decode_attention(
        a["q"], a["q_sb"], a["q_sh"], a["pool"], a["pool_pages"], a["pt"], a["pt_sb"],
        a["max_pages"], a["lens"], a["num_pages"], a["page_used"], a["page_start"], a["mask"],
        a["mask_dtype"], a["mask_sb"], a["out"], a["out_sb"], a["out_sh"], a["lse"], a["ws"],
        a["ws_bytes"], a["batch"], a["hq"], a["hkv"], a["d"], a["page"], a["dtype"],
        a["out_dtype"], 0.088, 0.0, 0, None)


def _prefill(**kw):
    a = dict(q=P16, q_sb=65536, q_sh=128, q_ss=512, pool=P16, pool_pages=64, pt=P16, pt_sb=19,
             max_pages=19, lens=P16, mask=None, mask_dtype=0, mask_sb=0, mask_sq=0, out=P16,
             o_sb=65536, o_sh=128, o_ss=512, ws=0x100000, ws_bytes=1 << 30, batch=1, S=64, hq=4,
             hkv=2, d=128, page=16, dtype=BF16, causal=1)
    a.update(kw)
    return _capi.lib().helm_paged_prefill_attention(
        a["q"], a["q_sb"], a["q_sh"], a["q_ss"], a["pool"], a["pool_pages"], a["pt"], a["pt_sb"],
        a["max_pages"], a["lens"], None, a["mask"], a["mask_dtype"], a["mask_sb"],
        a["mask_sq"],
        a["out"], a["o_sb"], a["o_sh"], a["o_ss"], a["ws"], a["ws_bytes"], a["batch"], a["S"],
        a["hq"], a["hkv"], a["d"], a["page"], a["dtype"], a["causal"], 0.088, 0.0, 300, None)


def test_decode_attention_refusals():
    assert _decode(q=None) == INVALID
    assert _decode(batch=0) == INVALID
    assert _decode(hq=30) == INVALID            # query heads not a multiple of KV heads
    assert _decode(hq=136) == UNSUPPORTED       # GQA group of 17
    assert _decode(d=96) == UNSUPPORTED
    assert _decode(dtype=_capi.DTYPE_FP32) == UNSUPPORTED
    assert _decode(num_pages=P16) == INVALID    # ragged lists need all three arrays
    assert _decode(mask=P16, mask_dtype=7) == INVALID
    assert _decode(q=P16 + 2) == ALIGN
    assert _decode(pool=P16 + 8) == ALIGN
    assert _decode(ws_bytes=16) == WORKSPACE


def test_prefill_attention_refusals():
    assert _prefill(q=None) == INVALID
    assert _prefill(S=0) == INVALID
    assert _prefill(hq=5) == INVALID
    assert _prefill(d=256) == UNSUPPORTED
    assert _prefill(page=8) == UNSUPPORTED      # 16-key boxes must stay inside a page
    assert _prefill(dtype=_capi.DTYPE_FP32) == UNSUPPORTED
    assert _prefill(mask=P16, mask_dtype=9) == INVALID
    assert _prefill(q=P16 + 2) == ALIGN
    assert _prefill(out=P16 + 4) == ALIGN
    assert _prefill(o_ss=514) == ALIGN
    assert _prefill(max_pages=1 << 28) == UNSUPPORTED  # key positions must fit 30 bits


def test_gemv_refusals():
    lib = _capi.lib()

    def gemv(x=P16, w=P16, y=P16, n=384, k=512, batch=1, dtype=BF16):
        return lib.helm_decode_gemv(x, k, None, ctypes.c_float(1e-6), w, None, n, k, None, 0, y,
                                    n, 0, batch, dtype, None)

    assert gemv(x=None) == INVALID
    assert gemv(n=0) == INVALID
    assert gemv(batch=17) == UNSUPPORTED
    assert gemv(k=520) == UNSUPPORTED            # k must be a multiple of 16
    assert gemv(dtype=_capi.DTYPE_FP32) == UNSUPPORTED


def test_status_strings_cover_codes():
    lib = _capi.lib()
    for code in (OK, INVALID, UNSUPPORTED, 3, WORKSPACE, ALIGN):
        assert lib.helm_status_string(code) != b"unknown status"
    assert lib.helm_status_string(99) == b"unknown status"
