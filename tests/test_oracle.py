"""Pins the CPU oracle (oracle/) to the reference's own outputs (tests/golden/).

These run without a GPU.  The oracle is what the GPU tests compare the CUDA
kernels against, so it is first checked here against fixtures produced by
running the HELM reference (tests/golden/make_golden.py).
"""
import numpy as np
import pytest

import oracle
from oracle import merge, norm_rope, placement


def _pool_dtype(case):
    return oracle.DT_F16 if case["dtype"] == "float16" else oracle.DT_BF16


def _to_f32(bits, dtype):
    if dtype == "float16":
        return np.asarray(bits, np.uint16).view(np.float16).astype(np.float32)
    return norm_rope.bf16_bits_to_f32(bits)


def _run_oracle(case, threads=1):
    q = _to_f32(case["q"], case["dtype"])
    return oracle.paged_attention(
        q, case["pool"], _pool_dtype(case), case["page_table"], case["num_pages"],
        case["page_used"], num_kv_heads=case["Hkv"], page_size=case["P"],
        scale=case["scale_f"], softcap=case["softcap_f"], mask=case.get("mask"),
        threads=threads)


def test_oracle_matches_reference_fp32(attention_golden):
    """fp32 restatement vs the reference run in fp32 on the same (exact) inputs."""
    for name, case in attention_golden.items():
        out, _ = _run_oracle(case)
        ref = case["out_fp32"]
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=2e-5, err_msg=name)


def test_oracle_matches_reference_in_model_dtype(attention_golden):
    """Rounded to the query dtype, the oracle reproduces the reference's output
    (the reference casts its fp32 result with out.to(dtype))."""
    for name, case in attention_golden.items():
        out, _ = _run_oracle(case)
        rounded = norm_rope.round_to(out, case["dtype"])
        ref = _to_f32(case["out"], case["dtype"])
        # identical except where fp32 summation order crosses a rounding boundary
        diff = np.abs(rounded - ref)
        ulp = np.abs(ref) * (2 ** -7 if case["dtype"] == "bfloat16" else 2 ** -10) + 1e-6
        assert np.all(diff <= ulp), name
        assert np.mean(diff == 0) > 0.97, name


def test_oracle_threads_agree(attention_golden):
    case = attention_golden["dense_bf16_d128_p16"]
    a, la = _run_oracle(case, threads=1)
    b, lb = _run_oracle(case, threads=4)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(la, lb)


def test_oracle_empty_sequence_is_zero(attention_golden):
    for name in ("no_pages", "zero_used_page"):
        out, lse = _run_oracle(attention_golden[name])
        assert np.all(out == 0), name
        assert np.all(np.isneginf(lse)), name


def test_oracle_lse_is_logsumexp(attention_golden):
    """LSE (not produced by the reference) equals logsumexp of the scores,
    computed independently in float64."""
    case = attention_golden["dense_bf16_mask_softcap"]
    _, lse = _run_oracle(case)
    q = _to_f32(case["q"], case["dtype"]).astype(np.float64)
    pool = _to_f32(case["pool"], case["dtype"]).astype(np.float64)
    Hq, Hkv, P = case["Hq"], case["Hkv"], case["P"]
    G = Hq // Hkv
    for b in range(q.shape[0]):
        ks = []
        for i in range(int(case["num_pages"][b])):
            slot = case["page_table"][b, i]
            ks.append(pool[slot, 0, :, :case["page_used"][b, i]])
        K = np.concatenate(ks, axis=1)  # [Hkv, T, D]
        for h in range(Hq):
            s = K[h // G] @ q[b, h] * case["scale_f"]
            if case["softcap_f"] > 0:
                s = np.tanh(s / case["softcap_f"]) * case["softcap_f"]
            s = s + case["mask"][b, :s.shape[0]]
            m = s.max()
            ref = m + np.log(np.exp(s - m).sum())
            assert abs(lse[b, h] - ref) < 1e-4 * max(1.0, abs(ref))


def test_merge_oracle_recovers_full_attention(attention_golden):
    """Splitting the pages of a sequence in two and merging the partial
    (O, LSE) states gives the unsplit result (sequence-split math)."""
    case = attention_golden["dense_bf16_d128_p16"]
    full, full_lse = _run_oracle(case)
    npg = case["num_pages"].copy()
    first = npg // 2
    parts_o, parts_l = [], []
    for lo_hi in (0, 1):
        used = case["page_used"].copy()
        for b in range(used.shape[0]):
            if lo_hi == 0:
                used[b, first[b]:] = 0
            else:
                used[b, :first[b]] = 0
        o, l = oracle.paged_attention(
            _to_f32(case["q"], case["dtype"]), case["pool"], _pool_dtype(case),
            case["page_table"], npg, used, num_kv_heads=case["Hkv"], page_size=case["P"],
            scale=case["scale_f"])
        parts_o.append(o.reshape(-1, o.shape[-1]))
        parts_l.append(l.reshape(-1))
    mo, ml = merge.merge_states(np.stack(parts_o), np.stack(parts_l))
    np.testing.assert_allclose(mo, full.reshape(mo.shape), rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(ml, full_lse.reshape(-1), rtol=1e-6, atol=1e-5)


def test_merge_oracle_empty_partition_has_no_weight():
    o = np.random.default_rng(0).standard_normal((2, 3, 8)).astype(np.float32)
    lse = np.array([[1.0, 2.0, -np.inf], [-np.inf, -np.inf, -np.inf]], np.float32)
    mo, ml = merge.merge_states(o, lse)
    np.testing.assert_allclose(mo[:2], o[0, :2], rtol=1e-6)
    assert np.all(mo[2] == 0) and np.isneginf(ml[2])


def test_placement_oracle_matches_reference(placement_golden):
    for entry in placement_golden:
        sc = entry["scenario"]
        snaps = placement.run_scenario(sc)
        assert len(snaps) == len(entry["snapshots"]), sc["name"]
        for i, (mine, ref) in enumerate(zip(snaps, entry["snapshots"])):
            assert mine == ref, f"{sc['name']} snapshot {i}"


def test_norm_rope_oracle_matches_hf(norm_rope_golden):
    z = norm_rope_golden
    tags = sorted({k.split("/")[0] for k in z.files})
    for tag in tags:
        dtype = "float16" if tag.startswith("float16") else "bfloat16"
        conv = (lambda a: _to_f32(a, dtype))
        q, k = conv(z[tag + "/q"]), conv(z[tag + "/k"])
        cos, sin = conv(z[tag + "/cos"]), conv(z[tag + "/sin"])
        qo = norm_rope.rope(norm_rope.rms_norm(q, conv(z[tag + "/qw"]), 1e-6, dtype),
                            cos[:, None, :], sin[:, None, :], dtype)
        ko = norm_rope.rope(norm_rope.rms_norm(k, conv(z[tag + "/kw"]), 1e-6, dtype),
                            cos[:, None, :], sin[:, None, :], dtype)
        for got, ref in ((qo, conv(z[tag + "/q_out"])), (ko, conv(z[tag + "/k_out"]))):
            ulp = np.abs(ref) * (2 ** -7 if dtype == "bfloat16" else 2 ** -10) + 1e-6
            assert np.all(np.abs(got - ref) <= 2 * ulp), tag
            assert np.mean(got == ref) > 0.99, tag
        # HF's cos/sin tables are reproduced by the restatement of its rotary init
        c2, s2 = norm_rope.rope_tables(z[tag + "/pos"], q.shape[-1], float(z[tag + "/theta"][0]),
                                       dtype)
        assert np.mean(c2 == cos) > 0.99 and np.mean(s2 == sin) > 0.99, tag


def prefill_oracle(case):
    """A prefill chunk row by row: the oracle's streaming attention for one
    query, with that query's mask row (kv_cache.py:469-555 treats every query
    row independently)."""
    q = _to_f32(case["q"], case["dtype"])            # [B, Hq, S, D]
    B, Hq, S, D = q.shape
    lens = case["lens"]
    num_pages, page_used = oracle.dense_page_lists(lens, case["P"], case["page_table"].shape[1])
    out = np.zeros((B, Hq, S, D), np.float32)
    for s in range(S):
        o, _ = oracle.paged_attention(
            q[:, :, s], case["pool"], _pool_dtype(case), case["page_table"], num_pages,
            page_used, num_kv_heads=case["Hkv"], page_size=case["P"], scale=D ** -0.5,
            softcap=case["softcap_f"], mask=np.ascontiguousarray(case["mask"][:, 0, s]))
        out[:, :, s] = o
    return out


def test_prefill_oracle_matches_reference(prefill_golden):
    """Chunks of 30-100 queries under HELM's chunk mask (with key padding,
    softcap, first chunk): the oracle equals the reference's fp32 output."""
    for name, case in prefill_golden.items():
        got = prefill_oracle(case)
        ref = case["out_fp32"]
        assert np.allclose(got, ref, atol=2e-5, rtol=2e-5), (name, np.abs(got - ref).max())
