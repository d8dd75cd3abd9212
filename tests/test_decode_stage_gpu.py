"""Whole-model decode through FusedDecodeStage (GPU).

The fused step (RMSNorm+QKV GEMV, fused append, paged attention, o_proj and
down_proj with the residual add, RMSNorm+gate/up GEMV with SwiGLU, final norm
+ lm_head) replayed as a CUDA graph by GraphDecoder, teacher forced, against
HF's own modules over its DynamicCache in the model dtype and on an fp32 copy:
the fused logits must be at least as accurate as HF's low-precision path
(max |err vs fp32| <= 1.25 x HF's + 2e-2, mean <= 1.25 x HF's + 1e-3), with
and without cold-page offload.  Also the GEMV kernel alone against fp32 math.
"""
import copy

import pytest
import torch

from helm_b200 import _capi
from helm_b200.runtime.graph_decode import GraphDecoder
from helm_b200.runtime.kv_cache import get_paging_stats, reset_paging_stats
from helm_b200.runtime.kv_offload import KVOffloadConfig, KVOffloadManager
from helm_b200.synthetic import build_model, make_config
from test_model_gpu import _assert_logits_close, _hf_incremental

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda:0")


@pytest.mark.parametrize("B,N,K", [(1, 1000, 512), (3, 777, 1024), (8, 256, 2048),
                                   (16, 130, 640), (2, 300, 9008), (1, 513, 17408),
                                   (4, 100, 5120)])
def test_gemv_variants_vs_fp32(dev, B, N, K):
    g = torch.Generator(device=dev).manual_seed(B * 7 + N)
    x = torch.randn(B, K, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(N, K, device=dev, generator=g) * 0.05).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(K, device=dev, generator=g)).to(torch.bfloat16)
    res = torch.randn(B, N, device=dev, generator=g).to(torch.bfloat16)
    # plain
    y = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
    _capi.decode_gemv(x, w, out=y)
    ref = x.float() @ w.float().t()
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=1e-2)
    # rmsnorm (HF rounding: normalised x in bf16, then weight * x in bf16)
    xn = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)
    xn = nw * xn
    _capi.decode_gemv(x, w, out=y, norm_w=nw, eps=1e-6)
    assert torch.allclose(y.float(), xn.float() @ w.float().t(), atol=3e-2, rtol=2e-2)
    # swiglu
    _capi.decode_gemv(x, w, w2=w2, out=y)
    gate = (x.float() @ w.float().t()).to(torch.bfloat16)
    up = (x.float() @ w2.float().t()).to(torch.bfloat16)
    ref = (torch.nn.functional.silu(gate) * up).float()
    assert torch.allclose(y.float(), ref, atol=3e-2, rtol=2e-2)
    # residual, in place, fp32 output variant
    y32 = torch.empty(B, N, dtype=torch.float32, device=dev)
    _capi.decode_gemv(x, w, out=y32)
    assert torch.allclose(y32, (x.float() @ w.float().t()).to(torch.bfloat16).float(), atol=2e-2,
                          rtol=1e-2)
    h = res.clone()
    _capi.decode_gemv(x, w, out=h, residual=h)
    ref = (res.float() + (x.float() @ w.float().t()).to(torch.bfloat16).float())
    assert torch.allclose(h.float(), ref, atol=3e-2, rtol=2e-2)


def _tiny(family, dtype, dev, layers=3, head_dim=64):
    cfg = make_config("tiny", family=family, layers=layers, hidden=512, q_heads=8, kv_heads=4,
                      head_dim=head_dim, intermediate=1024, vocab=512,
                      theta=1e6 if family == "qwen3" else 1e4)
    return build_model(cfg, seed=0, std=0.05, dtype=dtype, device=dev)


@pytest.mark.parametrize("family,dtype,watermark,head_dim", [
    ("qwen3", torch.bfloat16, None, 64), ("qwen3", torch.bfloat16, 1024, 128),
    ("llama", torch.float16, None, 64)])
def test_fused_stage_logits_match_hf(dev, family, dtype, watermark, head_dim):
    model = _tiny(family, dtype, dev, head_dim=head_dim)
    g = torch.Generator().manual_seed(1)
    S, n = 96, 24
    prompt = torch.randint(0, 512, (1, S), generator=g).to(dev)
    forced = torch.randint(0, 512, (1, n), generator=g).to(dev)
    ref = _hf_incremental(model, prompt, forced, n)
    ref32 = _hf_incremental(copy.deepcopy(model).float(), prompt, forced, n)
    cfg = KVOffloadConfig.from_model(model, page_size=16, gpu_watermark_bytes=watermark)
    mgr = KVOffloadManager(model, cfg)
    try:
        reset_paging_stats()
        gd = GraphDecoder(model, mgr, max_len=S + n + 1, fused=True)
        _, logits = gd.generate(prompt, n, keep_logits=True, forced_tokens=forced)
        stats = get_paging_stats()
    finally:
        mgr.restore()
    mine = torch.stack(logits, 1)
    _assert_logits_close(mine, ref, ref32, dtype)
    if watermark is not None:
        assert stats["pages_evicted"] > 0 and stats["pages_prefetched"] > 0
