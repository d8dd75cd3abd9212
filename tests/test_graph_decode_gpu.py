"""Graph-replayed decode (GraphDecoder) against the eager decode loop (GPU).

The captured step runs the same kernels on the same inputs as the eager path;
only the decode kernel's split (grid sized for the graph's max length) differs,
so logits agree to fp32-rounding effects (<= 2e-2 + 2 ulp of the bf16 logit) and
greedy tokens are identical.  With forced cold-page offload the in-graph staging
copies (and the recaptures when the cold set grows) must give the same answer.
"""
import pytest
import torch

from helm_b200.runtime.decode_loop import DecodeLoop
from helm_b200.runtime.graph_decode import GraphDecoder
from helm_b200.runtime.kv_cache import get_paging_stats, reset_paging_stats
from helm_b200.runtime.kv_offload import KVOffloadConfig, KVOffloadManager
from helm_b200.synthetic import build_model, make_config

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    cfg = make_config("tiny", family="qwen3", layers=4, hidden=512, q_heads=8, kv_heads=4,
                      head_dim=128, intermediate=1024, vocab=512)
    return build_model(cfg, seed=0, std=0.05, dtype=torch.bfloat16, device="cuda")


def _close(a, b):
    a, b = a.float(), b.float()
    scale = torch.exp2(torch.floor(torch.log2(b.abs().clamp_min(1e-6))))
    assert bool(((a - b).abs() <= 2e-2 + 2 * 2 ** -7 * scale).all()), (a - b).abs().max()


def _placement(mgr):
    return [[(p.page_id, p.start_token, p.used_tokens, p.state) for p in layer.pages]
            for kvcm in mgr.kvcms for layer in kvcm.layers.values()]


@pytest.mark.parametrize("watermark", [None, 1024])
def test_graph_decode_matches_eager(model, watermark):
    """Same tokens and logits as the eager loop, and the same page placement
    and paging counters afterwards: the graph path's host plan (including its
    steady-step shortcut, which only advances tail pages) keeps the
    reference's bookkeeping."""
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, 512, (1, 128), generator=g).cuda()
    n = 40
    cfg = KVOffloadConfig.from_model(model, page_size=16, gpu_watermark_bytes=watermark)
    mgr = KVOffloadManager(model, cfg)
    try:   # each path on a fresh manager, so that page ids are comparable
        reset_paging_stats()
        toks_e, log_e = DecodeLoop(model, mgr).generate(prompt, n, keep_logits=True)
        stats_e, place_e = get_paging_stats(), _placement(mgr)
    finally:
        mgr.restore()
    mgr = KVOffloadManager(model, cfg)
    try:
        reset_paging_stats()
        gd = GraphDecoder(model, mgr, max_len=128 + n)
        toks_g, log_g = gd.generate(prompt, n, keep_logits=True)
        stats = get_paging_stats()
        place_g = _placement(mgr)
        runs = []
        for layer in mgr.kvcms[0].layers.values():   # host slots of a layer: few long runs
            slots = [p.slot for p in layer.pages if p.state == "CPU"]
            runs.append(1 + sum(b != a + 1 for a, b in zip(slots, slots[1:])) if slots else 0)
    finally:
        mgr.restore()
    assert torch.equal(toks_e, toks_g)
    for a, b in zip(log_g, log_e):
        _close(a, b)
    assert place_g == place_e
    for key in ("evict_calls", "pages_evicted", "bytes_evicted", "pages_prefetched",
                "bytes_prefetched"):
        assert stats[key] == stats_e[key], key
    if watermark is not None:
        assert stats["pages_evicted"] > 0
        assert gd.captures >= 2   # the cold set grew during decode
        assert max(runs) == 1
    else:
        assert gd.captures == 1
