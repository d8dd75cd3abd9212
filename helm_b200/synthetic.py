"""Random-initialised models of the BASELINE.json architectures (no checkpoints
are available offline).

Weights are N(0, std) drawn parameter by parameter in named_parameters()
order from one seeded generator, RMSNorm weights are 1.  Models up to ~1B
parameters draw on the CPU generator (device-independent values); larger ones
draw on the target CUDA device's generator, which is far faster and still
deterministic for a given GPU model and seed.
"""
from __future__ import annotations

import torch

ARCHS = {
    # name: (family, layers, hidden, q heads, kv heads, head_dim, intermediate, vocab, theta)
    "qwen3-0.6b": ("qwen3", 28, 1024, 16, 8, 128, 3072, 151936, 1e6),
    "qwen3-8b": ("qwen3", 36, 4096, 32, 8, 128, 12288, 151936, 1e6),
    "qwen3-14b": ("qwen3", 40, 5120, 40, 8, 128, 17408, 151936, 1e6),
    "llama2-13b": ("llama", 40, 5120, 40, 40, 128, 13824, 32000, 1e4),
}


def make_config(name: str, *, num_layers: int | None = None, max_positions: int = 40960,
                **overrides):
    """HF config of a named architecture ('qwen3-0.6b', ...) or of a tiny one
    given fully by keyword arguments (family='qwen3'|'llama', ...)."""
    if name in ARCHS:
        fam, L, hid, hq, hkv, d, inter, vocab, theta = ARCHS[name]
    else:
        fam = overrides.pop("family", "qwen3")
        L, hid, hq, hkv, d, inter, vocab, theta = (
            overrides.pop("layers", 2), overrides.pop("hidden", 512), overrides.pop("q_heads", 8),
            overrides.pop("kv_heads", 4), overrides.pop("head_dim", 64),
            overrides.pop("intermediate", 1024), overrides.pop("vocab", 1000),
            overrides.pop("theta", 1e6))
    if num_layers is not None:
        L = num_layers
    common = dict(vocab_size=vocab, hidden_size=hid, intermediate_size=inter,
                  num_hidden_layers=L, num_attention_heads=hq, num_key_value_heads=hkv,
                  head_dim=d, max_position_embeddings=max_positions, rms_norm_eps=1e-6,
                  attention_dropout=0.0)
    common.update(overrides)
    if fam == "qwen3":
        from transformers import Qwen3Config
        cfg = Qwen3Config(rope_theta=theta, tie_word_embeddings=(name == "qwen3-0.6b"),
                          **common)
    elif fam == "llama":
        from transformers import LlamaConfig
        cfg = LlamaConfig(rope_theta=theta, tie_word_embeddings=False, **common)
    else:
        raise ValueError(fam)
    cfg._attn_implementation = "sdpa"
    return cfg


@torch.no_grad()
def build_model(cfg, *, seed: int = 0, std: float = 0.02, dtype=torch.bfloat16,
                device="cuda", cpu_generator_limit: int = 1_500_000_000):
    """Random-init causal LM on `device` in `dtype` (see module docstring)."""
    from transformers import AutoModelForCausalLM
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(cfg)
    model = model.to_empty(device=device).to(dtype)
    n_params = sum(p.numel() for p in model.parameters())
    on_cpu = n_params <= cpu_generator_limit
    gen = torch.Generator(device="cpu" if on_cpu else device).manual_seed(seed)
    for name, p in model.named_parameters():
        if name.endswith("norm.weight") or "layernorm" in name or name.endswith("q_norm.weight") \
                or name.endswith("k_norm.weight"):
            p.fill_(1.0)
            continue
        t = torch.randn(p.shape, generator=gen, device="cpu" if on_cpu else device) * std
        p.copy_(t.to(device=device, dtype=dtype))
    # non-persistent buffers (rotary inv_freq) were left empty by to_empty: rebuild them
    for module in model.modules():
        if hasattr(module, "inv_freq") and hasattr(module, "rope_init_fn"):
            inv, scaling = module.rope_init_fn(module.config, device)
            module.inv_freq = inv
            module.original_inv_freq = inv.clone()
            module.attention_scaling = scaling
        elif hasattr(module, "inv_freq") and hasattr(module, "compute_default_rope_parameters"):
            inv, scaling = module.compute_default_rope_parameters(module.config, device)
            module.inv_freq = inv
            module.original_inv_freq = inv.clone()
            module.attention_scaling = scaling
    model.eval()
    return model
