"""Seeded synthetic Qwen3-0.6B weights (no checkpoint is available offline).

Every linear weight and the (tied) embedding is drawn bf16 from N(0, std) with a
torch CPU generator seeded once, in a fixed tensor order; a fraction
`outlier_frac` of entries is scaled by `outlier_scale`.  Norm weights are 1.0.
The LM head is tied to the embedding, as in Qwen3-0.6B.
"""
import torch

from .config import CFG

_LINEARS = (
    ("self_attn.q_proj", "q_size", "hidden_size"),
    ("self_attn.k_proj", "kv_size", "hidden_size"),
    ("self_attn.v_proj", "kv_size", "hidden_size"),
    ("self_attn.o_proj", "hidden_size", "q_size"),
    ("mlp.gate_proj", "intermediate_size", "hidden_size"),
    ("mlp.up_proj", "intermediate_size", "hidden_size"),
    ("mlp.down_proj", "hidden_size", "intermediate_size"),
)


def _draw(gen, shape, std, outlier_frac, outlier_scale):
    w = torch.randn(shape, generator=gen, dtype=torch.float32).mul_(std)
    if outlier_frac > 0:
        mask = torch.rand(shape, generator=gen) < outlier_frac
        w[mask] *= outlier_scale
    return w.to(torch.bfloat16)


def make_synthetic_state(seed=0, num_layers=CFG.num_layers, std=0.02, outlier_frac=1e-3, outlier_scale=20.0,
                         vocab_size=CFG.vocab_size, cfg=CFG):
    """Returns an HF-named bf16 CPU state dict (no lm_head.weight: tied)."""
    gen = torch.Generator().manual_seed(seed)
    st = {"model.embed_tokens.weight": _draw(gen, (vocab_size, cfg.hidden_size), std, outlier_frac, outlier_scale)}
    ones = lambda n: torch.ones(n, dtype=torch.bfloat16)
    for i in range(num_layers):
        p = f"model.layers.{i}"
        for name, o, k in _LINEARS:
            st[f"{p}.{name}.weight"] = _draw(gen, (getattr(cfg, o), getattr(cfg, k)), std, outlier_frac, outlier_scale)
        st[f"{p}.input_layernorm.weight"] = ones(cfg.hidden_size)
        st[f"{p}.post_attention_layernorm.weight"] = ones(cfg.hidden_size)
        st[f"{p}.self_attn.q_norm.weight"] = ones(cfg.head_dim)
        st[f"{p}.self_attn.k_norm.weight"] = ones(cfg.head_dim)
    st["model.norm.weight"] = ones(cfg.hidden_size)
    return st
