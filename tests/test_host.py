"""CPU: host-side logic of the package (config, synthetic weights, flat lists,
constructor validation, no CPU fallback)."""
import pytest
import torch

import megaqwen_b200 as mq
from megaqwen_b200 import config as C
from megaqwen_b200.decoder import layer_lists


def test_config_matches_qwen3_0p6b():
    assert (C.HIDDEN_SIZE, C.INTERMEDIATE_SIZE, C.NUM_Q_HEADS, C.NUM_KV_HEADS, C.HEAD_DIM) == (1024, 3072, 16, 8, 128)
    assert C.VOCAB_SIZE == 151936 and C.NUM_LAYERS == 28 and C.RMS_EPS == 1e-6


def test_synthetic_state_is_seeded_and_shaped():
    a = mq.make_synthetic_state(seed=3, num_layers=1, vocab_size=512)
    b = mq.make_synthetic_state(seed=3, num_layers=1, vocab_size=512)
    c = mq.make_synthetic_state(seed=4, num_layers=1, vocab_size=512)
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert not torch.equal(a["model.layers.0.mlp.up_proj.weight"], c["model.layers.0.mlp.up_proj.weight"])
    w = a["model.layers.0.mlp.down_proj.weight"]
    assert w.dtype == torch.bfloat16 and w.shape == (1024, 3072)
    assert 0.015 < w.float().std().item() < 0.05          # N(0, 0.02) plus outliers
    assert w.float().abs().max().item() > 0.2               # the x20 outliers exist
    assert torch.all(a["model.layers.0.input_layernorm.weight"] == 1)
    assert "lm_head.weight" not in a                        # tied embeddings


def test_layer_lists_order():
    st = {}
    for i in range(2):
        p = f"model.layers.{i}"
        for j, n in enumerate(("input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                               "self_attn.q_norm", "self_attn.k_norm", "self_attn.o_proj",
                               "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")):
            st[f"{p}.{n}.weight"] = (torch.full((1,), 100 * i + j), torch.full((1,), -(100 * i + j)))
    layers, scales = layer_lists(st, 2, True)
    assert [int(t) for t in layers] == [100 * i + j for i in range(2) for j in range(11)]
    assert [int(t) for t in scales] == [-(100 * i + j) for i in range(2) for j in (1, 2, 3, 6, 8, 9, 10)]


def test_no_cpu_fallback():
    with pytest.raises(ValueError):
        mq.quantize_per_channel(torch.zeros(4, 1024, dtype=torch.bfloat16))
    emb = torch.zeros(C.VOCAB_SIZE, C.HIDDEN_SIZE, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        mq.A10MegakernelDecoder(emb, [], emb[0], emb, emb[:4, :128], emb[:4, :128], 1, 4)


def test_rope_product_matches_oracle():
    from oracle import oracle as O
    cos, sin = mq.make_rope(300, device="cpu")
    oc, os_ = O.rope_tables(300)
    assert torch.equal(cos, oc) and torch.equal(sin, os_)
