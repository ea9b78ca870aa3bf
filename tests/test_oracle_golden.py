"""CPU: the oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py)."""
import torch

from oracle import oracle as O


def test_quantizer_bit_exact_vs_reference(golden):
    for name, c in golden["quant"].items():
        q, s = O.quantize_per_channel(c["w"])
        assert torch.equal(q, c["q"]), name
        assert torch.equal(s.view(torch.int32), c["scale"].view(torch.int32)), name


def test_quantizer_clamps_to_127_and_zero_row():
    w = torch.zeros(2, 1024, dtype=torch.bfloat16)
    w[1, 3] = -2.0
    q, s = O.quantize_per_channel(w)
    assert s[0].item() == 1e-12 or abs(s[0].item() - 1e-12) < 1e-18
    assert int(q[0].abs().max()) == 0
    assert int(q[1, 3]) in (-127, -128)


def test_scale_division_unambiguous_for_all_bf16():
    """absmax/127 rounded to bf16 is the same whether computed as an fp32
    division, a multiplication by fp32(1/127) or exactly -- for every finite
    bf16 value -- so the CUDA quantizer can use an IEEE fp32 division."""
    a = torch.arange(0, 0x7F80, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    t = (a / 127.0).view(torch.int16)
    f = (a.float() / 127.0).to(torch.bfloat16).view(torch.int16)
    r = (a.float() * torch.tensor(1.0 / 127.0, dtype=torch.float32)).to(torch.bfloat16).view(torch.int16)
    assert torch.equal(t, f) and torch.equal(t, r)


def test_rope_tables_match_reference(golden):
    r = golden["rope"]
    cos, sin = O.rope_tables(r["max_seq_len"], theta=r["theta"])
    assert torch.equal(cos.view(torch.int16), r["cos"].view(torch.int16))
    assert torch.equal(sin.view(torch.int16), r["sin"].view(torch.int16))


def test_oracle_decoder_matches_reference_decoder(golden):
    """Reference-module configuration (bf16 q/k/v, fp16 activations into the INT8
    matvecs, fp32 residual) reproduces QwenDecoder.decode_step."""
    from megaqwen_b200.synth import make_synthetic_state
    d = golden["decoder"]
    st = make_synthetic_state(seed=d["seed"], num_layers=d["layers"])
    o = O.OracleDecoder(st, d["layers"], max_seq_len=64, qkv_int8=False, act_half=True, bf16_hidden=False)
    t = d["start"]
    for i, ref_tok in enumerate(d["tokens"]):
        t, logits, _ = o.step(t, want_logits=True)
        assert t == ref_tok, (i, t, ref_tok)
        assert O.rel_err(d["normalized"][i], o.normalized) < 1e-5
        assert torch.allclose(logits[d["top_idx"][i]], d["top_vals"][i], rtol=1e-5, atol=1e-5)


def test_bytes_per_step_matches_published_formula():
    assert O.bytes_per_step_int8(28, 0) == 598_101_504
    assert O.bytes_per_step_int8(28, 200) - O.bytes_per_step_int8(28, 0) == 200 * 114_688
