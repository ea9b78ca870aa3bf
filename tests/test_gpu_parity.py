"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Tolerances:
  * INT8 codes and fp32 scales: bit-exact.
  * per-matvec rel_err = max|a-b|/max|a| <= 1e-2 and cosine >= 0.9998
    (a = oracle on the same int8 codes; the kernel typically lands near 1e-6).
  * logits of a full decode step: same bar; greedy tokens: >= 95 % agreement.
"""
import pytest
import torch

import megaqwen_b200 as mq
from megaqwen_b200 import _lib
from megaqwen_b200.decoder import layer_lists
from oracle import oracle as O

pytestmark = pytest.mark.gpu
REL, COS = 1e-2, 0.9998
DEV = "cuda"


def close(a, b, rel=REL, cos=COS):
    e, c = O.rel_err(a, b), O.cosine(a, b)
    assert e <= rel and c >= cos, f"rel_err {e:.3e} cos {c:.7f}"
    return e, c


@pytest.fixture(scope="module")
def small_state():
    """2-layer synthetic model with non-unit norm weights, so every norm weight
    (input, post-attention, q_norm, k_norm, final) is exercised."""
    st = mq.make_synthetic_state(seed=0, num_layers=2)
    g = torch.Generator().manual_seed(99)
    for k in st:
        if "norm" in k:
            st[k] = (1.0 + 0.2 * torch.randn(st[k].shape, generator=g)).to(torch.bfloat16)
    return st


def build_int8(state, L, max_seq):
    q = mq.quantize_state(state, num_layers=L, device=DEV)
    layers, scales = layer_lists(q, L, True)
    cos, sin = mq.make_rope(max_seq, device=DEV)
    lm_q, lm_s = q["lm_head.weight"]
    return mq.A10Int8MegakernelDecoder(q["model.embed_tokens.weight"], layers, scales, lm_q, lm_s,
                                       q["model.norm.weight"], cos, sin, L, max_seq)


def build_bf16(state, L, max_seq):
    st = {k: v.to(DEV) for k, v in state.items()}
    layers, _ = layer_lists(st, L, False)
    cos, sin = mq.make_rope(max_seq, device=DEV)
    return mq.A10MegakernelDecoder(st["model.embed_tokens.weight"], layers, st["model.norm.weight"],
                                   st["model.embed_tokens.weight"], cos, sin, L, max_seq)


# --------------------------------------------------------------------------- quantizer
def test_quantizer_bit_exact(golden, small_state):
    cases = [c["w"] for c in golden["quant"].values()]
    cases.append(small_state["model.layers.0.self_attn.q_proj.weight"])
    cases.append(small_state["model.embed_tokens.weight"])            # full LM head, 151936 x 1024
    for w in cases:
        qr, sr = O.quantize_per_channel(w)
        qg, sg = mq.quantize_per_channel(w.to(DEV))
        assert torch.equal(qg.cpu(), qr)
        assert torch.equal(sg.cpu().view(torch.int32), sr.view(torch.int32))


def test_quantizer_matches_golden_directly(golden):
    for name, c in golden["quant"].items():
        qg, sg = mq.quantize_per_channel(c["w"].to(DEV))
        assert torch.equal(qg.cpu(), c["q"]), name
        assert torch.equal(sg.cpu(), c["scale"]), name


# --------------------------------------------------------------------------- matvec
def _matvec(kind, W, s, x, M, K):
    y = torch.empty(M, dtype=torch.float32, device=DEV)
    import ctypes
    rc = _lib.load().mq_matvec(kind, ctypes.c_void_p(W.data_ptr()),
                               ctypes.c_void_p(s.data_ptr() if s is not None else 0),
                               ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), M, K,
                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "mq_matvec")
    torch.cuda.synchronize()
    return y.cpu()


@pytest.mark.parametrize("M,K", [(4096, 1024), (1024, 2048), (3072, 1024), (1024, 3072), (151936, 1024),
                                 (1, 1024), (7, 3072), (149, 2048), (300, 1024)])
def test_matvec_int8_and_bf16(M, K):
    g = torch.Generator().manual_seed(M * 7 + K)
    w = (torch.randn(M, K, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(K, generator=g)
    q, s = O.quantize_per_channel(w)
    ref = O.matvec_int8(x, q, s)
    got = _matvec(0, q.to(DEV), s.to(DEV), x.to(DEV), M, K)
    if M >= 16:
        close(ref, got)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-4 * float(ref.abs().max()))
    ref16 = w.float() @ x
    got16 = _matvec(1, w.to(DEV), None, x.to(DEV), M, K)
    assert torch.allclose(got16, ref16, rtol=1e-4, atol=1e-4 * float(ref16.abs().max()))


# --------------------------------------------------------------------------- decode
def _teacher_forced(dec, orc, start, steps, L):
    """Feeds both decoders the oracle's token sequence; compares every step."""
    tok = start
    logits = torch.empty(mq.CFG.vocab_size, dtype=torch.float32, device=DEV)
    hid = torch.empty(L, 1024, dtype=torch.float32, device=DEV)
    agree = 0
    errs = []
    for i in range(steps):
        out = dec.decode_steps(tok, 1, logits=logits, layer_hidden=hid)
        t_o, l_o, h_o = orc.step(tok, want_logits=True)
        g = int(out.item())
        dec.check_device()
        errs.append(close(l_o, logits.cpu()))
        for li in range(L):
            close(h_o[li], hid[li].cpu())
        close(orc.normalized, dec.normalized.cpu())
        agree += int(g == t_o)
        tok = t_o
    return agree, errs


def test_decode_int8_two_layers_teacher_forced(small_state):
    L, steps = 2, 40
    dec = build_int8(small_state, L, 128)
    orc = O.OracleDecoder(small_state, L, max_seq_len=128)
    agree, errs = _teacher_forced(dec, orc, 17, steps, L)
    assert agree >= 0.95 * steps, agree
    # the KV cache written by the kernel equals the oracle's (bf16 values, within rounding)
    kc, vc = dec.k_cache[:, :, :steps].float().cpu(), dec.v_cache[:, :, :steps].float().cpu()
    close(orc.k_cache[:, :, :steps].float(), kc)
    close(orc.v_cache[:, :, :steps].float(), vc)


def test_decode_step_reference_surface(small_state):
    """decode_step/reset/position as the reference's pybind class."""
    L = 2
    dec = build_int8(small_state, L, 64)
    orc = O.OracleDecoder(small_state, L, max_seq_len=64)
    t_g = t_o = 5
    for _ in range(10):
        t_g = dec.decode_step(t_g)
        t_o = orc.decode_step(t_o)
    assert dec.position() == 10
    first = dec.decode_step(t_g)
    # the reference-signature C entry point on the dense layout gives the same step
    dec.reset()
    orc2 = O.OracleDecoder(small_state, L, max_seq_len=64)
    t_in, agree = 5, 0
    for _ in range(6):   # teacher-forced on the oracle's tokens
        t_a = dec.decode_step_reference_abi(t_in)
        t_b = orc2.decode_step(t_in)
        agree += int(t_a == t_b)
        t_in = t_b
    assert agree >= 5, agree
    dec.reset()
    assert dec.position() == 0 and int(dec.k_cache.abs().sum()) == 0
    with pytest.raises(ValueError):
        dec.decode_step(mq.CFG.vocab_size)


def test_decode_bf16_two_layers_teacher_forced(small_state):
    L, steps = 2, 16
    dec = build_bf16(small_state, L, 64)
    orc = O.OracleDecoder(small_state, L, max_seq_len=64, quantized=False)
    agree, _ = _teacher_forced(dec, orc, 3, steps, L)
    assert agree >= 0.95 * steps


@pytest.mark.parametrize("ctx", [700, 4096, 16384, 32768])
def test_long_context_split_attention(small_state, ctx):
    """Pre-filled random KV cache (N(0,1) bf16) -> one step at position ctx
    exercises the split-K attention merge."""
    L = 2
    dec = build_int8(small_state, L, ctx + 8)
    orc = O.OracleDecoder(small_state, L, max_seq_len=ctx + 8)
    g = torch.Generator().manual_seed(ctx)
    kv = torch.randn((2, L, 8, ctx, 128), generator=g).to(torch.bfloat16)
    orc.k_cache[:, :, :ctx] = kv[0]
    orc.v_cache[:, :, :ctx] = kv[1]
    dec.k_cache[:, :, :ctx] = kv[0].to(DEV)
    dec.v_cache[:, :, :ctx] = kv[1].to(DEV)
    orc.position = ctx
    dec.set_position(ctx)
    logits = torch.empty(mq.CFG.vocab_size, dtype=torch.float32, device=DEV)
    out = dec.decode_steps(11, 1, logits=logits)
    t_o, l_o, _ = orc.step(11, want_logits=True)
    dec.check_device()
    close(l_o, logits.cpu())
    assert int(out.item()) == t_o


def test_run_twice_bitwise_deterministic(small_state):
    L = 2
    dec = build_int8(small_state, L, 64)
    outs = []
    for _ in range(2):
        dec.reset()
        logits = torch.empty(mq.CFG.vocab_size, dtype=torch.float32, device=DEV)
        toks = dec.decode_steps(9, 12, logits=logits)
        outs.append((toks.cpu(), logits.cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])


def test_bounded_wait_reports_timeout_and_context_survives(small_state):
    """A CTA that skips its QKV publish makes every consumer's bounded wait run
    out; the kernel records MQ_DEV_TIMEOUT_EXCHANGE and returns, and the CUDA
    context stays usable."""
    L = 2
    dec = build_int8(small_state, L, 64)
    _lib.device_status(clear=True)
    _lib.set_wait_budget_ns(50_000_000)
    try:
        _lib.inject_skip_publish(True, 0)
        with pytest.raises(_lib.MQError, match="exchange wait timed out"):
            dec.decode_step(1)
    finally:
        _lib.inject_skip_publish(False)
        _lib.set_wait_budget_ns(2_000_000_000)
    dec.reset()
    assert dec.decode_step(1) >= 0
    assert _lib.device_status() == (0, 0)
