"""GPU: the BASELINE configs beyond config 1 checked directly against the CPU
oracle (the reference's PyTorch formulation, int8_decoder.py:263-298 restated).

  * config 2: the 28-layer BF16 model, 200 greedy steps with on-device token
    feedback, teacher-forced oracle agreement >= 95 % plus a final step on the
    kernel's own KV cache (logits rel_err <= 1e-2, cosine >= 0.9998);
  * config 4: one batched step of the 28-layer INT8 model, four sequences at
    positions spread over 128..2048 with random N(0,1) KV caches, each compared
    with the oracle on the same cache: equal tokens, logits within 2.5x of the
    batch-1 kernel's own deviation from the oracle (see REL_28 below);
  * chunked prefill: one 64-token chunk of the 28-layer model against the
    oracle fed the prompt one token per step (KV cache cosine; last-position
    logits on the chunk's own cache to the same bar);
  * the batched fp16 operand path with large-magnitude activation dims: it
    either meets the bar or stops the step cleanly with MQ_DEV_RANGE;
  * A10Decoder.generate (a10_decode.py:358-393) against the oracle's greedy
    next-token choices on the same sequence.
"""
import pytest
import torch

import megaqwen_b200 as mq
from megaqwen_b200 import _lib
from oracle import oracle as O
from test_gpu_parity import build_bf16, build_int8, close

pytestmark = [pytest.mark.gpu, pytest.mark.slow]
V = mq.CFG.vocab_size
# End-to-end bar for one step through all 28 layers of the tensor-core paths
# (batched decode, prefill).  Their GEMMs meet the per-matvec bar by far
# (rel_err <= 1e-3 against fp64, test_gpu_batch_gemm.py); what adds up is the
# residual stream's rounding to bf16 after every layer (the kernel-faithful
# formulation, a10_int8_decode_kernel.cu:571): any rounding-level difference
# flips some bf16 roundings (2^-8 relative each) and 28 layers compound them,
# most with random N(0,1) KV caches.  The exact-integer batch-1 kernel itself
# lands at logits rel_err 1.4e-2 .. 1.8e-2 (cosine 0.99984 .. 0.99990) against
# the oracle on these inputs, so the batched step is held to equal greedy
# tokens and to at most 2.5x the batch-1 kernel's own deviation (rel_err and
# 1 - cosine), measured side by side on the same inputs; REL_28 is the floor.
REL_28 = 2.5e-2


@pytest.fixture(scope="module")
def state28():
    return mq.make_synthetic_state(seed=0, num_layers=28)


def test_bf16_28_layers_200_steps(state28):
    L, steps, start = 28, 200, 4242
    dec = build_bf16(state28, L, 256)
    toks = dec.decode_steps(start, steps).cpu().tolist()
    dec.check_device()
    orc = O.OracleDecoder(state28, L, max_seq_len=256, quantized=False)
    inputs = [start] + toks[:-1]
    agree = sum(int(orc.decode_step(t) == toks[i]) for i, t in enumerate(inputs))
    assert agree >= 0.95 * steps, f"{agree}/{steps}"
    orc.k_cache[:, :, :steps] = dec.k_cache[:, :, :steps].cpu()
    orc.v_cache[:, :, :steps] = dec.v_cache[:, :, :steps].cpu()
    lg = torch.empty(V, dtype=torch.float32, device="cuda")
    dec.decode_steps(toks[-1], 1, logits=lg)
    _, l_o, _ = orc.step(toks[-1], want_logits=True)
    close(l_o, lg.cpu())


def test_batched_28_layers_vs_oracle(state28):
    L, max_seq = 28, 2080
    positions = [128, 700, 1400, 2047]
    tokens = [11, 4242, 90001, 151935]
    dec = build_int8(state28, L, max_seq)
    bd = mq.BatchedDecoder(dec, len(positions), max_seq)
    g = torch.Generator(device="cuda").manual_seed(77)
    for b, p in enumerate(positions):
        bd.k_cache[b, :, :, :p].normal_(generator=g)
        bd.v_cache[b, :, :, :p].normal_(generator=g)
    kc, vc = bd.k_cache.cpu(), bd.v_cache.cpu()
    bd.set_state(tokens, positions)
    logits = torch.empty(len(positions), V, dtype=torch.float32, device="cuda")
    out = bd.step(1, logits=logits).cpu().tolist()
    bd.check_device()
    orc = O.OracleDecoder(state28, L, max_seq_len=max_seq)
    for b, p in enumerate(positions):
        orc.reset()
        orc.k_cache[:, :, :p] = kc[b, :, :, :p]
        orc.v_cache[:, :, :p] = vc[b, :, :, :p]
        orc.position = p
        t_o, l_o, _ = orc.step(tokens[b], want_logits=True)
        # the batch-1 kernel on the same inputs, for reference
        dec.k_cache.copy_(kc[b].to("cuda"))
        dec.v_cache.copy_(vc[b].to("cuda"))
        dec.set_position(p)
        l1 = torch.empty(V, dtype=torch.float32, device="cuda")
        dec.decode_steps(tokens[b], 1, logits=l1)
        print("seq %d pos %d: batched rel_err %.3e cos %.7f | batch-1 rel_err %.3e cos %.7f | batched vs batch-1 %.3e" % (
            b, p, O.rel_err(l_o, logits[b].cpu()), O.cosine(l_o, logits[b].cpu()), O.rel_err(l_o, l1.cpu()),
            O.cosine(l_o, l1.cpu()), O.rel_err(l1.cpu(), logits[b].cpu())))
        e_b, c_b = O.rel_err(l_o, logits[b].cpu()), O.cosine(l_o, logits[b].cpu())
        e_1, c_1 = O.rel_err(l_o, l1.cpu()), O.cosine(l_o, l1.cpu())
        assert e_b <= max(REL_28, 2.5 * e_1) and (1 - c_b) <= 2.5 * max(1 - c_1, 1e-5), (b, e_b, c_b, e_1, c_1)
        assert out[b] == t_o, (b, out[b], t_o)
        # the K/V the batched step wrote for this position
        assert O.cosine(orc.k_cache[:, :, p].float(), bd.k_cache[b, :, :, p].float().cpu()) >= 0.9998
        assert O.cosine(orc.v_cache[:, :, p].float(), bd.v_cache[b, :, :, p].float().cpu()) >= 0.9998


def test_prefill_chunk_28_layers_vs_oracle(state28):
    L, n = 28, 64
    dec = build_int8(state28, L, 128)
    ids = torch.randint(0, V, (n,), generator=torch.Generator().manual_seed(3)).tolist()
    lg = torch.empty(n, V, dtype=torch.float32, device="cuda")
    nxt = dec.prefill(ids, logits=lg)
    orc = O.OracleDecoder(state28, L, max_seq_len=128)
    for t in ids:
        orc.decode_step(t)
    # the KV cache the chunk wrote for all 64 prompt positions
    assert O.cosine(orc.k_cache[:, :, :n].float(), dec.k_cache[:, :, :n].float().cpu()) >= 0.9998
    assert O.cosine(orc.v_cache[:, :, :n].float(), dec.v_cache[:, :, :n].float().cpu()) >= 0.9998
    # the last prompt position on identical inputs: the oracle attends over the
    # chunk's own cache for positions 0..62
    orc.reset()
    orc.k_cache[:, :, :n - 1] = dec.k_cache[:, :, :n - 1].cpu()
    orc.v_cache[:, :, :n - 1] = dec.v_cache[:, :, :n - 1].cpu()
    orc.position = n - 1
    t_o, l_o, _ = orc.step(ids[-1], want_logits=True)
    print("prefill last position rel_err %.3e cos %.7f" % (O.rel_err(l_o, lg[n - 1].cpu()), O.cosine(l_o, lg[n - 1].cpu())))
    close(l_o, lg[n - 1].cpu(), rel=REL_28)
    assert nxt == t_o


def test_batched_large_activations_meet_bar_or_refuse():
    """Real checkpoints carry a few residual dims in the hundreds to thousands.
    Scaling three input-norm weight dims of layer 1 by 1e3 puts such values into
    the batched path's fp16 GEMM operands (h * w * 2^-8)."""
    L, max_seq = 2, 64
    st = mq.make_synthetic_state(seed=1, num_layers=L)
    w = st["model.layers.1.input_layernorm.weight"].float()
    w[[5, 77, 300]] *= 1000.0
    st["model.layers.1.input_layernorm.weight"] = w.bfloat16()
    dec = build_int8(st, L, max_seq)
    positions, tokens = [3, 10], [7, 123]
    bd = mq.BatchedDecoder(dec, 2, max_seq)
    g = torch.Generator(device="cuda").manual_seed(5)
    for b, p in enumerate(positions):
        bd.k_cache[b, :, :, :p].normal_(generator=g)
        bd.v_cache[b, :, :, :p].normal_(generator=g)
    kc, vc = bd.k_cache.cpu(), bd.v_cache.cpu()
    bd.set_state(tokens, positions)
    logits = torch.empty(2, V, dtype=torch.float32, device="cuda")
    out = bd.step(1, logits=logits).cpu().tolist()
    code, _ = bd.status()
    if code:
        assert code == 5, code          # MQ_DEV_RANGE: refused cleanly, tokens left at -1
        assert out == [-1, -1]
        return
    orc = O.OracleDecoder(st, L, max_seq_len=max_seq)
    for b, p in enumerate(positions):
        orc.reset()
        orc.k_cache[:, :, :p] = kc[b, :, :, :p]
        orc.v_cache[:, :, :p] = vc[b, :, :, :p]
        orc.position = p
        t_o, l_o, _ = orc.step(tokens[b], want_logits=True)
        close(l_o, logits[b].cpu())
        assert out[b] == t_o


@pytest.mark.parametrize("quantized", [True, False])
def test_generate_matches_oracle_greedy(quantized):
    L = 4
    st = mq.make_synthetic_state(seed=2, num_layers=L)
    dec = mq.A10Decoder(st, quantized=quantized, max_seq_len=128, num_layers=L)
    prompt = torch.randint(0, V, (20,), generator=torch.Generator().manual_seed(9)).tolist()
    out = dec.generate(prompt, max_new_tokens=30)
    assert out[:20] == prompt and len(out) == 50
    orc = O.OracleDecoder(st, L, max_seq_len=128, quantized=quantized)
    agree = 0
    for i in range(len(out) - 1):
        t = orc.decode_step(out[i])
        if i >= 19:
            agree += int(t == out[i + 1])
    assert agree >= 0.95 * 30, f"{agree}/30"
