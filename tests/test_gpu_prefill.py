"""GPU: chunked prefill (A10Int8MegakernelDecoder.prefill, MQBatchArgs.prefill)
against feeding the same prompt one decode step per token.

Prefill runs up to 64 prompt tokens per launch through the batched tensor-core
kernel (activations rounded to fp16 at the GEMM inputs); the decode path keeps
fp32 activations and exact-integer matvecs.  Bar: the KV cache written for the
prompt to cosine >= 0.9998, the logits of the last prompt position to
rel_err <= 1e-2 and cosine >= 0.9998, the same greedy next token.
"""
import pytest
import torch

import megaqwen_b200 as mq
from oracle import oracle as O
from test_gpu_parity import build_int8

pytestmark = pytest.mark.gpu


def _stepwise(dec, ids, logits):
    for t in ids[:-1]:
        dec.decode_step(t)
    tok = int(dec.decode_steps(ids[-1], 1, logits=logits).item())
    dec.check_device()
    return tok


@pytest.mark.parametrize("n_before,n_prompt", [(0, 37), (0, 100), (5, 64), (3, 1)])
def test_prefill_matches_stepwise(n_before, n_prompt):
    L, max_seq = 2, 256
    st = mq.make_synthetic_state(seed=7, num_layers=L)
    a, b = build_int8(st, L, max_seq), build_int8(st, L, max_seq)
    g = torch.Generator().manual_seed(n_prompt)
    ids = torch.randint(0, mq.CFG.vocab_size, (n_before + n_prompt,), generator=g).tolist()
    V = mq.CFG.vocab_size
    for t in ids[:n_before]:           # same history decoded step by step in both
        a.decode_step(t)
    last = (n_prompt - 1) % 64 + 1
    logits_a = torch.empty(last, V, dtype=torch.float32, device="cuda")
    tok_a = a.prefill(ids[n_before:], logits=logits_a)
    assert a.position() == n_before + n_prompt
    logits_b = torch.empty(V, dtype=torch.float32, device="cuda")
    tok_b = _stepwise(b, ids, logits_b)
    n = n_before + n_prompt
    for ca, cb in ((a.k_cache, b.k_cache), (a.v_cache, b.v_cache)):
        assert O.cosine(ca[:, :, :n].float().cpu(), cb[:, :, :n].float().cpu()) >= 0.9998
    la, lb = logits_a[-1].cpu(), logits_b.cpu()
    e, c = O.rel_err(lb, la), O.cosine(lb, la)
    assert e <= 1e-2 and c >= 0.9998, (e, c)
    assert tok_a == tok_b
    # decoding continues from the prefilled cache like from the stepwise one
    na = int(a.decode_steps(tok_a, 4)[-1].item())
    nb = int(b.decode_steps(tok_b, 4)[-1].item())
    assert na == nb


def test_prefill_rejects_overflow():
    st = mq.make_synthetic_state(seed=1, num_layers=1)
    a = build_int8(st, 1, 32)
    with pytest.raises(ValueError):
        a.prefill(list(range(33)))
    with pytest.raises(ValueError):
        a.prefill([])
