"""GPU: batched decode (csrc/batch_kernel.cu) against the batch-1 kernel.

Each batched step is compared sequence by sequence with a batch-1 step fed
exactly the same input: the sequence's token, position and KV cache (copied
from the batched state before the step).  The batched path rounds activations
to fp16 at the tensor-core GEMM inputs (the batch-1 path keeps fp32), so the
bar is the north-star per-output tolerance: logits rel_err <= 1e-2 and
cosine >= 0.9998, the K/V written for the step to cosine >= 0.9998, and
>= 95 % equal argmax tokens.
"""
import pytest
import torch

import megaqwen_b200 as mq
from oracle import oracle as O
from test_gpu_parity import build_int8

pytestmark = pytest.mark.gpu


def _compare(L, positions, tokens, steps, max_seq, seed=0):
    st = mq.make_synthetic_state(seed=seed, num_layers=L)
    dec = build_int8(st, L, max_seq)
    B = len(positions)
    bd = mq.BatchedDecoder(dec, B, max_seq)
    g = torch.Generator(device="cuda").manual_seed(1234)
    for b, p in enumerate(positions):
        if p:
            bd.k_cache[b, :, :, :p].normal_(generator=g)
            bd.v_cache[b, :, :, :p].normal_(generator=g)
    bd.set_state(tokens, positions)
    agree = total = 0
    logits_b = torch.empty(B, mq.CFG.vocab_size, dtype=torch.float32, device="cuda")
    logits_1 = torch.empty(mq.CFG.vocab_size, dtype=torch.float32, device="cuda")
    for _ in range(steps):
        k_before, v_before = bd.k_cache.clone(), bd.v_cache.clone()
        pos = bd.positions.cpu().tolist()
        tok = bd.tokens.cpu().tolist()
        out = bd.step(1, logits=logits_b).cpu().tolist()
        bd.check_device()
        assert bd.positions.cpu().tolist() == [p + 1 for p in pos]
        for b in range(B):
            dec.k_cache.copy_(k_before[b])
            dec.v_cache.copy_(v_before[b])
            dec.set_position(pos[b])
            t1 = int(dec.decode_steps(tok[b], 1, logits=logits_1).item())
            dec.check_device()
            e, c = O.rel_err(logits_1.cpu(), logits_b[b].cpu()), O.cosine(logits_1.cpu(), logits_b[b].cpu())
            assert e <= 1e-2 and c >= 0.9998, (b, e, c)
            kb = bd.k_cache[b, :, :, pos[b]].float().cpu()
            assert O.cosine(dec.k_cache[:, :, pos[b]].float().cpu(), kb) >= 0.9998
            assert O.cosine(dec.v_cache[:, :, pos[b]].float().cpu(), bd.v_cache[b, :, :, pos[b]].float().cpu()) >= 0.9998
            agree += int(t1 == out[b])
            total += 1
    assert agree >= 0.95 * total, (agree, total)


def test_batched_small_mixed_positions():
    _compare(L=2, positions=[0, 5, 300, 700], tokens=[17, 5, 999, 123456], steps=4, max_seq=1024)


def test_batched_full_batch_of_64():
    g = torch.Generator().manual_seed(7)
    positions = torch.randint(0, 600, (64,), generator=g).tolist()
    tokens = torch.randint(0, mq.CFG.vocab_size, (64,), generator=g).tolist()
    _compare(L=2, positions=positions, tokens=tokens, steps=2, max_seq=640)


def test_batched_rejects_bad_input_on_device():
    st = mq.make_synthetic_state(seed=1, num_layers=1)
    dec = build_int8(st, 1, 64)
    bd = mq.BatchedDecoder(dec, 2, 64)
    bd.set_state([1, 2], [0, 0])
    bd.positions[1] = 999          # past max_seq_len: the kernel must refuse before touching memory
    out = bd.step(1).cpu().tolist()
    assert out == [-1, -1]
    assert bd.status()[0] == 4


def test_batched_long_context_and_single_sequence():
    # one sequence deep in a long cache (many attention pieces per head) next to a short one
    _compare(L=2, positions=[20000, 3], tokens=[11, 22], steps=2, max_seq=20480)
    _compare(L=2, positions=[1500], tokens=[99], steps=2, max_seq=2048)
