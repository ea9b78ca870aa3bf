"""GPU: the allocation-free INT8 decode entry point (launch_a10_int8_decode_static).

It exists for callers that cannot call cudaMalloc while they decode -- e.g. a
plugin inside a host framework that owns all device memory through its own
arena -- and keeps its hand-off workspace in a static device array of the
library instead.  This test calls it through the C ABI on two steps in a row
and checks each step against the allocating entry point
(launch_a10_int8_decode, via decode_step_reference_abi) fed identical inputs: same argmax token, final RMSNorm
output and written K/V within the parity tolerance (rel_err <= 1e-2, cosine >=
0.9998).  The file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

import megaqwen_b200 as mq
from megaqwen_b200 import _lib
from megaqwen_b200.decoder import layer_lists
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _close(a, b):
    e, c = O.rel_err(a, b), O.cosine(a, b)
    assert e <= 1e-2 and c >= 0.9998, (e, c)


def test_static_workspace_entry_matches_allocating_entry():
    L, max_seq = 2, 64
    st = mq.make_synthetic_state(seed=5, num_layers=L)
    q = mq.quantize_state(st, num_layers=L, device="cuda")
    layers, scales = layer_lists(q, L, True)
    cos, sin = mq.make_rope(max_seq, device="cuda")
    lm_q, lm_s = q["lm_head.weight"]
    dec = mq.A10Int8MegakernelDecoder(q["model.embed_tokens.weight"], layers, scales, lm_q, lm_s,
                                      q["model.norm.weight"], cos, sin, L, max_seq)
    lib = _lib.load()
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    kc2, vc2 = dec.k_cache.clone(), dec.v_cache.clone()
    out2 = torch.empty(1, dtype=torch.int32, device="cuda")
    norm2 = torch.empty(1024, dtype=torch.float32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    tok = 23
    for step in range(2):
        pos = dec.position()
        rc = lib.launch_a10_int8_decode_static(
            tok, p(out2), p(dec.embed_weight_), p(dec.d_layer_weights_), p(dec.final_norm_weight_),
            p(dec.lm_head_weight_), p(dec.lm_head_scale_), p(dec.cos_table_), p(dec.sin_table_), p(kc2), p(vc2),
            p(norm2), L, pos, pos + 1, max_seq, ctypes.c_float(dec.attn_scale_), p(dec.d_layer_scales_), stream)
        assert rc == 0, rc
        ref_tok = dec.decode_step_reference_abi(tok)   # launch_a10_int8_decode, same inputs
        got_tok = int(out2.item())
        assert got_tok == ref_tok, (step, got_tok, ref_tok)
        _close(dec.normalized.cpu(), norm2.cpu())
        _close(dec.k_cache[:, :, :pos + 1].float().cpu(), kc2[:, :, :pos + 1].float().cpu())
        _close(dec.v_cache[:, :, :pos + 1].float().cpu(), vc2[:, :, :pos + 1].float().cpu())
        tok = ref_tok


def test_static_workspace_entry_rejects_too_many_layers():
    lib = _lib.load()
    n = ctypes.c_void_p(0)
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    d = ctypes.c_void_p(dummy.data_ptr())
    rc = lib.launch_a10_int8_decode_static(0, d, d, d, d, d, d, d, d, d, d, n, 33, 0, 1, 64,
                                           ctypes.c_float(0.1), d, n)
    assert rc == -5  # MQ_ERR_SIZE
