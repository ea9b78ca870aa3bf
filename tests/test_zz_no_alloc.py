"""GPU: the allocation-free INT8 decode entry point (launch_a10_int8_decode_static).

It exists for callers that cannot call cudaMalloc while they decode -- e.g. a
plugin inside a host framework that owns all device memory through its own
arena -- and keeps its hand-off workspace in a static device array of the
library instead.

The checks run in a fresh child process, so that nothing else has touched the
library before the static entry point's first call:
  * two steps in a row through the static entry point (C ABI), then the same
    two steps through the allocating entry point (launch_a10_int8_decode) on
    identical inputs: tokens, final RMSNorm output and the written K/V are
    bitwise equal (same kernel, same inputs, order-independent integer sums);
  * free device memory is unchanged across static calls after the first, and
    the allocating path's workspace was never created by them;
  * a static call whose bounded wait runs out (a short wait budget plus the
    host-side skip-publish hook) returns token -1, and the next call at the
    same position gives the allocating path's result again.
The file is named so that pytest collects it last.
"""
import ctypes
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _child():
    sys.path.insert(0, os.path.join(ROOT, "megaqwen-a10_b200"))
    sys.path.insert(0, ROOT)
    import torch
    import megaqwen_b200 as mq
    from megaqwen_b200 import _lib
    from megaqwen_b200.decoder import layer_lists

    L, max_seq = 2, 64
    torch.cuda.init()
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
    torch.cuda.synchronize()

    def static_call(tok, pos):
        rc = lib.launch_a10_int8_decode_static(
            tok, p(out2), p(dec.embed_weight_), p(dec.d_layer_weights_), p(dec.final_norm_weight_),
            p(dec.lm_head_weight_), p(dec.lm_head_scale_), p(dec.cos_table_), p(dec.sin_table_), p(kc2), p(vc2),
            p(norm2), L, pos, pos + 1, max_seq, ctypes.c_float(dec.attn_scale_), p(dec.d_layer_scales_), stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        return int(out2.item())

    # 1. static entry point first, two steps in a row
    toks, norms = [], []
    tok = 23
    static_call(tok, 0)                       # set-up call (first call on the device)
    free0 = torch.cuda.mem_get_info()[0]
    for pos in range(2):
        tok_s = static_call(tok, pos)
        toks.append(tok_s)
        norms.append(norm2.clone())
        tok = tok_s
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, ("device memory changed across static calls", free0, free1)
    assert not _lib.library_info()["workspace_allocated"], "static calls created the allocating workspace"

    # 2. a static call whose bounded wait runs out reports -1; the next call recovers
    _lib.set_wait_budget_ns(2_000_000)
    _lib.inject_skip_publish(True, 3)
    bad = static_call(toks[-1], 2)
    _lib.set_wait_budget_ns(2_000_000_000)
    assert bad == -1, bad
    tok_after = static_call(toks[-1], 2)

    # 3. the allocating entry point on identical inputs: bitwise equal results
    tok = 23
    for pos in range(2):
        ref = dec.decode_step_reference_abi(tok)
        assert ref == toks[pos], (pos, ref, toks[pos])
        assert torch.equal(dec.normalized, norms[pos]), pos
        tok = ref
    ref3 = dec.decode_step_reference_abi(tok)
    assert ref3 == tok_after, (ref3, tok_after)
    assert torch.equal(dec.normalized, norm2)
    assert torch.equal(dec.k_cache[:, :, :3], kc2[:, :, :3])
    assert torch.equal(dec.v_cache[:, :, :3], vc2[:, :, :3])
    dec.check_device()
    print("no-alloc child ok")


def test_static_workspace_entry_matches_allocating_entry_and_allocates_nothing():
    r = subprocess.run([sys.executable, os.path.abspath(__file__), "--child"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT)
    assert r.returncode == 0 and "no-alloc child ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]


def test_static_workspace_entry_rejects_too_many_layers():
    import torch
    from megaqwen_b200 import _lib
    lib = _lib.load()
    n = ctypes.c_void_p(0)
    dummy = torch.zeros(16, dtype=torch.uint8, device="cuda")
    d = ctypes.c_void_p(dummy.data_ptr())
    rc = lib.launch_a10_int8_decode_static(0, d, d, d, d, d, d, d, d, d, d, n, 33, 0, 1, 64,
                                           ctypes.c_float(0.1), d, n)
    assert rc == -5  # MQ_ERR_SIZE


if __name__ == "__main__" and "--child" in sys.argv:
    _child()
