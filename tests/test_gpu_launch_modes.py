"""GPU: the two launch modes of the batch-1 decode step give identical results.

By default a step is a plain launch of one CTA per SM with programmatic stream
serialisation (the next step's read-only prologue overlaps the previous step's
tail; the kernel waits on griddepcontrol.wait before reading anything the
previous step wrote).  MQ_COOPERATIVE=1 selects a cooperative launch without
that overlap.  The launch mode is read once per process, so each mode runs in
a child process; both decode the same 2-layer model for 24 steps with on-device
token feedback, then 4 host-synchronous decode_step calls, and the tokens, the
last logits and the KV cache must be bitwise equal.
"""
import hashlib
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
    from megaqwen_b200.decoder import layer_lists
    L, max_seq = 2, 64
    st = mq.make_synthetic_state(seed=3, num_layers=L)
    q = mq.quantize_state(st, num_layers=L, device="cuda")
    layers, scales = layer_lists(q, L, True)
    cos, sin = mq.make_rope(max_seq, device="cuda")
    dec = mq.A10Int8MegakernelDecoder(q["model.embed_tokens.weight"], layers, scales, *q["lm_head.weight"],
                                      q["model.norm.weight"], cos, sin, L, max_seq)
    logits = torch.empty(mq.CFG.vocab_size, dtype=torch.float32, device="cuda")
    toks = dec.decode_steps(41, 24, logits=logits).cpu().tolist()
    tok = toks[-1]
    for _ in range(4):
        tok = dec.decode_step(tok)
        toks.append(tok)
    dec.check_device()
    h = hashlib.sha256()
    for t in (logits, dec.k_cache, dec.v_cache):
        h.update(t.contiguous().view(torch.uint8).cpu().numpy().tobytes())
    print("RESULT", toks, h.hexdigest())


def _run(env_extra):
    env = dict(os.environ)
    env.pop("MQ_COOPERATIVE", None)
    env.update(env_extra)
    r = subprocess.run([sys.executable, os.path.abspath(__file__), "--child"], capture_output=True, text=True,
                       timeout=600, cwd=ROOT, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")][-1]


def test_programmatic_and_cooperative_launch_bitwise_equal():
    a = _run({})
    b = _run({"MQ_COOPERATIVE": "1"})
    assert a == b, (a[:200], b[:200])


if __name__ == "__main__" and "--child" in sys.argv:
    _child()
