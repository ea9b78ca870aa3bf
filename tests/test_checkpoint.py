"""CPU: checkpoint I/O (megaqwen_b200/checkpoint.py) -- reading an HF-style
safetensors checkpoint (single file and sharded index) and the quantized-state
file round trip, bit-exact; GPU: a decoder built from the checkpoint directory
(quantizing, then from the saved quantized file) decodes the same tokens as one
built from the in-memory state."""
import json
import os

import pytest
import torch
from safetensors.torch import save_file

import megaqwen_b200 as mq
from megaqwen_b200 import checkpoint as ck


def _write_ckpt(state, d, shards=1):
    keys = sorted(state)
    if shards == 1:
        save_file({k: state[k].contiguous() for k in keys}, os.path.join(d, "model.safetensors"))
        return
    wm = {}
    for s in range(shards):
        part = keys[s::shards]
        name = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        save_file({k: state[k].contiguous() for k in part}, os.path.join(d, name))
        wm.update({k: name for k in part})
    with open(os.path.join(d, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)


@pytest.mark.parametrize("shards", [1, 3])
def test_load_state_roundtrip(tmp_path, shards):
    st = mq.make_synthetic_state(seed=2, num_layers=2)
    st["extra.unused"] = torch.zeros(3)   # ignored
    _write_ckpt(st, str(tmp_path), shards)
    got = ck.load_state(str(tmp_path), num_layers=2)
    for k in ck.needed_keys(2):
        assert torch.equal(got[k], st[k].to(torch.bfloat16)), k
    assert "extra.unused" not in got


def test_load_state_missing_tensor(tmp_path):
    st = mq.make_synthetic_state(seed=2, num_layers=2)
    del st["model.layers.1.mlp.down_proj.weight"]
    _write_ckpt(st, str(tmp_path))
    with pytest.raises(KeyError):
        ck.load_state(str(tmp_path), num_layers=2)


def test_quantized_file_roundtrip(tmp_path):
    g = torch.Generator().manual_seed(0)
    q = {"model.layers.0.self_attn.q_proj.weight": (torch.randint(-128, 128, (32, 64), generator=g, dtype=torch.int8),
                                                   torch.rand(32, generator=g)),
         "model.norm.weight": torch.randn(64, generator=g).to(torch.bfloat16)}
    p = str(tmp_path / "q.safetensors")
    ck.save_quantized(q, p, num_layers=1)
    back, n = ck.load_quantized(p)
    assert n == 1
    a, b = q["model.layers.0.self_attn.q_proj.weight"], back["model.layers.0.self_attn.q_proj.weight"]
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) and b[0].dtype == torch.int8
    assert torch.equal(q["model.norm.weight"], back["model.norm.weight"])


def test_load_quantized_rejects_other_files(tmp_path):
    p = str(tmp_path / "x.safetensors")
    save_file({"a": torch.zeros(2)}, p)
    with pytest.raises(ValueError):
        ck.load_quantized(p)


@pytest.mark.gpu
def test_from_pretrained_decodes_like_in_memory(tmp_path):
    L = 2
    st = mq.make_synthetic_state(seed=4, num_layers=L)
    _write_ckpt(st, str(tmp_path))
    qp = str(tmp_path / "quant.safetensors")
    ref = mq.A10Decoder(st, quantized=True, max_seq_len=64, num_layers=L)
    a = mq.A10Decoder.from_pretrained(str(tmp_path), max_seq_len=64, num_layers=L, quantized_path=qp)
    assert os.path.exists(qp)
    b = mq.A10Decoder.from_pretrained(str(tmp_path), max_seq_len=64, num_layers=L, quantized_path=qp)
    prompt = [11, 22, 33, 44]
    want = ref.generate(prompt, max_new_tokens=6)
    assert a.generate(prompt, max_new_tokens=6) == want
    assert b.generate(prompt, max_new_tokens=6) == want
    # the reference's constructor shape: A10Decoder(model_path, max_seq_len)
    c = mq.A10Decoder(str(tmp_path), 64, num_layers=L)
    assert c.max_seq_len == 64 and c.generate(prompt, max_new_tokens=6) == want


@pytest.mark.gpu
def test_stream_yields_generate_tokens():
    st = mq.make_synthetic_state(seed=5, num_layers=2)
    d = mq.A10Decoder(st, quantized=True, max_seq_len=64, num_layers=2)
    prompt = [3, 1, 4, 1, 5]
    full = d.generate(prompt, max_new_tokens=7)
    assert list(d.stream(prompt, max_new_tokens=7)) == full[len(prompt):]
