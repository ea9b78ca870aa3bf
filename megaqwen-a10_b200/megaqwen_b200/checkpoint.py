"""Checkpoint I/O for the decoder: an HF Qwen3 checkpoint (safetensors, one file
or an index of shards) -> bf16 state dict, and the quantized state (INT8 codes +
fp32 scales) to and from one safetensors file, so that startup quantization can
be skipped.

The reference loads weights through transformers' from_pretrained
(a10_decode.py:281-327) and re-quantizes at every start (load_quantized_state,
bench_int8.py:27-55).  Here the safetensors files are read directly; only the
tensors the decoder uses are kept.
"""
import json
import os

import torch
from safetensors import safe_open
from safetensors.torch import save_file

from .config import NUM_LAYERS

QUANT_FORMAT = "megaqwen-int8-per-channel-v1"
_PROJ = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
         "mlp.up_proj", "mlp.down_proj")
_NORMS = ("input_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
          "post_attention_layernorm.weight")


def needed_keys(num_layers=NUM_LAYERS):
    """State-dict names the decoder reads (lm_head.weight is optional: tied embeddings)."""
    keys = ["model.embed_tokens.weight", "model.norm.weight"]
    for i in range(num_layers):
        p = f"model.layers.{i}"
        keys += [f"{p}.{proj}.weight" for proj in _PROJ] + [f"{p}.{n}" for n in _NORMS]
    return keys


def _files(path):
    if os.path.isfile(path):
        return [path]
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, s) for s in shards]
    single = os.path.join(path, "model.safetensors")
    if os.path.exists(single):
        return [single]
    raise FileNotFoundError(f"no model.safetensors or model.safetensors.index.json under {path}")


def load_state(path, num_layers=NUM_LAYERS, dtype=torch.bfloat16, device="cpu"):
    """HF Qwen3 checkpoint (file or directory) -> {name: tensor} with the decoder's
    tensors in `dtype`.  Raises KeyError naming the first missing tensor."""
    want = set(needed_keys(num_layers)) | {"lm_head.weight"}
    state = {}
    for fn in _files(path):
        with safe_open(fn, framework="pt", device="cpu") as f:
            for k in f.keys():
                if k in want:
                    state[k] = f.get_tensor(k).to(dtype).to(device)
    for k in needed_keys(num_layers):
        if k not in state:
            raise KeyError(f"checkpoint lacks {k}")
    return state


def save_quantized(q, path, num_layers=NUM_LAYERS):
    """Quantized state (quantize_state's output: (int8, fp32 scale) tuples for the
    projections and the LM head, bf16 tensors otherwise) -> one safetensors file."""
    flat = {}
    for k, v in q.items():
        if isinstance(v, tuple):
            flat[k + ".qweight"] = v[0].contiguous().cpu()
            flat[k + ".scale"] = v[1].contiguous().cpu()
        else:
            flat[k] = v.contiguous().cpu()
    save_file(flat, path, metadata={"format": QUANT_FORMAT, "num_layers": str(num_layers)})


def load_quantized(path, device="cpu"):
    """The inverse of save_quantized: {name: tensor or (int8, fp32 scale)}."""
    q = {}
    with safe_open(path, framework="pt", device="cpu") as f:
        meta = f.metadata() or {}
        if meta.get("format") != QUANT_FORMAT:
            raise ValueError(f"{path}: not a {QUANT_FORMAT} file")
        names = list(f.keys())
        for k in names:
            if k.endswith(".scale"):
                continue
            if k.endswith(".qweight"):
                base = k[: -len(".qweight")]
                q[base] = (f.get_tensor(k).to(device), f.get_tensor(base + ".scale").to(device))
            else:
                q[k] = f.get_tensor(k).to(device)
    return q, int(meta.get("num_layers", NUM_LAYERS))


__all__ = ["load_state", "save_quantized", "load_quantized", "needed_keys", "QUANT_FORMAT"]
