"""Per-output-channel symmetric INT8 quantization on the GPU.

Same arithmetic as quantize_per_channel (bench_int8.py:19-24): scale[j] =
fp32(bf16(absmax(W[j,:]) / 127)) clamped to >= 1e-12, q = clamp(round_half_even(
fp32(W)/scale), -128, 127).  Runs the CUDA kernel in csrc/quantize.cu; a
non-CUDA input raises instead of falling back to a CPU path.
"""
import ctypes

import torch

from . import _lib
from .config import NUM_LAYERS, LAYER_SCALE_ORDER


def quantize_per_channel(tensor):
    """tensor: bf16 [M, K] on a CUDA device -> (int8 [M, K], fp32 [M])."""
    if not tensor.is_cuda:
        raise ValueError("quantize_per_channel needs a CUDA tensor (no CPU path in this library)")
    if tensor.dtype != torch.bfloat16 or tensor.dim() != 2:
        raise ValueError(f"expected a 2-D bf16 tensor, got {tensor.dtype} {tuple(tensor.shape)}")
    w = tensor.contiguous()
    M, K = w.shape
    q = torch.empty((M, K), dtype=torch.int8, device=w.device)
    s = torch.empty((M,), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        stream = torch.cuda.current_stream(w.device).cuda_stream
        rc = _lib.load().mq_quantize_per_channel(ctypes.c_void_p(w.data_ptr()), M, K, ctypes.c_void_p(q.data_ptr()),
                                                  ctypes.c_void_p(s.data_ptr()), ctypes.c_void_p(stream))
    _lib.check(rc, "mq_quantize_per_channel")
    return q, s


def quantize_state(state, num_layers=NUM_LAYERS, device="cuda"):
    """HF-named bf16 state dict -> the quantized state of load_quantized_state
    (bench_int8.py:27-55): projections and the LM head become (int8, scale)
    tuples, norms and the embedding stay bf16.  A missing lm_head.weight means
    tied embeddings: the LM head is quantized from the embedding."""
    q = {}
    for i in range(num_layers):
        p = f"model.layers.{i}"
        for proj in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                     "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"):
            q[f"{p}.{proj}.weight"] = quantize_per_channel(state[f"{p}.{proj}.weight"].to(device))
        for other in ("input_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                      "post_attention_layernorm.weight"):
            q[f"{p}.{other}"] = state[f"{p}.{other}"].to(device)
    lm = state.get("lm_head.weight", state["model.embed_tokens.weight"])
    q["lm_head.weight"] = quantize_per_channel(lm.to(device))
    q["model.embed_tokens.weight"] = state["model.embed_tokens.weight"].to(device)
    q["model.norm.weight"] = state["model.norm.weight"].to(device)
    return q


__all__ = ["quantize_per_channel", "quantize_state", "LAYER_SCALE_ORDER"]
