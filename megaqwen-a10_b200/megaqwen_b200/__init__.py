"""megaqwen_b200 -- B200 (sm_100a) fused Qwen3-0.6B decode, INT8 weight-only and BF16.

The compute runs in the in-tree CUDA library lib/libmqb200.so (C ABI:
include/megaqwen_b200.h).  This package is the Python surface that mirrors the
reference's decoder wrappers.
"""
from .config import CFG, Qwen3Config
from .quant import quantize_per_channel, quantize_state
from .rope import make_rope
from .synth import make_synthetic_state
from .decoder import A10Decoder, A10Int8MegakernelDecoder, A10MegakernelDecoder, layer_lists
from .batch import BatchedDecoder, batch_matmul, pack_tiles
from . import _lib, checkpoint
from ._lib import MQError
from .chat import A10Chat

__all__ = ["CFG", "Qwen3Config", "quantize_per_channel", "quantize_state", "make_rope", "make_synthetic_state",
           "A10Decoder", "A10Int8MegakernelDecoder", "A10MegakernelDecoder", "BatchedDecoder", "batch_matmul", "pack_tiles", "layer_lists",
           "MQError", "A10Chat"]
