"""Qwen3-0.6B shape constants: the single source of truth on the Python side.

Values are those of the reference's config.cuh:30-40 and the module constants
repeated in bench_int8.py:11-16 / a10_decode.py:16-26.  The CUDA side keeps the
same numbers as constexprs in csrc/common.cuh.
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class Qwen3Config:
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_q_heads: int = 16
    num_kv_heads: int = 8
    head_dim: int = 128
    num_layers: int = 28
    vocab_size: int = 151936
    rms_eps: float = 1e-6
    rope_theta: float = 1e6
    max_seq_len: int = 2048

    @property
    def q_size(self):
        return self.num_q_heads * self.head_dim

    @property
    def kv_size(self):
        return self.num_kv_heads * self.head_dim


CFG = Qwen3Config()
HIDDEN_SIZE = CFG.hidden_size
INTERMEDIATE_SIZE = CFG.intermediate_size
NUM_Q_HEADS = CFG.num_q_heads
NUM_KV_HEADS = CFG.num_kv_heads
HEAD_DIM = CFG.head_dim
Q_SIZE = CFG.q_size
KV_SIZE = CFG.kv_size
NUM_LAYERS = CFG.num_layers
VOCAB_SIZE = CFG.vocab_size
MAX_SEQ_LEN = CFG.max_seq_len
RMS_EPS = CFG.rms_eps

# Order of the 11 per-layer tensors in the flat weight list the decoder
# constructors take (bench_int8.py:291-320, config.cuh:45-57).
LAYER_TENSOR_ORDER = (
    "input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm",
    "o_proj", "post_attention_layernorm", "gate_proj", "up_proj", "down_proj",
)
# Order of the 7 per-layer scale tensors (bench_int8.py:322-330, config.cuh:59-67).
LAYER_SCALE_ORDER = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
