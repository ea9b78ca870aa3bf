"""RoPE tables in the HuggingFace layout the kernel's split-half rotation needs.

Follows precompute_rope_freqs (verify_correctness_a10.py:23-33): inv_freq =
theta^(-arange(0, d, 2)/d) in fp32, freqs = outer(positions, inv_freq), cos/sin
rounded to bf16, then each duplicated as cat([c, c]).  theta defaults to 1e6
(Qwen3).  The reference's benchmark scripts build theta=1e4 tables with a
pair-duplicated layout (bench_int8.py:270-279) that does not match the kernel's
rotation; that layout is deliberately not reproduced.  Tables are computed on
the CPU (deterministic) and then moved to `device`.
"""
import torch


def make_rope(max_seq_len, head_dim=128, device="cuda", theta=1_000_000.0):
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    cos = freqs.cos().to(torch.bfloat16)
    sin = freqs.sin().to(torch.bfloat16)
    cos = torch.cat([cos, cos], dim=-1).contiguous()
    sin = torch.cat([sin, sin], dim=-1).contiguous()
    return cos.to(device), sin.to(device)
