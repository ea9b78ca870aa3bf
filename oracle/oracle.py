"""CPU oracle for the Qwen3-0.6B decode path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU baseline.
The product (megaqwen-a10_b200/) never imports it.

It restates, in plain PyTorch on the CPU, the reference's formulation of the
decode math (Yunle-Lee/MegaQwen-A10):
  * quantize_per_channel      bench_int8.py:19-24 (= int8_decoder.py:45-56)
  * rope_tables               verify_correctness_a10.py:23-33 (HF layout, theta 1e6)
  * rmsnorm                   int8_decoder.py:228-232
  * apply_rope                int8_decoder.py:234-240 (split half, cos[:64])
  * attention                 int8_decoder.py:242-255 (GQA kvh = qh // 2)
  * decode_step               int8_decoder.py:263-298
  * int8 matvec               int8_gemv semantics, int8_decoder.py:100-115:
                              y = scale * (int8 W as fp32 @ x)
Switches select between the reference's two formulations:
  * qkv_int8      -- True: q/k/v are INT8 like every other projection
                     (bench_int8.py:36-51, the kernel being reproduced);
                     False: bf16 q/k/v as in QwenDecoder (int8_decoder.py:268-270).
  * act_half      -- True: activations cast to fp16 before an INT8 matvec, as
                     QwenDecoder._matvec does (int8_decoder.py:259); False: fp32,
                     as the CUDA kernels do (a10_int8_decode_kernel.cu:119-130).
  * bf16_hidden   -- True: the residual stream is rounded to bf16 after the
                     embedding and after every layer, as the kernel does
                     (a10_int8_decode_kernel.cu:30, :571); False: fp32 as in
                     QwenDecoder.
The product kernel corresponds to qkv_int8=True, act_half=False, bf16_hidden=True
(the default).  The reference-module configuration (False, True, False) is what
tests/golden/make_golden.py pins against the reference's own QwenDecoder.
"""
import torch
import torch.nn.functional as F

HIDDEN_SIZE = 1024
INTERMEDIATE_SIZE = 3072
NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128
Q_SIZE = NUM_Q_HEADS * HEAD_DIM
KV_SIZE = NUM_KV_HEADS * HEAD_DIM
VOCAB_SIZE = 151936
RMS_EPS = 1e-6
PROJS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
         "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def quantize_per_channel(tensor):
    """bench_int8.py:19-24.  `tensor` bf16 [M, K] -> (int8 [M, K], fp32 [M]).
    absmax stays bf16, so absmax / 127.0 is a bf16 quotient."""
    max_abs = tensor.abs().amax(dim=1)
    scale = (max_abs / 127.0).to(torch.float32).clamp(min=1e-12)
    w_int8 = (tensor / scale.view(-1, 1)).round().clamp(-128, 127).to(torch.int8)
    return w_int8, scale


def rope_tables(max_seq_len, head_dim=HEAD_DIM, theta=1_000_000.0):
    """verify_correctness_a10.py:23-33 on the CPU."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    cos = freqs.cos().to(torch.bfloat16)
    sin = freqs.sin().to(torch.bfloat16)
    return torch.cat([cos, cos], dim=-1), torch.cat([sin, sin], dim=-1)


def rmsnorm(x, weight, eps=RMS_EPS):
    """int8_decoder.py:228-232."""
    x_f = x.float()
    rstd = (x_f.pow(2).mean() + eps).rsqrt()
    return x_f * rstd * weight.float()


def apply_rope(x, cos_row, sin_row):
    """int8_decoder.py:234-240: [x1*c - x2*s, x1*s + x2*c] with c, s = cos[:64], sin[:64]."""
    half = HEAD_DIM // 2
    c, s = cos_row[:half], sin_row[:half]
    x1, x2 = x[:half], x[half:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c])


def matvec_int8(x, q, scale, act_half=False):
    """y = scale * (fp32(q) @ x); with act_half x is rounded to fp16 first."""
    xx = x.half().float() if act_half else x.float()
    return (q.float() @ xx) * scale


def matvec_bf16(x, w):
    """QwenDecoder._matvec bf16 branch, int8_decoder.py:260."""
    return (x.bfloat16() @ w.T).float()


class OracleDecoder:
    """Single-sequence greedy decoder on the CPU over an HF-named bf16 state.

    quantized=True: INT8 weight-only (per the switches above); quantized=False:
    every projection and the LM head in bf16 (the BF16 kernel's math: bf16
    weights, fp32 activations and accumulation)."""

    def __init__(self, state, num_layers, max_seq_len=256, quantized=True, qkv_int8=True, act_half=False,
                 bf16_hidden=True, rope_theta=1_000_000.0, threads=None):
        if threads:
            torch.set_num_threads(threads)
        self.L = num_layers
        self.max_seq_len = max_seq_len
        self.quantized = quantized
        self.qkv_int8 = qkv_int8
        self.act_half = act_half
        self.bf16_hidden = bf16_hidden
        self.embed = state["model.embed_tokens.weight"]
        lm = state.get("lm_head.weight", self.embed)
        self.final_norm = state["model.norm.weight"]
        self.layers = []
        for i in range(num_layers):
            p = f"model.layers.{i}"
            d = {k: state[f"{p}.{k}.weight"] for k in ("input_layernorm", "post_attention_layernorm",
                                                      "self_attn.q_norm", "self_attn.k_norm")}
            for proj in PROJS:
                w = state[f"{p}.{proj}.weight"]
                if quantized and (qkv_int8 or proj not in PROJS[:3]):
                    q, s = quantize_per_channel(w)
                    d[proj] = ("int8", q.float(), s)   # fp32 copy of the int8 codes
                else:
                    # fp32 copy of the bf16 weights, made once: the BF16 kernel's
                    # math (bf16 weights, fp32 activations and accumulation) on
                    # exactly representable values; converting per step would only be slower
                    d[proj] = ("bf16", w.float() if not quantized else w, None)
            self.layers.append(d)
        if quantized:
            q, s = quantize_per_channel(lm)
            self.lm = ("int8", q.float(), s)
        else:
            self.lm = ("bf16", lm.float(), None)
        self.cos, self.sin = rope_tables(max_seq_len, theta=rope_theta)
        self.reset()

    def reset(self):
        self.position = 0
        shape = (self.L, NUM_KV_HEADS, self.max_seq_len, HEAD_DIM)
        self.k_cache = torch.zeros(shape, dtype=torch.bfloat16)
        self.v_cache = torch.zeros(shape, dtype=torch.bfloat16)

    def _mv(self, x, spec):
        kind, w, s = spec
        if kind == "int8":
            xx = x.half().float() if self.act_half else x.float()
            return (w @ xx) * s
        if self.quantized:
            return matvec_bf16(x, w)            # QwenDecoder's bf16 q/k/v
        return w @ x.float()                    # BF16 kernel: fp32 weights (exact bf16) x fp32 activations

    def attention(self, q_rope, li, cache_len):
        """int8_decoder.py:242-255."""
        out = torch.zeros(Q_SIZE, dtype=torch.float32)
        gqa = NUM_Q_HEADS // NUM_KV_HEADS
        for qh in range(NUM_Q_HEADS):
            kvh = qh // gqa
            s = qh * HEAD_DIM
            q_h = q_rope[s:s + HEAD_DIM]
            k_h = self.k_cache[li, kvh, :cache_len, :].float()
            v_h = self.v_cache[li, kvh, :cache_len, :].float()
            scores = q_h @ k_h.T * (HEAD_DIM ** -0.5)
            e = torch.exp(scores - scores.max())
            out[s:s + HEAD_DIM] = (e @ v_h) / e.sum()
        return out

    @torch.no_grad()
    def step(self, token_id, want_logits=False):
        """int8_decoder.py:263-298.  Returns (token, logits or None, per-layer hidden list)."""
        pos = self.position
        if pos >= self.max_seq_len:
            raise ValueError("KV cache full")
        rnd = (lambda t: t.bfloat16().float()) if self.bf16_hidden else (lambda t: t)
        hidden = self.embed[token_id].float()
        hiddens = []
        for li in range(self.L):
            ld = self.layers[li]
            normalized = rmsnorm(hidden, ld["input_layernorm"])
            q = self._mv(normalized, ld["self_attn.q_proj"])
            k = self._mv(normalized, ld["self_attn.k_proj"])
            v = self._mv(normalized, ld["self_attn.v_proj"])
            residual = hidden
            q_rope = torch.empty_like(q)
            k_rope = torch.empty_like(k)
            for h in range(NUM_Q_HEADS):
                s = h * HEAD_DIM
                q_rope[s:s + HEAD_DIM] = apply_rope(rmsnorm(q[s:s + HEAD_DIM], ld["self_attn.q_norm"]),
                                                    self.cos[pos], self.sin[pos])
            for h in range(NUM_KV_HEADS):
                s = h * HEAD_DIM
                k_rope[s:s + HEAD_DIM] = apply_rope(rmsnorm(k[s:s + HEAD_DIM], ld["self_attn.k_norm"]),
                                                    self.cos[pos], self.sin[pos])
            self.k_cache[li, :, pos, :] = k_rope.view(NUM_KV_HEADS, HEAD_DIM)
            self.v_cache[li, :, pos, :] = v.view(NUM_KV_HEADS, HEAD_DIM)
            attn = self.attention(q_rope, li, pos + 1)
            hidden = residual + self._mv(attn, ld["self_attn.o_proj"])
            normalized = rmsnorm(hidden, ld["post_attention_layernorm"])
            residual = hidden
            gate = self._mv(normalized, ld["mlp.gate_proj"])
            up = self._mv(normalized, ld["mlp.up_proj"])
            act = F.silu(gate) * up
            hidden = rnd(residual + self._mv(act, ld["mlp.down_proj"]))
            hiddens.append(hidden)
        normalized = rmsnorm(hidden, self.final_norm)
        self.normalized = normalized
        logits = self._mv(normalized, self.lm)
        self.position += 1
        tok = int(logits.argmax().item())
        return tok, (logits if want_logits else None), hiddens

    def decode_step(self, token_id):
        return self.step(token_id)[0]


def rel_err(a, b):
    """int8_decoder.py:504: max|a - b| / max|a| (a = reference)."""
    a, b = a.double().flatten(), b.double().flatten()
    return float((a - b).abs().max() / a.abs().max().clamp_min(1e-30))


def cosine(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    return float((a @ b) / (a.norm() * b.norm()).clamp_min(1e-30))


def greedy_reference(state, num_layers, start_token, steps, **kw):
    """Greedy token sequence of `steps` steps from `start_token` at position 0."""
    o = OracleDecoder(state, num_layers, max_seq_len=max(steps + 1, 2), **kw)
    toks, t = [], start_token
    for _ in range(steps):
        t = o.decode_step(t)
        toks.append(t)
    return toks


def bytes_per_step_int8(num_layers, cache_len):
    """Algorithmic HBM bytes of one INT8 batch-1 step: weights + scales + norms +
    embedding row + final norm + KV read of the cache_len-1 cached positions +
    KV write of the new one = 598,101,504 + 114,688 * cache_len for 28 layers."""
    per_layer = (Q_SIZE + 2 * KV_SIZE) * HIDDEN_SIZE + HIDDEN_SIZE * Q_SIZE + 3 * INTERMEDIATE_SIZE * HIDDEN_SIZE
    scales = 4 * (Q_SIZE + 2 * KV_SIZE + HIDDEN_SIZE + 2 * INTERMEDIATE_SIZE + HIDDEN_SIZE)
    norms = 2 * (2 * HIDDEN_SIZE + 2 * HEAD_DIM)
    lm = VOCAB_SIZE * HIDDEN_SIZE + 4 * VOCAB_SIZE
    kv = 2 * NUM_KV_HEADS * HEAD_DIM * 2  # K+V bytes per position per layer
    return num_layers * (per_layer + scales + norms + kv * (cache_len - 1) + kv) + lm + 2 * HIDDEN_SIZE * 2

