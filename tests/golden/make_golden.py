"""Generate tests/golden/golden.pt by running the REFERENCE's own Python code.

Run in a container that has the reference checkout ($MQ_REFERENCE_DIR, else a
directory named "reference" beside this repository):  python tests/golden/make_golden.py
The fixture is committed; the GPU box never needs the reference.

What is recorded (all on the CPU, seeded):
  1. quantizer   -- bench_int8.quantize_per_channel (bench_int8.py:19-24) on
                    seeded bf16 matrices and hand-made edge rows (all-zero row,
                    single outlier, exact .5 quotients, negative extremes).
  2. rope        -- verify_correctness_a10.precompute_rope_freqs
                    (verify_correctness_a10.py:23-33), theta 1e6, 64 positions.
  3. decoder     -- int8_decoder.QwenDecoder.decode_step (int8_decoder.py:263-298)
                    on a 2-layer synthetic model (seed 0).  QwenDecoder.__init__
                    needs HF weights and CUDA, so the object is built with
                    __new__ and its attributes are set from the synthetic state;
                    its Triton int8_gemv is replaced by the CPU statement of the
                    same math (scale * (int8 W as fp32 @ fp16 x)); its RoPE
                    tables are the HF/theta-1e6 tables of (2).  Recorded per
                    step: the token, the final RMSNorm output and the top-32
                    logits with their indices.
"""
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("MQ_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
sys.dont_write_bytecode = True
sys.path.insert(0, os.path.join(ROOT, "megaqwen-a10_b200"))
sys.path.insert(0, REF)

QUANT_SEED = 1234
DECODER_SEED = 0
DECODER_LAYERS = 2
DECODER_STEPS = 8
START_TOKEN = 17


def quant_cases():
    g = torch.Generator().manual_seed(QUANT_SEED)
    cases = {}
    w = torch.randn(64, 1024, generator=g) * 0.02
    w[torch.rand(64, 1024, generator=g) < 1e-3] *= 20
    cases["seeded_64x1024"] = w.to(torch.bfloat16)
    w = torch.randn(16, 3072, generator=g) * 0.02
    cases["seeded_16x3072"] = w.to(torch.bfloat16)
    e = torch.zeros(6, 1024)
    e[1, 5] = 3.0                                   # single outlier, rest zero
    e[2] = torch.linspace(-1.0, 1.0, 1024)          # symmetric ramp
    e[3, :] = -0.5; e[3, 7] = 0.25                  # negative extreme row
    e[4] = (torch.arange(1024) % 255 - 127) / 127.0 * 0.254   # exact .5 quotient candidates
    e[5] = torch.randn(1024, generator=g) * 1e-30   # denormal-range magnitudes
    cases["edge_rows"] = e.to(torch.bfloat16)
    return cases


def main():
    import bench_int8
    import int8_decoder
    import verify_correctness_a10
    from megaqwen_b200.synth import make_synthetic_state

    out = {"meta": {"reference": "Yunle-Lee/MegaQwen-A10", "torch": torch.__version__}}
    q = {}
    for name, w in quant_cases().items():
        qi, sc = bench_int8.quantize_per_channel(w)
        q[name] = {"w": w, "q": qi, "scale": sc}
    out["quant"] = q

    cos, sin = verify_correctness_a10.precompute_rope_freqs(128, 64, theta=1000000.0, device="cpu")
    out["rope"] = {"cos": cos, "sin": sin, "theta": 1e6, "max_seq_len": 64}

    # --- reference decoder on the CPU ---
    int8_decoder.NUM_LAYERS = DECODER_LAYERS
    int8_decoder.MAX_SEQ_LEN = 64
    int8_decoder.int8_gemv = lambda x, w, s: (w.float() @ x.float()) * s
    state = make_synthetic_state(seed=DECODER_SEED, num_layers=DECODER_LAYERS)
    dec = int8_decoder.QwenDecoder.__new__(int8_decoder.QwenDecoder)
    dec.device = torch.device("cpu")
    dec.use_int8 = True
    dec.embed_weight = state["model.embed_tokens.weight"]
    qpc = int8_decoder.quantize_per_channel
    dec.layers = []
    for i in range(DECODER_LAYERS):
        p = f"model.layers.{i}"
        ow, gw, uw, dw = (state[f"{p}.{n}.weight"] for n in ("self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj",
                                                            "mlp.down_proj"))
        dec.layers.append(int8_decoder.LayerData(
            input_layernorm_weight=state[f"{p}.input_layernorm.weight"],
            q_norm_weight=state[f"{p}.self_attn.q_norm.weight"],
            k_norm_weight=state[f"{p}.self_attn.k_norm.weight"],
            post_attention_layernorm_weight=state[f"{p}.post_attention_layernorm.weight"],
            q_proj_weight=state[f"{p}.self_attn.q_proj.weight"],
            k_proj_weight=state[f"{p}.self_attn.k_proj.weight"],
            v_proj_weight=state[f"{p}.self_attn.v_proj.weight"],
            o_proj_int8=qpc(ow)[0], o_proj_scale=qpc(ow)[1], o_proj_weight=ow,
            gate_proj_int8=qpc(gw)[0], gate_proj_scale=qpc(gw)[1], gate_proj_weight=gw,
            up_proj_int8=qpc(uw)[0], up_proj_scale=qpc(uw)[1], up_proj_weight=uw,
            down_proj_int8=qpc(dw)[0], down_proj_scale=qpc(dw)[1], down_proj_weight=dw))
    dec.final_norm_weight = state["model.norm.weight"]
    dec.lm_head_weight = state["model.embed_tokens.weight"]
    dec.lm_head_int8, dec.lm_head_scale = qpc(dec.lm_head_weight)
    dec.cos_table, dec.sin_table = cos, sin
    dec._reset_state()

    captured = {}
    orig_rms = dec.rmsnorm

    def rms_capture(x, w):
        y = orig_rms(x, w)
        if w is dec.final_norm_weight:
            captured["normalized"] = y.clone()
        return y

    orig_mv = dec._matvec

    def mv_capture(x, w16, w8=None, s=None):
        y = orig_mv(x, w16, w8, s)
        if w8 is dec.lm_head_int8:
            captured["logits"] = y.clone()
        return y

    dec.rmsnorm = rms_capture
    dec._matvec = mv_capture
    toks, norms, topv, topi = [], [], [], []
    t = START_TOKEN
    for _ in range(DECODER_STEPS):
        t = dec.decode_step(t)
        toks.append(t)
        norms.append(captured["normalized"])
        v, i = captured["logits"].topk(32)
        topv.append(v)
        topi.append(i)
    out["decoder"] = {"seed": DECODER_SEED, "layers": DECODER_LAYERS, "start": START_TOKEN, "tokens": toks,
                      "normalized": torch.stack(norms), "top_vals": torch.stack(topv), "top_idx": torch.stack(topi)}
    path = os.path.join(HERE, "golden.pt")
    torch.save(out, path)
    print("wrote", path, os.path.getsize(path), "bytes; tokens", toks)


if __name__ == "__main__":
    main()
