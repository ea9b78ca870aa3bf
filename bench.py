"""Benchmark: batch-1 INT8 greedy decode of Qwen3-0.6B on B200.

Workload: 28 layers, INT8 weight-only on all projections and
the LM head, seeded synthetic weights N(0, 0.02) with 0.1 % x20 outliers, one
start token, decode positions 0..K-1 (K = --steps, default 200).  A "step" is
one decoded token.  Weights (621 MB/step) are far larger than L2 (126 MB), so
every step streams them from HBM; no extra flush is needed.

  value   tokens/s with everything resident on the GPU: K steps with on-device
          token feedback (mq_decode_multi), CUDA events on the launching stream.
  e2e     the same tokens/s through the reference-facing call
          A10Int8MegakernelDecoder.decode_step(token) -> int, which passes the
          token to the kernel and reads the argmax back into host memory every
          step (the kernel writes it into pinned memory; stream synchronise).
  --impl reference   the reference's PyTorch formulation of the same math
          (oracle/oracle.py, a CPU restatement of int8_decoder.py:263-298 with
          INT8 on every projection) timed on the host cores.
Multi-GPU (torchrun): the line is config 4 (batched decode, 64 sequences per
GPU) unless --config says otherwise; every rank runs an independent replica (no
collective on the data path); value = all ranks' tokens / max over ranks of
the CUDA-event time.  --config 0/2/3 and --prefill select the other BASELINE
configs on one GPU.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "megaqwen-a10_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "batch-1 INT8 decode tok/s (Qwen3-0.6B, positions 0..K-1)"
BATCHED_METRIC = "batched INT8 decode tok/s (64 sequences per GPU, positions 128..2048)"
BYTES_FIXED = 598_101_504      # INT8 weights + scales + norms + embed row + final norm per step
BYTES_PER_POS = 114_688        # K+V bytes per cached position over 28 layers


def max_over_ranks(x, dist, device="cuda"):
    """The maximum of a per-rank float over all ranks (x itself without a process group).
    device: "cuda" under NCCL, "cpu" under gloo."""
    if not dist:
        return float(x)
    t = torch.tensor([float(x)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def aggregate_tok_s(world, tokens_per_rank, t_max_s):
    """Whole-job throughput: every rank decodes tokens_per_rank tokens; time = max over ranks."""
    return world * tokens_per_rank / t_max_s


def step_bytes(pos):
    return BYTES_FIXED + BYTES_PER_POS * (pos + 1)


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    p = os.path.join(ROOT, "profiles", "decode_int8_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("dram_bytes_per_launch")
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 100 ms during the timed region."""
    Q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()
            self.t.join(timeout=2)

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in self.rows:
            try:
                sm.append(float(r[0]))
                mx = float(r[1])
                for n, v in zip(names, r[3:7]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
            except (ValueError, IndexError):
                pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def build_decoder(L, max_seq, seed=0):
    import megaqwen_b200 as mq
    from megaqwen_b200.decoder import layer_lists
    st = mq.make_synthetic_state(seed=seed, num_layers=L)
    q = mq.quantize_state(st, num_layers=L, device="cuda")
    del st
    layers, scales = layer_lists(q, L, True)
    cos, sin = mq.make_rope(max_seq, device="cuda")
    lm_q, lm_s = q["lm_head.weight"]
    return mq.A10Int8MegakernelDecoder(q["model.embed_tokens.weight"], layers, scales, lm_q, lm_s,
                                       q["model.norm.weight"], cos, sin, L, max_seq)


def build_decoder_bf16(L, max_seq, seed=0):
    import megaqwen_b200 as mq
    from megaqwen_b200.decoder import layer_lists
    st = {k: v.to("cuda") for k, v in mq.make_synthetic_state(seed=seed, num_layers=L).items()}
    layers, _ = layer_lists(st, L, False)
    cos, sin = mq.make_rope(max_seq, device="cuda")
    emb = st["model.embed_tokens.weight"]
    return mq.A10MegakernelDecoder(emb, layers, st["model.norm.weight"], emb, cos, sin, L, max_seq)


def run_long_context(args, ctx):
    """one INT8 step at cache length ctx + 1 with a KV cache
    pre-filled with seeded N(0,1) bf16; --steps repetitions of that same step."""
    L, K = args.layers, args.steps
    dec = build_decoder(L, ctx + 8)
    g = torch.Generator(device="cuda").manual_seed(ctx)
    for cache in (dec.k_cache, dec.v_cache):
        cache[:, :, :ctx].normal_(generator=g)
    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        dec.set_position(ctx)
        dec.decode_steps(11, 1)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        a.record(stream)
        for _ in range(K):
            dec.set_position(ctx)
            dec.decode_steps(11, 1)
        b.record(stream)
        torch.cuda.synchronize()
    dec.check_device()
    ms = a.elapsed_time(b) / K
    # end to end: decode_step(int) -> int with the host read-back, same step
    dec.set_position(ctx)
    dec.decode_step(11)
    t0 = time.perf_counter()
    for _ in range(K):
        dec.set_position(ctx)
        dec.decode_step(11)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / K
    alg = BYTES_FIXED + BYTES_PER_POS * (ctx + 1)
    peak, kind = measured_peak()
    ach = alg / (ms / 1000.0) / 1e9
    line = {"metric": f"long-context INT8 single-step decode, cache_len {ctx + 1}", "value": round(1000.0 / ms, 2),
            "unit": "steps/s", "higher_is_better": True, "n_gpus": 1, "ms_per_step": round(ms, 4), "steps": K,
            "dtype": "int8-weights/fp32-accum", "data": "synthetic (seeded weights, seeded N(0,1) bf16 KV)",
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "peak_kind": kind, "kernel": "decode_kernel<W8>",
                         "algorithmic_bytes_per_launch": alg},
            "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "steps/s", "h2d_bytes_per_step": 4,
                    "d2h_bytes_per_step": 4, "api": "A10Int8MegakernelDecoder.decode_step(int) -> int"},
            "config": {"workload": "config3", "context": ctx, "kv": "seeded N(0,1) bf16",
                       "l2": "inputs larger than L2"},
            "clocks": clk.summary(), "gpu_launches": K}
    del dec
    torch.cuda.empty_cache()
    if not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v = cpu_oracle_long_rate(threads, ctx)
        line["cpu_baseline"] = {"value": round(v, 4), "unit": "steps/s", "cores": threads, "kind": "port",
                                "sample": f"one 28-layer step at cache length {ctx + 1} (seeded N(0,1) KV), "
                                          f"oracle/oracle.py on torch CPU"}
    print(json.dumps(line), flush=True)


def run_prefill(args):
    """Chunked prefill (64 tokens per launch on the tensor-core path) of an
    args.prefill-token prompt vs the same prompt fed one decode step per token."""
    n, L = args.prefill, args.layers
    dec = build_decoder(L, n + 8)
    ids = torch.randint(0, 151936, (n,), generator=torch.Generator().manual_seed(5)).tolist()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(max(args.warmup, 3)):
        dec.reset()
        dec.prefill(ids)
    times = []
    for _ in range(max(args.steps, 1)):
        dec.reset()
        torch.cuda.synchronize()
        a.record(stream)
        dec.prefill(ids)
        b.record(stream)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    ms = statistics.median(times)
    dec.reset()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for t in ids:
        dec.decode_step(t)
    step_ms = (time.perf_counter() - t0) * 1000.0
    line = {"metric": "prefill tok/s (chunked, 64 tokens per launch)", "value": round(n / (ms / 1000.0), 1),
            "unit": "tok/s", "n_gpus": 1, "steps": len(times), "warmup": max(args.warmup, 3), "ms": round(ms, 3),
            "higher_is_better": True, "dtype": "int8-weights/fp16-activations/fp32-accum", "data": "synthetic",
            "config": {"workload": f"prefill of a {n}-token prompt, {L} layers", "prompt_tokens": n},
            "stepwise": {"ms": round(step_ms, 3), "tok_s": round(n / (step_ms / 1000.0), 1),
                         "api": "decode_step(int) per prompt token"},
            "gpu_launches": (n + 63) // 64}
    print(json.dumps(line), flush=True)


def run_batched(args, rank, world, dist):
    """64 independent sequences per GPU, positions drawn
    uniformly from 128..2048 (seeded per rank), KV caches pre-filled with seeded
    N(0,1) bf16; --steps batched steps with on-device token feedback.
    Multi-GPU: one replica per rank, no collective on the data path."""
    import megaqwen_b200 as mq
    B, L, K, W = 64, args.layers, args.steps, max(args.warmup, 3)
    shard = bool(args.vocab_shard) and world > 1
    g = torch.Generator().manual_seed(1000 + (0 if shard else rank))
    pos = torch.randint(128, 2049, (B,), generator=g)
    toks = torch.randint(0, 151936, (B,), generator=g)
    max_seq = 2048 + 2 * K + W + 8   # timed steps, then as many end-to-end steps
    dec = build_decoder(L, max_seq)
    bd = mq.BatchedDecoder(dec, B, max_seq, vocab_shard=(rank, world, dist, None) if shard else None)
    gk = torch.Generator(device="cuda").manual_seed(2000 + (0 if shard else rank))
    for b in range(B):
        bd.k_cache[b, :, :, :int(pos[b])].normal_(generator=gk)
        bd.v_cache[b, :, :, :int(pos[b])].normal_(generator=gk)
    bd.set_state(toks.tolist(), (pos - W).tolist())
    bd.step(W)
    torch.cuda.synchronize()
    bd.check_device()
    start = bd.positions.clone()
    stream = torch.cuda.current_stream()
    a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(int(os.environ.get("LOCAL_RANK", "0"))) as clk:
        a.record(stream)
        bd.step(K)
        b_.record(stream)
        torch.cuda.synchronize()
    ms = a.elapsed_time(b_)
    bd.check_device()
    t_max = max_over_ranks(ms, dist)
    # ---- end-to-end through the public API: host tokens in (pinned), host tokens out, every step ----
    host_in = torch.empty(B, dtype=torch.int32).pin_memory()
    host_out = torch.empty(B, dtype=torch.int32).pin_memory()
    host_in.copy_(bd.tokens.cpu())
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(K):
        bd.tokens.copy_(host_in, non_blocking=True)
        out = bd.step(1)
        host_out.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        host_in.copy_(host_out)
    e2e_s = max_over_ranks(time.perf_counter() - t0, dist)
    bd.check_device()
    c_sum = int((start + 1).sum()) * K + B * K * (K - 1) // 2
    alg = (BYTES_FIXED * K + BYTES_PER_POS * c_sum) / K
    peak, kind = measured_peak()
    ach = alg / ((ms / 1000.0) / K) / 1e9
    jobs = 1 if shard else world   # with a sharded LM head all ranks decode the same sequences
    line = {"metric": BATCHED_METRIC if not shard else
            "batched INT8 decode tok/s (64 sequences, LM head vocab-sharded over the GPUs)",
            "value": round(aggregate_tok_s(jobs, B * K, t_max / 1000.0), 1), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(t_max / K, 4), "higher_is_better": True, "scaling": "strong" if shard else "weak",
            "vs_baseline": None, "dtype": "int8-weights/fp16-activations/fp32-accum",
            "data": "synthetic (seeded weights, seeded N(0,1) KV caches)",
            "config": {"workload": "config4: batched decode, 64 sequences per GPU", "global_batch": world * B,
                       "parallelism": ("vocab-sharded LM head" if shard else "replicas") if world > 1 else "single"},
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "peak_kind": kind, "kernel": "batch_kernel",
                         "algorithmic_bytes_per_launch": int(alg)},
            "e2e": {"value": round(aggregate_tok_s(jobs, B * K, e2e_s), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B,
                    "api": "BatchedDecoder.step(1) with host token vectors copied in and out every step"},
            "clocks": clk.summary(), "gpu_launches": K}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample = cpu_oracle_batched_rate(threads)
        line["cpu_baseline"] = {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": sample}
    del bd, dec
    torch.cuda.empty_cache()
    return line


def cpu_oracle_batched_rate(threads, steps=2, pos=1088):
    """Batched tok/s of the CPU oracle: a CPU decodes the 64 sequences one after
    another, so its batched rate is 1 / (time of one sequence's step).  Sample:
    one 28-layer sequence at the mean config-4 position (1088) with a seeded
    N(0,1) bf16 KV cache, `steps` steps."""
    import megaqwen_b200 as mq
    from oracle import oracle as O
    torch.set_num_threads(threads)
    st = mq.make_synthetic_state(seed=0, num_layers=28)
    o = O.OracleDecoder(st, 28, max_seq_len=pos + steps + 1)
    g = torch.Generator().manual_seed(7)
    o.k_cache[:, :, :pos].normal_(generator=g)
    o.v_cache[:, :, :pos].normal_(generator=g)
    o.position = pos
    tok = 4242
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = o.decode_step(tok)
    v = steps / (time.perf_counter() - t0)
    return v, (f"{steps} steps of one sequence at positions {pos}..{pos + steps - 1} (seeded N(0,1) KV), 28 layers, "
               f"oracle/oracle.py on torch CPU ({threads} threads); batched tok/s = 1 / time per sequence step")


def cpu_oracle_long_rate(threads, ctx):
    """steps/s of the CPU oracle for one config-3 step at cache length ctx + 1."""
    import megaqwen_b200 as mq
    from oracle import oracle as O
    torch.set_num_threads(threads)
    st = mq.make_synthetic_state(seed=0, num_layers=28)
    o = O.OracleDecoder(st, 28, max_seq_len=ctx + 1)
    g = torch.Generator().manual_seed(ctx)
    o.k_cache[:, :, :ctx].normal_(generator=g)
    o.v_cache[:, :, :ctx].normal_(generator=g)
    o.position = ctx
    t0 = time.perf_counter()
    o.decode_step(11)
    return 1.0 / (time.perf_counter() - t0)


def cpu_oracle_rate(L, steps, threads, quantized=True):
    """tok/s of the CPU oracle (reference formulation) over `steps` steps at positions 0..steps-1."""
    import megaqwen_b200 as mq
    from oracle import oracle as O
    torch.set_num_threads(threads)
    st = mq.make_synthetic_state(seed=0, num_layers=L)
    o = O.OracleDecoder(st, L, max_seq_len=steps + 1, quantized=quantized)
    tok = 4242
    o.decode_step(tok)  # warm-up (position 0)
    o.reset()
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = o.decode_step(tok)
    return steps / (time.perf_counter() - t0)


def run_reference(args, rank, world, config):
    """Reference arm: the reference's PyTorch formulation (the oracle port) on the
    host cores, rank 0 only, on the same config, metric and unit as our arm."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    if config == 4:
        v, sample = cpu_oracle_batched_rate(threads)
        metric, workload = BATCHED_METRIC, "config4: batched decode, 64 sequences per GPU"
    else:
        n = max(1, min(args.steps, args.ref_sample_steps))
        v = cpu_oracle_rate(28, n, threads, quantized=config != 2)
        metric = METRIC.replace("INT8", "BF16") if config == 2 else METRIC
        workload = f"config{config}: Qwen3-0.6B batch-1 {'BF16' if config == 2 else 'INT8'} greedy decode, 28 layers"
        sample = f"{n} decode steps at positions 0..{n - 1}, 28 layers, oracle/oracle.py on torch CPU ({threads} threads)"
    line = {"impl": "reference", "metric": metric, "value": round(v, 3), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / v, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8-weights/fp32",
            "data": "synthetic", "config": {"workload": workload, "parallelism": "replicas"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_config0(args):
    """the dequant matvec of the six decoder-layer / LM-head
    shapes against an fp32 activation, on the host cores (the oracle's
    matvec_int8, i.e. the reference's PyTorch formulation) and on the GPU
    (mq_matvec, the same streaming kernel code as the decode step)."""
    import megaqwen_b200 as mq
    from megaqwen_b200 import _lib
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    shapes = {"qkv": (4096, 1024), "o": (1024, 2048), "gate": (3072, 1024), "up": (3072, 1024),
              "down": (1024, 3072), "lm_head": (151936, 1024)}
    peak, kind = measured_peak()
    rows, tot_cpu, tot_gpu, tot_bytes = {}, 0.0, 0.0, 0
    for name, (M, K) in shapes.items():
        w = (torch.randn(M, K, generator=g) * 0.02)
        w = torch.where(torch.rand(M, K, generator=g) < 0.001, w * 20, w).bfloat16()
        q, sc = O.quantize_per_channel(w)
        x = torch.randn(K, generator=g)
        qf = q.float()
        O.matvec_int8(x, q, sc)
        reps = 3 if M > 100000 else 20
        t0 = time.perf_counter()
        for _ in range(reps):
            y_cpu = (qf @ x) * sc      # the oracle's matvec on a pre-dequantised copy
        cpu_us = (time.perf_counter() - t0) / reps * 1e6
        qd, sd, xd = q.cuda(), sc.cuda(), x.cuda()
        yd = torch.empty(M, dtype=torch.float32, device="cuda")
        st = torch.cuda.current_stream()
        for _ in range(3):
            _lib.check(_lib.load().mq_matvec(0, qd.data_ptr(), sd.data_ptr(), xd.data_ptr(), yd.data_ptr(), M, K,
                                             st.cuda_stream), "mq_matvec")
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 50
        a.record(st)
        for _ in range(n):
            _lib.load().mq_matvec(0, qd.data_ptr(), sd.data_ptr(), xd.data_ptr(), yd.data_ptr(), M, K, st.cuda_stream)
        b.record(st)
        torch.cuda.synchronize()
        gpu_us = a.elapsed_time(b) / n * 1000.0
        err = O.rel_err(y_cpu, yd.cpu())
        by = M * K + 4 * M + 4 * (K + M)
        rows[name] = {"M": M, "K": K, "cpu_us": round(cpu_us, 1), "gpu_us": round(gpu_us, 2),
                      "gpu_gbs": round(by / gpu_us / 1e3, 1), "rel_err": err}
        tot_cpu += cpu_us
        tot_gpu += gpu_us
        tot_bytes += by
    ach = tot_bytes / tot_gpu / 1e3
    line = {"metric": "config0: dequant matvec time of the six layer / LM-head shapes", "value": round(tot_gpu, 2),
            "unit": "us (sum of the six shapes, GPU)", "higher_is_better": False, "n_gpus": 1,
            "dtype": "int8-weights/fp32-accum", "data": "synthetic (seed 0, N(0,0.02), 0.1% x20 outliers)",
            "config": {"workload": "config0: one decoder layer's matvecs + LM head"},
            "shapes": rows,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "peak_kind": kind, "kernel": "matvec_kernel<W8>",
                         "note": "each shape's weights fit in L2 except the LM head; back-to-back launches"},
            "cpu_baseline": {"value": round(tot_cpu, 1), "unit": "us (sum of the six shapes)", "cores": threads,
                             "kind": "port", "sample": "oracle matvec_int8 formulation, 20 reps per shape (3 for "
                                                       "the LM head), int8 codes pre-converted to fp32"}}
    print(json.dumps(line), flush=True)


def run_batch1(args, world, dist, local, bf16):
    """BASELINE configs 1 (INT8) and 2 (BF16): batch-1 greedy decode from position 0."""
    K, W, L = args.steps, args.warmup, args.layers
    max_seq = max(K, W, 200) + 8
    dec = build_decoder_bf16(L, max_seq) if bf16 else build_decoder(L, max_seq)
    stream = torch.cuda.current_stream()
    dec.reset()
    dec.decode_steps(4242, W)
    torch.cuda.synchronize()
    dec.check_device()
    # ---- device-resident timed region ----
    dec.reset()
    tok0 = torch.tensor([4242], dtype=torch.int32, device="cuda")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0.record(stream)
        toks = dec.decode_steps(tok0, K)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    dec.check_device()
    t_max = max_over_ranks(ms, dist)
    value = aggregate_tok_s(world, K, t_max / 1000.0)
    # ---- end-to-end through the reference-facing call ----
    dec.reset()
    dec.decode_step(4242)      # first call builds the step plan
    dec.reset()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok = 4242
    for _ in range(K):
        tok = dec.decode_step(tok)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, dist)
    e2e = aggregate_tok_s(world, K, e2e_s)
    # ---- per-position table in the reference's definition (bench_and_plot_int8.py:78-85:
    #      N decode_step calls from position 0, each with its host read-back; N / wall time) ----
    positions = {}
    for n in (1, 25, 50, 100, 200):
        dec.reset()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        tok = 4242
        for _ in range(n):
            tok = dec.decode_step(tok)
        positions[str(n)] = round(n / (time.perf_counter() - t0), 1)
    # ---- roofline of the decode kernel (one launch per step) ----
    peak, peak_kind = measured_peak()
    fixed = 1_192_101_888 if bf16 else BYTES_FIXED
    alg = sum(fixed + BYTES_PER_POS * (p + 1) for p in range(K)) / K
    achieved = alg / ((ms / 1000.0) / K) / 1e9
    metric = METRIC.replace("INT8", "BF16") if bf16 else METRIC
    cfg = 2 if bf16 else 1
    line = {"metric": metric, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(t_max / K, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16-weights/fp32-accum" if bf16 else "int8-weights/fp32-accum",
            "data": "synthetic (seeded N(0,0.02) bf16 weights, 0.1% x20 outliers)",
            "config": {"workload": f"config{cfg}: Qwen3-0.6B batch-1 {'BF16' if bf16 else 'INT8'} greedy decode, {L} layers",
                       "global_batch": world, "seq_len": K, "positions": f"0..{K - 1}",
                       "parallelism": "replicas" if world > 1 else "single",
                       "l2": "inputs larger than L2 (weights streamed every step)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": None if bf16 else ncu_traffic(),
                         "peak_kind": peak_kind,
                         "kernel": "decode_kernel<W16>" if bf16 else "decode_kernel<W8>",
                         "algorithmic_bytes_per_launch": int(alg)},
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                    "api": ("A10MegakernelDecoder" if bf16 else "A10Int8MegakernelDecoder") + ".decode_step(int) -> int"},
            "tok_s_at_position": positions,
            "tok_s_at_position_def": "N decode_step(int) calls from position 0 with the host read-back, N / wall time",
            "clocks": clk.summary(), "gpu_launches": K,
            "last_token": int(toks[-1].item())}
    if not args.no_cpu_baseline and world == 1:
        threads = os.cpu_count() or 1
        n = max(1, min(K, args.ref_sample_steps))
        v = cpu_oracle_rate(L, n, threads, quantized=not bf16)
        line["cpu_baseline"] = {"value": round(v, 3), "unit": "tok/s", "cores": threads, "kind": "port",
                                "sample": f"{n} steps at positions 0..{n - 1} of the same {L}-layer model, "
                                          f"oracle/oracle.py on torch CPU"}
    del dec
    torch.cuda.empty_cache()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=28)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-batched", action="store_true",
                    help="config 1 at N=1: skip the nested config-4 (batched) measurement")
    ap.add_argument("--ref-sample-steps", type=int, default=20)
    ap.add_argument("--ncu-case", action="store_true",
                    help="profiling case: --ncu-pos untimed steps, then 2 steps (capture with ncu -s <pos> -c 1)")
    ap.add_argument("--ncu-pos", type=int, default=10)
    ap.add_argument("--trace", action="store_true", help="print the per-phase timeline of one step at each --trace-pos")
    ap.add_argument("--trace-pos", default="10,200", help="comma-separated positions for --trace")
    ap.add_argument("--config", type=int, default=None, choices=[0, 1, 2, 3, 4],
                    help="BASELINE config: 0 matvec shapes, 1 INT8 batch-1 (default without torchrun), 2 BF16 "
                         "batch-1, 3 long context, 4 batched, 64 sequences per GPU (default under torchrun)")
    ap.add_argument("--context", type=str, default="4096,16384,32768",
                    help="config 3: comma-separated cached positions before the timed step")
    ap.add_argument("--vocab-shard", action="store_true",
                    help="config 4 under torchrun: every rank decodes the SAME 64 sequences and scores 1/N of the "
                         "vocabulary; one NCCL int64 max all-reduce per step picks the tokens")
    ap.add_argument("--prefill", type=int, default=0,
                    help="time the chunked prefill of a prompt of this many tokens (INT8, 28 layers) "
                         "against feeding it one decode step per token")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # Under torchrun the metric is the batched one (BASELINE: batched tok/s at
    # 1/2/4/8 GPUs); a plain single-process run measures the batch-1 headline.
    torchrun = "TORCHELASTIC_RUN_ID" in os.environ or world > 1
    config = args.config if args.config is not None else (4 if torchrun else 1)
    dist = None
    if world > 1:
        import torch.distributed as dist
        if args.impl == "ours":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo")
    if args.impl == "reference":
        run_reference(args, rank, world, config)
        if dist:
            dist.destroy_process_group()
        return
    args.warmup = max(args.warmup, 3)
    torch.cuda.set_device(local)
    from megaqwen_b200 import _lib
    if args.prefill:
        run_prefill(args)
        return
    if config == 0:
        run_config0(args)
        return
    if config == 3:
        for ctx in (int(x) for x in args.context.split(",")):
            run_long_context(args, ctx)
        return
    if config == 4:
        line = run_batched(args, rank, world, dist)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist:
            dist.destroy_process_group()
        return
    if args.trace:
        from megaqwen_b200 import trace
        tpos = [int(x) for x in args.trace_pos.split(",")]
        dec = build_decoder(args.layers, max(256, max(tpos) + 8))
        for p in tpos:
            dec.reset()
            if p > 256:       # long context: a zero cache of p positions times the same as a decoded one
                dec.set_position(p)
            elif p:
                dec.decode_steps(5, p)
            torch.cuda.synchronize()
            out = trace.summarize(trace.capture_step(dec), args.layers)
            out["position"] = p
            print(json.dumps(out), flush=True)
        dec.check_device()
        return
    if args.ncu_case:
        dec = build_decoder(args.layers, 256)
        dec.decode_steps(5, args.ncu_pos)
        torch.cuda.synchronize()
        dec.decode_steps(5, 2)
        torch.cuda.synchronize()
        dec.check_device()
        return
    line = run_batch1(args, world, dist, local, bf16=config == 2)
    if config == 1 and world == 1 and not args.no_batched:
        # The batched half of the BASELINE metric at N=1 (the N>1 points come from torchrun runs).
        b = run_batched(argparse.Namespace(**{**vars(args), "steps": min(args.steps, 20)}), rank, world, dist)
        line["batched"] = {k: b[k] for k in ("metric", "value", "unit", "ms_per_step", "steps", "roofline", "e2e",
                                             "cpu_baseline", "config", "gpu_launches") if k in b}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    _lib.device_status()


if __name__ == "__main__":
    main()
